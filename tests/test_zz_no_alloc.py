"""The allocation-free statistics entry point (``b2o_grad_stats_noalloc``).

Some hosts cannot hand this library any device memory for scratch: an FFI caller that only holds
pointers another runtime gave it, or a training process already at its memory ceiling.  For them
the library keeps the statistics scratch in one fixed array of its own.  These tests call that
entry point through the C ABI and check it against the workspace-based ``b2o_grad_stats`` on the
same inputs, on consecutive calls (the fixed array keeps the previous call's contents, so the
second call shows that nothing stale leaks through).

This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from minigpt_train_infra_b200 import _lib
from minigpt_train_infra_b200.plan import ChunkPlan, Entry, stream_ptr

RTOL = 1e-6


def _plan(device, grads, chunk_elems):
    dummy = torch.zeros(64, dtype=torch.float32, device=device)  # stats pass never touches it
    entries = [Entry(grad=g.data_ptr(), param=0, master=dummy.data_ptr(),
                     exp_avg=dummy.data_ptr(), exp_avg_sq=dummy.data_ptr(), numel=g.numel(),
                     group=0, slot=i) for i, g in enumerate(grads)]
    gd = _lib.BF16 if grads[0].dtype == torch.bfloat16 else _lib.F32
    return ChunkPlan(device, entries, 1, len(grads), gd, _lib.F32, chunk_elems), dummy


def _with_workspace(plan, n_slots, scale):
    out = torch.full((2,), -1.0, dtype=torch.float32, device=plan.device)
    exch = torch.zeros(n_slots + 1, dtype=torch.float64, device=plan.device)
    _lib.call("b2o_grad_stats", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr, plan.n_chunks,
              n_slots, plan.grad_dtype, scale.data_ptr(), plan.workspace.data_ptr(),
              exch.data_ptr(), _lib.STATS_CLEAR | _lib.STATS_FINALIZE, out.data_ptr(),
              out.data_ptr() + 4, stream_ptr(plan.device))
    return out


def _without_workspace(plan, n_slots, scale):
    out = torch.full((2,), -1.0, dtype=torch.float32, device=plan.device)
    _lib.call("b2o_grad_stats_noalloc", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr,
              plan.n_chunks, n_slots, plan.grad_dtype, scale.data_ptr(), out.data_ptr(),
              out.data_ptr() + 4, stream_ptr(plan.device))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(dtype):
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device).manual_seed(31)
    sizes = [1, 7, 4096, 100003, 1 << 20, 9]
    scale = torch.tensor(2.0 ** 14, dtype=torch.float32, device=device)
    calls = []
    for call in range(2):
        grads = [(torch.randn(n, generator=gen, device=device) * (1e-2 * (call + 1)) * 2.0 ** 14
                  ).to(dtype) for n in sizes]
        if call == 1:
            grads[3][777] = float("inf")
        plan, _keep = _plan(device, grads, chunk_elems=4096)
        ref = _with_workspace(plan, len(sizes), scale)
        got = _without_workspace(plan, len(sizes), scale)
        torch.cuda.synchronize()
        ref_h, got_h = ref.cpu().numpy(), got.cpu().numpy()
        calls.append((ref_h, got_h))
        assert got_h[0] == ref_h[0] == (1.0 if call == 1 else 0.0)
        if np.isfinite(ref_h[1]):
            assert abs(got_h[1] - ref_h[1]) <= RTOL * abs(ref_h[1])
            exact = float(torch.sqrt(sum((g.double() / 2.0 ** 14).pow(2).sum() for g in grads)))
            assert abs(got_h[1] - exact) <= RTOL * exact
        else:
            assert not np.isfinite(got_h[1]) and np.isnan(got_h[1]) == np.isnan(ref_h[1])
    assert calls[0][1][1] != calls[1][1][1]


def test_noalloc_rejects_plans_beyond_its_fixed_scratch():
    """Size limits are checked before any CUDA call, so this runs on a CPU-only host too."""
    lib = _lib.load()
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    c = np.zeros(1, dtype=_lib.CHUNK_DTYPE)
    out = np.zeros(2, dtype=np.float32)
    too_many_chunks = lib.b2o_grad_stats_noalloc(
        _lib.ptr(t), 1, _lib.ptr(c), _lib.NOALLOC_MAX_CHUNKS + 1, 1, _lib.BF16, None,
        _lib.ptr(out), _lib.ptr(out) + 4, None)
    too_many_slots = lib.b2o_grad_stats_noalloc(
        _lib.ptr(t), 1, _lib.ptr(c), 1, _lib.NOALLOC_MAX_SLOTS + 1, _lib.BF16, None,
        _lib.ptr(out), _lib.ptr(out) + 4, None)
    assert too_many_chunks == too_many_slots == _lib.ERR_TOO_LARGE
    assert b"fixed scratch" in lib.b2o_status_string(_lib.ERR_TOO_LARGE)

"""The allocation-free statistics entry point (``b2o_grad_stats_noalloc``).

Some hosts cannot hand this library any device memory for scratch: an FFI caller that only holds
pointers another runtime gave it, or a training process already at its memory ceiling.  For them
the library keeps the statistics scratch in one fixed array of its own.  These tests call that
entry point through the C ABI and check it against the workspace-based ``b2o_grad_stats`` on the
same inputs, on consecutive calls (the fixed array keeps the previous call's contents, so the
second call shows that nothing stale leaks through).  Both entry points run the same kernel with
the same fold order over the same tables, so their outputs must agree bit for bit; the norm is
also checked against an fp64 norm within a tolerance.

This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from minigpt_train_infra_b200 import _lib
from minigpt_train_infra_b200.plan import ChunkPlan, Entry, _plan_chunks, stream_ptr

RTOL = 1e-6  # kernel norm vs the fp64 norm


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


def _bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _fp64_norm(grads, scale: float) -> float:
    return float(torch.sqrt(sum((g.double() / scale).pow(2).sum() for g in grads)))


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
        assert np.array_equal(_bits(got_h), _bits(ref_h)), (got_h, ref_h)
        if np.isfinite(ref_h[1]):
            exact = _fp64_norm(grads, 2.0 ** 14)
            assert abs(got_h[1] - exact) <= RTOL * exact
    assert calls[0][1][1] != calls[1][1][1]


@pytest.mark.gpu
def test_noalloc_at_exactly_its_chunk_and_slot_limits():
    """A plan of exactly B2O_NOALLOC_MAX_CHUNKS chunks and B2O_NOALLOC_MAX_SLOTS slots, where
    the per-chunk partials and the per-slot sums reach the last byte of the fixed array: 4095
    one-element tensors plus one tensor cut into the remaining chunks of 8 elements."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    n_slots = _lib.NOALLOC_MAX_SLOTS
    big = (_lib.NOALLOC_MAX_CHUNKS - (n_slots - 1)) * 8
    gen = torch.Generator(device=device).manual_seed(77)
    scale = torch.tensor(2.0 ** 10, dtype=torch.float32, device=device)
    for call in range(2):
        flat = (torch.randn(n_slots - 1 + big, generator=gen, device=device) * 2.0 ** 10
                ).to(torch.bfloat16)
        grads = [flat[i:i + 1] for i in range(n_slots - 1)] + [flat[n_slots - 1:]]
        plan, _keep = _plan(device, grads, chunk_elems=8)
        assert plan.n_chunks == _lib.NOALLOC_MAX_CHUNKS and plan.n_tensors == n_slots
        ref = _with_workspace(plan, n_slots, scale)
        got = _without_workspace(plan, n_slots, scale)
        torch.cuda.synchronize()
        ref_h, got_h = ref.cpu().numpy(), got.cpu().numpy()
        assert got_h[0] == ref_h[0] == 0.0
        assert np.array_equal(_bits(got_h), _bits(ref_h)), (call, got_h, ref_h)
        exact = _fp64_norm([flat], 2.0 ** 10)
        assert abs(got_h[1] - exact) <= RTOL * exact


@pytest.mark.gpu
def test_noalloc_in_a_driver_context_of_the_callers_own():
    """A host that is not a runtime-API program may run in a CUDA context it created itself
    rather than the device's primary context.  The fixed array has a different address in each
    context, so the entry point must use the copy of the context current at the call.  This
    runs it in the primary context, then in a context made with cuCtxCreate (all buffers
    allocated in that context), then in the primary context again, and compares every result
    with the workspace entry point bit for bit."""
    from cuda.bindings import driver as cu

    def ok(res):
        err = res[0] if isinstance(res, tuple) else res
        assert err == cu.CUresult.CUDA_SUCCESS, err
        return res[1] if isinstance(res, tuple) and len(res) == 2 else None

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    lib = _lib.load()
    gen = torch.Generator(device=device).manual_seed(5)
    sizes = [3, 4096, 70001, 1 << 18]
    grads = [(torch.randn(n, generator=gen, device=device) * 0.03 * 256.0).to(torch.bfloat16)
             for n in sizes]
    scale = torch.tensor(256.0, dtype=torch.float32, device=device)
    plan, _keep = _plan(device, grads, chunk_elems=4096)
    ref = _with_workspace(plan, len(sizes), scale)
    first = _without_workspace(plan, len(sizes), scale)
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    assert np.array_equal(_bits(first.cpu().numpy()), _bits(ref_h))

    # the same gradients and tables in a context of our own
    host_g = [g.view(torch.int16).cpu().numpy() for g in grads]
    ok(cu.cuInit(0))
    dev = ok(cu.cuDeviceGet(0))
    ctx = ok(cu.cuCtxCreate(0, dev))
    allocs = []
    try:
        def alloc(nbytes):
            p = int(ok(cu.cuMemAlloc(max(int(nbytes), 16))))
            allocs.append(p)
            return p

        def upload(arr):
            arr = np.ascontiguousarray(arr)
            p = alloc(arr.nbytes)
            ok(cu.cuMemcpyHtoD(p, arr.ctypes.data, arr.nbytes))
            return p

        gptr = [upload(h) for h in host_g]
        dummy = alloc(256)
        host_t = np.zeros(len(sizes), dtype=_lib.TENSOR_DTYPE)
        for i, (p, n) in enumerate(zip(gptr, sizes)):
            host_t[i] = (p, 0, dummy, dummy, dummy, n, 0, i, 0, 0, 0, 0)
        host_c = _plan_chunks(lib, host_t, 1, len(sizes), 4096, _lib.BF16)
        t_dev, c_dev = upload(host_t), upload(host_c)
        s_dev = upload(np.array([256.0], dtype=np.float32))
        results = []
        for _ in range(2):
            out_dev = upload(np.full(2, -1.0, dtype=np.float32))
            st = lib.b2o_grad_stats_noalloc(t_dev, len(sizes), c_dev, len(host_c), len(sizes),
                                            _lib.BF16, s_dev, out_dev, out_dev + 4, None)
            assert st == 0, lib.b2o_status_string(st)
            ok(cu.cuCtxSynchronize())
            out = np.zeros(2, dtype=np.float32)
            ok(cu.cuMemcpyDtoH(out.ctypes.data, out_dev, 8))
            results.append(out)
        for out in results:
            assert np.array_equal(_bits(out), _bits(ref_h)), (out, ref_h)
    finally:
        for p in allocs:
            cu.cuMemFree(p)
        cu.cuCtxDestroy(ctx)

    # back in the primary context: the cached address of the primary context's copy
    torch.cuda.set_device(device)
    again = _without_workspace(plan, len(sizes), scale)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(again.cpu().numpy()), _bits(ref_h))


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

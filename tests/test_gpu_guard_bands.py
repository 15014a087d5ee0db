"""Out-of-bounds detection without a sanitizer: every tensor the kernels touch sits between guard
bands of a sentinel bit pattern, and the step is run through the C ABI.

* A write outside any tensor changes a guard band (checked bit for bit after the step).
* A gradient read outside any tensor reads the sentinel, a bf16 NaN, and raises the non-finite
  flag (checked: the flag stays 0 and the norm is finite).
* Every in-bounds value must equal the oracle given the kernel's norm (bit for bit).

Sizes cover the ragged cases of the planner and both kernel paths: empty, 1, 7, 9 and 65
elements, 4097, 2**20 + 3, a tensor spanning many statistics chunks, and views moved off the
16-byte boundary (scalar path).  Chunk sizes: the defaults and 64 elements.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import adamw_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

GUARD = 256                    # elements of sentinel before and after every tensor
F32_SENTINEL = 0x7FC0DEAD      # a quiet fp32 NaN with a payload
BF16_SENTINEL = 0x7FC1         # a bf16 NaN
SIZES = [1, 7, 0, 9, 4097, 65, (1 << 20) + 3, 300_001]
MISALIGNED = {3, 5}            # tensors whose views start one element past a 16-byte boundary


def _layout(sizes, misaligned):
    """Offsets (elements) of every tensor inside one guard-banded buffer, 16-byte aligned
    (a multiple of 8 elements) except the misaligned ones, which start one element later."""
    offs, pos = [], GUARD
    for i, n in enumerate(sizes):
        start = pos + (1 if i in misaligned else 0)
        offs.append(start)
        pos = (start + n + GUARD + 7) // 8 * 8
    return offs, pos + GUARD


def _guarded(total, dtype, sentinel):
    # both sentinels are positive in the signed integer view of their width
    t = torch.empty(total, dtype=dtype, device=DEV)
    t.view(torch.int32 if dtype == torch.float32 else torch.int16).fill_(sentinel)
    return t


def _bits(t):
    return t.view(torch.int32 if t.dtype == torch.float32 else torch.int16).cpu().numpy()


@pytest.mark.parametrize("grad_kind", ["bf16", "f32"])
@pytest.mark.parametrize("chunk_elems", [None, 64])
def test_kernels_stay_inside_their_tensors(chunk_elems, grad_kind):
    """bf16: bf16 gradients and parameters with fp32 masters; f32: fp32 gradients and fp32
    parameters (the master is the parameter), the reference's own configuration."""
    from minigpt_train_infra_b200 import _lib
    from minigpt_train_infra_b200.plan import ChunkPlan, Entry, stream_ptr
    offs, total = _layout(SIZES, MISALIGNED)
    bf16 = grad_kind == "bf16"
    grad = _guarded(total, torch.bfloat16, BF16_SENTINEL) if bf16 else \
        _guarded(total, torch.float32, F32_SENTINEL)
    param = _guarded(total, torch.bfloat16, BF16_SENTINEL)
    master, m, v = (_guarded(total, torch.float32, F32_SENTINEL) for _ in range(3))
    gen = torch.Generator().manual_seed(11)
    scale = 2.0 ** 12
    host = []
    for i, (o, n) in enumerate(zip(offs, SIZES)):
        w0 = torch.randn(n, generator=gen) * 0.02
        m0 = torch.randn(n, generator=gen) * 1e-3
        v0 = torch.randn(n, generator=gen).abs() * 1e-6
        g0 = torch.randn(n, generator=gen) * 0.05 * scale
        if bf16:
            g0 = g0.to(torch.bfloat16)
        master[o:o + n] = w0.to(DEV)
        m[o:o + n] = m0.to(DEV)
        v[o:o + n] = v0.to(DEV)
        param[o:o + n] = w0.to(torch.bfloat16).to(DEV)
        grad[o:o + n] = g0.to(DEV)
        host.append((w0.numpy(), m0.numpy(), v0.numpy(),
                     O.bf16_bits_to_f32(g0.view(torch.int16).numpy().view(np.uint16)) if bf16
                     else g0.numpy()))
    before = {k: _bits(t) for k, t in
              (("grad", grad), ("param", param), ("master", master), ("m", m), ("v", v))}

    def addr(t, o):
        return t.data_ptr() + o * t.element_size()

    gd = _lib.BF16 if bf16 else _lib.F32
    entries = [Entry(addr(grad, o), addr(param, o) if bf16 else 0, addr(master, o), addr(m, o),
                     addr(v, o), n, i % 2, i) for i, (o, n) in enumerate(zip(offs, SIZES))]
    plan = ChunkPlan(DEV, entries, 2, len(SIZES), gd, gd, chunk_elems)
    groups = np.zeros(2, dtype=_lib.GROUP_DTYPE)
    groups[0] = (1e-3, 0.9, 0.95, 1e-8, 0.1)
    groups[1] = (3e-4, 0.9, 0.95, 1e-8, 0.0)
    steps = torch.full((len(SIZES),), 4.0, device=DEV)
    ls = torch.tensor([scale], dtype=torch.float32, device=DEV)
    out = torch.zeros(2, dtype=torch.float32, device=DEV)
    stream = stream_ptr(DEV)
    _lib.call("b2o_grad_stats", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr,
              plan.n_chunks, len(SIZES), gd, ls.data_ptr(), plan.workspace.data_ptr(),
              None, _lib.STATS_CLEAR | _lib.STATS_FINALIZE, out.data_ptr(),
              out.data_ptr() + 4, stream)
    _lib.call("b2o_adamw_step", plan.tensors_ptr, plan.n_tensors, plan.update_chunks_ptr,
              plan.n_update_chunks, _lib.ptr(groups), 2, gd, gd,
              steps.data_ptr(), out.data_ptr(), ls.data_ptr(), out.data_ptr() + 4, 1.0, None,
              plan.workspace.data_ptr(), stream)
    torch.cuda.synchronize()
    found, norm = (float(x) for x in out.cpu())
    assert found == 0.0, "a gradient read left its tensor (read the NaN sentinel)"
    assert np.isfinite(norm)
    assert plan.vector_fraction() < 1.0  # the misaligned views took the scalar path

    after = {k: _bits(t) for k, t in
             (("grad", grad), ("param", param), ("master", master), ("m", m), ("v", v))}
    inside = np.zeros(total, dtype=bool)
    for o, n in zip(offs, SIZES):
        inside[o:o + n] = True
    for k in before:
        assert np.array_equal(before[k][~inside], after[k][~inside]), f"write outside: {k}"
    assert np.array_equal(before["grad"], after["grad"]), "gradients must be read-only"

    # in-bounds values: the oracle given the kernel's norm, bit for bit
    hp = [O.GroupHP(1e-3, 0.9, 0.95, 1e-8, 0.1), O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.0)]
    states = [O.TensorState(w=w.copy(), m=mm.copy(), v=vv.copy(), group=i % 2, step=4.0)
              for i, (w, mm, vv, _) in enumerate(host)]
    grads = [g for _, _, _, g in host]
    sc = O.ScalerState(scale=np.float32(scale))
    O.optimizer_step(states, grads, hp, sc, 1.0, norm=np.float32(norm))
    f32 = {k: after[k].view(np.float32) for k in ("master", "m", "v")}
    p16 = after["param"].view(np.uint16)
    for st, o, n in zip(states, offs, SIZES):
        np.testing.assert_array_equal(f32["master"][o:o + n], st.w)
        np.testing.assert_array_equal(f32["m"][o:o + n], st.m)
        np.testing.assert_array_equal(f32["v"][o:o + n], st.v)
        if bf16:
            np.testing.assert_array_equal(p16[o:o + n], O.f32_to_bf16_bits(st.w))
    np.testing.assert_array_equal(steps.cpu().numpy(), np.full(len(SIZES), 5.0, np.float32))

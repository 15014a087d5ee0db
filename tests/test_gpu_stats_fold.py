"""The final fold of the statistics pass, at plan shapes that reach every branch of it.

The CTA that finishes ``grad_stats_kernel`` last folds each tensor's chunk partials (one fp64 sum
of squares per chunk) into ``exch[slot]``.  It takes the tensor table in blocks of 256 tensors and
stages each block's partials in shared memory 4096 at a time; a tensor's piece of such a window is
summed by one thread when it holds at most 128 partials and by a warp when it holds more, and a
tensor whose chunks span windows adds its windows' sums in window order.  Realistic plans (64 Ki
or 128 Ki elements per chunk) reach only some of these branches at test sizes, so these cases plan
8-element chunks: a few hundred thousand elements then make tens of thousands of partials, with
tensors that span one, two and three windows, pieces of every length around the 128 boundary,
ragged tensor ends, two table blocks, and empty tensors at the first and last place of each block.

Checked through the C ABI (``b2o_grad_stats``): every ``exch[slot]`` against the fp64 sum of the
unscaled squares (slots permuted, so a wrong slot shows), the norm against the two-level norm of
the fp64 sums, the non-finite count, and that a second call gives the same bits.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from minigpt_train_infra_b200 import _lib
from minigpt_train_infra_b200.plan import ChunkPlan, Entry, stream_ptr

RTOL = 1e-6      # per-tensor sums and the norm vs fp64: eight-element fp32 chains, then fp64
CHUNK = 8        # elements per chunk: one partial per vector
SCALE = 2.0 ** 12

# Chunk counts of the tensors between the fixed ones below: every piece length around the
# thread/warp boundary (128) and the window size (4096), plus small ones.
_COUNTS = [1, 2, 3, 31, 32, 33, 127, 128, 129, 255, 256, 257, 1000, 4095, 4096, 4097, 8193]


def _numels() -> list[int]:
    rng = np.random.default_rng(11)
    n = [0, 8 * 4096 * 2 + 40]                              # empty first; spans three windows
    n += [CHUNK * c for c in _COUNTS]
    n += [5, 13, 8 * 130 + 3, 8 * 4096 + 1]                 # ragged tensor ends
    while len(n) < 255:
        n.append(int(rng.integers(1, 41)) * CHUNK - int(rng.integers(0, 8)))
    n += [0, 0, 8 * 5000]                                   # empty last of block 0 and first of
    while len(n) < 299:                                     # block 1; a tensor spanning windows
        n.append(int(rng.integers(1, 200)) * CHUNK)         # in block 1
    n.append(0)                                             # empty last of block 1
    return n


def _run(grads, slots, n_slots, dtype):
    dev = grads[0].device
    dummy = torch.zeros(64, dtype=torch.float32, device=dev)  # the statistics pass never reads it
    entries = [Entry(grad=g.data_ptr(), param=0, master=dummy.data_ptr(),
                     exp_avg=dummy.data_ptr(), exp_avg_sq=dummy.data_ptr(), numel=g.numel(),
                     group=0, slot=int(s)) for g, s in zip(grads, slots)]
    gd = _lib.BF16 if dtype == torch.bfloat16 else _lib.F32
    plan = ChunkPlan(dev, entries, 1, n_slots, gd, _lib.F32, CHUNK)
    scale = torch.tensor(SCALE, dtype=torch.float32, device=dev)
    outs = []
    for _ in range(2):
        out = torch.full((2,), -1.0, dtype=torch.float32, device=dev)
        exch = torch.full((n_slots + 1,), -7.0, dtype=torch.float64, device=dev)
        _lib.call("b2o_grad_stats", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr,
                  plan.n_chunks, n_slots, gd, scale.data_ptr(), plan.workspace.data_ptr(),
                  exch.data_ptr(), _lib.STATS_CLEAR | _lib.STATS_FINALIZE, out.data_ptr(),
                  out.data_ptr() + 4, stream_ptr(dev))
        outs.append((exch.cpu().numpy(), out.cpu().numpy()))
    torch.cuda.synchronize(dev)
    return plan, outs


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fold_matches_fp64_sums_at_every_branch(dtype):
    dev = torch.device("cuda", 0)
    numels = _numels()
    gen = torch.Generator(device=dev).manual_seed(5)
    grads = [(torch.randn(n, generator=gen, device=dev) * SCALE * 1e-3).to(dtype) for n in numels]
    n_slots = len(grads) + 3                       # slots no tensor uses stay cleared
    slots = np.random.default_rng(3).permutation(n_slots)[:len(grads)]
    plan, outs = _run(grads, slots, n_slots, dtype)
    assert plan.n_tensors == 300 and plan.n_chunks > 3 * 4096

    ref = np.zeros(n_slots, dtype=np.float64)
    for g, s in zip(grads, slots):
        ref[s] = float((g.double() / SCALE).pow(2).sum()) if g.numel() else 0.0
    exch, out = outs[0]
    assert exch[n_slots] == 0.0 and out[0] == 0.0            # nothing non-finite
    np.testing.assert_allclose(exch[:n_slots], ref, rtol=RTOL, atol=0.0)
    for s in set(range(n_slots)) - set(int(x) for x in slots):
        assert exch[s] == 0.0
    # the two-level norm of clip_grad.py:_get_total_norm over the fp64 sums
    per_tensor = np.sqrt(ref).astype(np.float32).astype(np.float64)
    norm = float(np.sqrt(np.dot(per_tensor, per_tensor)))
    assert abs(float(out[1]) - norm) <= RTOL * norm, (out[1], norm)
    # same plan, same inputs: the same bits
    exch2, out2 = outs[1]
    assert np.array_equal(exch.view(np.uint64), exch2.view(np.uint64))
    assert np.array_equal(out.view(np.uint32), out2.view(np.uint32))


@pytest.mark.gpu
def test_fold_counts_a_non_finite_gradient_in_the_second_table_block():
    dev = torch.device("cuda", 0)
    numels = _numels()
    gen = torch.Generator(device=dev).manual_seed(6)
    grads = [torch.randn(n, generator=gen, device=dev).to(torch.bfloat16) for n in numels]
    grads[257][4321] = float("inf")
    slots = np.arange(len(grads))
    _, outs = _run(grads, slots, len(grads), torch.bfloat16)
    for exch, out in outs:
        assert exch[len(grads)] == 1.0 and out[0] == 1.0
        assert not np.isfinite(exch[257])

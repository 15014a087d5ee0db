"""The kernel's gradient norm and clip coefficient against torch's CUDA ``clip_grad_norm_``.

On a GPU the reference's loop clips with ``torch.nn.utils.clip_grad_norm_`` over CUDA gradients
(``train.py:486``; AdamW is built with ``fused=True`` there, ``train.py:364`` and
``runtime.py:164``).  That norm is torch's ``_get_total_norm`` (``clip_grad.py:50-118``): a
``_foreach_norm`` per tensor on the GPU, then the norm of the stacked per-tensor norms; the
coefficient is ``clamp(max_norm / (norm + 1e-6), max=1)`` (``clip_grad.py:165-169``).  Its
accumulation order differs from the statistics kernel's (fp64 chunk partials folded in chunk
order), so the two agree to rounding, not bit for bit.  This test measures the difference at
BASELINE configs 2-5 on the same seeded gradients -- bf16 values times the loss scale, unscaled
exactly (the scales are powers of two) into the fp32 gradients torch's path would hold -- and
checks that both are within 1e-6 relative of an fp64 norm.  The measured differences are printed
(``pytest -s``).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from minigpt_train_infra_b200 import _lib, workloads
from minigpt_train_infra_b200.plan import ChunkPlan, Entry, stream_ptr
from oracle import adamw_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
CONFIGS = {  # workload, gradient std, loss scale
    2: ("flat_2_28", 1e-2, 2.0 ** 16),
    3: ("gpt2_124m", 1e-3, 2.0 ** 16),
    4: ("qwen3_1_7b", 1e-3, 2.0 ** 16),
    5: ("qwen3_8b", 1e-3, 2.0 ** 15),
}
REL_TOL = 1e-6


def _kernel_norm(grads, scale: float) -> float:
    """The statistics kernel's norm over ``grads`` (bf16, scaled), through the C ABI."""
    dummy = torch.zeros(64, dtype=torch.float32, device=DEV)  # the pass reads gradients only
    entries = [Entry(grad=g.data_ptr(), param=0, master=dummy.data_ptr(),
                     exp_avg=dummy.data_ptr(), exp_avg_sq=dummy.data_ptr(), numel=g.numel(),
                     group=0, slot=i) for i, g in enumerate(grads)]
    plan = ChunkPlan(DEV, entries, 1, len(grads), _lib.BF16, _lib.F32)
    out = torch.empty(2, dtype=torch.float32, device=DEV)
    exch = torch.zeros(len(grads) + 1, dtype=torch.float64, device=DEV)
    ls = torch.tensor(scale, dtype=torch.float32, device=DEV)
    _lib.call("b2o_grad_stats", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr, plan.n_chunks,
              len(grads), _lib.BF16, ls.data_ptr(), plan.workspace.data_ptr(), exch.data_ptr(),
              _lib.STATS_CLEAR | _lib.STATS_FINALIZE, out.data_ptr(), out.data_ptr() + 4,
              stream_ptr(DEV))
    torch.cuda.synchronize()
    assert float(out[0]) == 0.0
    return float(out[1])


def _torch_cuda_norm(grads, scale: float) -> tuple[float, float]:
    """torch's CUDA norm and clip coefficient over the fp32 gradients the reference would hold
    (bf16 upcast, times 1/scale: exact), as clip_grad_norm_ computes them."""
    g32 = [g.float().mul_(1.0 / scale) for g in grads]
    norm = torch.nn.utils.get_total_norm(g32, 2.0, False, None)
    coef = torch.clamp(1.0 / (norm + 1e-6), max=1.0)  # python float / tensor, clip_grad.py:165
    out = float(norm), float(coef)
    del g32
    torch.cuda.empty_cache()
    return out


def _fp64_norm(grads, scale: float, piece: int = 1 << 26) -> float:
    total = 0.0
    for g in grads:
        flat = g.view(-1)
        acc = 0.0
        for a in range(0, flat.numel(), piece):
            x = flat[a:a + piece].double() / scale
            acc += float((x * x).sum())
        total += acc
    return math.sqrt(total)


@pytest.mark.parametrize("config", sorted(CONFIGS))
def test_kernel_norm_vs_torch_cuda_clip(config):
    name, std, scale = CONFIGS[config]
    torch.cuda.empty_cache()
    gen = torch.Generator(device=DEV).manual_seed(100 + config)
    grads = []
    for _, shape, _ in workloads.shapes(name):
        g = torch.empty(shape, dtype=torch.bfloat16, device=DEV)
        flat = g.view(-1)
        for a in range(0, flat.numel(), 1 << 27):
            part = flat[a:a + (1 << 27)]
            part.copy_(torch.randn(part.numel(), generator=gen, device=DEV) * std * scale)
        grads.append(g)
    ours = _kernel_norm(grads, scale)
    theirs, theirs_coef = _torch_cuda_norm(grads, scale)
    exact = _fp64_norm(grads, scale)
    ours_coef = float(O.clip_coefficient(np.float32(ours), 1.0))
    rel_norm = abs(ours - theirs) / theirs
    rel_coef = abs(ours_coef - theirs_coef) / theirs_coef
    print(f"\nconfig {config} ({name}, {sum(g.numel() for g in grads):,} params): kernel norm "
          f"{ours!r}, torch CUDA norm {theirs!r}, fp64 {exact!r}; relative difference "
          f"{rel_norm:.3e} (kernel vs fp64 {abs(ours - exact) / exact:.3e}, torch vs fp64 "
          f"{abs(theirs - exact) / exact:.3e}); clip coefficient {ours_coef!r} vs "
          f"{theirs_coef!r}, relative difference {rel_coef:.3e}")
    assert abs(ours - exact) <= REL_TOL * exact
    assert abs(theirs - exact) <= REL_TOL * exact
    assert rel_norm <= 2 * REL_TOL and rel_coef <= 2 * REL_TOL
    del grads
    torch.cuda.empty_cache()

"""Numpy restatement of the reference's mixed-precision optimizer step (CPU oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Nothing in the product imports this.

The reference (``train.py:485-491``) runs, once per optimizer step::

    scaler.unscale_(optimizer)                       # torch/amp/grad_scaler.py:302-361
    clip_grad_norm_(model.parameters(), grad_clip)   # torch/nn/utils/clip_grad.py:186
    scaler.step(optimizer)                           # torch/amp/grad_scaler.py:375-482
    scaler.update()                                  # torch/amp/grad_scaler.py:484-560

with ``optimizer = torch.optim.AdamW(build_adamw_param_groups(...))`` (``train.py:359-365``,
``src/minigpt/optim.py:15-64``).  The arithmetic lives in PyTorch (third party, not vendored;
the reference pins ``torch>=2.8`` in ``requirements.txt:1``; this restatement was checked
against torch 2.11.0).  Every function below cites the torch line it follows and states the
fp32 rounding sequence that torch's CPU kernels apply, which was established by comparing
against torch on this container's CPU:

* scalar arguments that Python computes in double are rounded to fp32 before the tensor op;
* ``Tensor.lerp_(end, w)`` with ``w < 0.5`` is ``fma(w, end - self, self)`` (one rounding
  for the product-and-add), with ``w >= 0.5`` it is ``fma(w - 1, end - self, end)``;
* ``Tensor.addcmul_(t1, t2, value=c)`` is ``fma(c * t1, t2, self)``;
* ``Tensor.addcdiv_(t1, t2, value=c)`` is ``self + (c * t1) / t2`` with three roundings;
* ``Tensor / python_float`` is a true fp32 division;
* ``python_float / Tensor`` is ``Tensor.reciprocal() * python_float`` (torch/_tensor.py
  ``__rdiv__``).

Two places where this restatement deliberately differs from torch's CPU build:

* ``Tensor.sqrt`` on an AVX512 host is faithfully but not always correctly rounded (about
  0.6% of fp32 inputs come out one ulp away); the oracle (and the CUDA kernel) use the IEEE
  correctly rounded square root.
* torch's CPU L2 norm (``_foreach_norm`` / ``linalg.vector_norm`` on fp32) accumulates in
  fp32 and loses accuracy on large tensors (measured relative error -1.0e-5 at 1e6 elements,
  -3.1e-4 at 1e7, -4.3e-2 at 2**28).  The oracle computes each per-tensor norm as the fp32
  rounding of the exact root-sum-of-squares (accumulated in fp64), then combines the fp32
  per-tensor norms exactly as ``_get_total_norm`` does (``clip_grad.py:96,106``).  Where a
  test needs the reference's own (inexact) norm it passes it in through ``norm=``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

F32 = np.float32
F64 = np.float64


# --------------------------------------------------------------------------------------------
# bf16 helpers (storage is uint16 bit patterns; torch.bfloat16 has no numpy dtype)
# --------------------------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns to fp32 (the ``.float()`` of a bf16 tensor)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even narrowing of fp32 to bf16 bits (``Tensor.to(torch.bfloat16)``).

    NaN maps to a quiet NaN with the sign kept; only NaN-ness is compared by the tests.
    """
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        out = out.copy()
        out[nan] = (((u[nan] >> 16) & 0x8000) | 0x7FC0).astype(np.uint16)
    return out


# --------------------------------------------------------------------------------------------
# exact fp32 fused multiply-add
# --------------------------------------------------------------------------------------------

def fma32(a, b, c) -> np.ndarray:
    """Correctly rounded fp32 ``a*b + c``.

    ``a*b`` of two fp32 values is exact in fp64.  The fp64 sum ``s = fl(p + c)`` can round, so
    the exact error ``e`` is recovered with Knuth's TwoSum and ``s`` is replaced by its
    round-to-odd neighbour when ``e != 0``; rounding a round-to-odd fp64 value (53 bits) to
    fp32 (24 bits) is then correctly rounded because 53 >= 24 + 2 (Boldo and Melquiond,
    "Emulation of FMA and correctly rounded sums: proved algorithms using rounding to odd",
    IEEE TC 2008).
    """
    a = np.asarray(a, dtype=F32).astype(F64)
    b = np.asarray(b, dtype=F32).astype(F64)
    c = np.asarray(c, dtype=F32).astype(F64)
    p = a * b
    with np.errstate(invalid="ignore", over="ignore"):
        s = p + c
        bp = s - c
        ap = s - bp
        e = (p - ap) + (c - bp)
        mant_even = (s.view(np.int64) & 1) == 0
        fix = (e != 0) & mant_even & np.isfinite(s)
        if np.any(fix):
            s = np.where(fix, np.nextafter(s, s + e), s)
    return s.astype(F32)


# --------------------------------------------------------------------------------------------
# unscale + inf check + norm + clip coefficient
# --------------------------------------------------------------------------------------------

def inv_scale_of(scale: float) -> np.float32:
    """``self._scale.double().reciprocal().float()`` (grad_scaler.py:351-355)."""
    return F32(1.0 / float(F64(F32(scale))))


def nonfinite_any(grads: Sequence[np.ndarray]) -> bool:
    """``found_inf`` of ``_amp_foreach_non_finite_check_and_unscale_``: any non-finite input."""
    return any(not np.all(np.isfinite(g)) for g in grads)


def unscale(g: np.ndarray, inv_scale: np.float32) -> np.ndarray:
    """``g *= inv_scale`` in fp32 (grad_scaler.py:294-298)."""
    with np.errstate(over="ignore", invalid="ignore"):
        return (np.asarray(g, dtype=F32) * F32(inv_scale)).astype(F32)


def tensor_norm(x: np.ndarray) -> np.float32:
    """fp32 rounding of the exact L2 norm of one tensor (see module docstring)."""
    x64 = np.asarray(x, dtype=F32).astype(F64).ravel()
    with np.errstate(over="ignore", invalid="ignore"):
        return F32(math.sqrt(float(np.dot(x64, x64)))) if x64.size else F32(0.0)


def total_norm(norms: Sequence[np.float32]) -> np.float32:
    """``vector_norm(stack(norms))`` of the per-tensor fp32 norms (clip_grad.py:106)."""
    n64 = np.asarray(norms, dtype=F32).astype(F64)
    with np.errstate(over="ignore", invalid="ignore"):
        return F32(math.sqrt(float(np.dot(n64, n64)))) if n64.size else F32(0.0)


def clip_coefficient(norm: np.float32, max_norm: float) -> np.float32:
    """``clamp(max_norm / (total_norm + 1e-6), max=1.0)`` (clip_grad.py:165,169).

    ``total_norm + 1e-6`` is an fp32 add, ``max_norm / t`` is ``t.reciprocal() * max_norm`` and
    ``clamp`` keeps a NaN coefficient NaN.
    """
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        t = F32(F32(norm) + F32(1e-6))
        coef = F32(F32(F32(1.0) / t) * F32(max_norm))
    return coef if (np.isnan(coef) or coef <= F32(1.0)) else F32(1.0)


# --------------------------------------------------------------------------------------------
# AdamW (decoupled weight decay), torch/optim/adam.py:_single_tensor_adam
# --------------------------------------------------------------------------------------------

@dataclass
class GroupHP:
    lr: float
    beta1: float
    beta2: float
    eps: float
    weight_decay: float


def adamw_scalars(hp: GroupHP, step: float) -> dict:
    """Host-double scalars of one AdamW step at (post-increment) ``step`` (adam.py:529-536)."""
    bc1 = 1.0 - hp.beta1 ** step
    bc2 = 1.0 - hp.beta2 ** step
    step_size = hp.lr / bc1
    return {
        "decay": F32(1.0 - hp.lr * hp.weight_decay),
        "w1": F32(1.0 - hp.beta1),
        "beta2": F32(hp.beta2),
        "omb2": F32(1.0 - hp.beta2),
        "bc2_sqrt": F32(bc2 ** 0.5),
        "neg_step_size": F32(-step_size),
        "eps": F32(hp.eps),
    }


def adamw_update(w: np.ndarray, m: np.ndarray, v: np.ndarray, g: np.ndarray,
                 hp: GroupHP, step: float) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """One AdamW element update at post-increment ``step``; returns new (w, m, v).

    Follows adam.py:416-419 (``param.mul_(1 - lr*wd)``), :457 (``exp_avg.lerp_``),
    :476 (``exp_avg_sq.mul_(beta2).addcmul_``), :531-545 (bias corrections and ``denom``) and
    :547 (``param.addcdiv_``) with the fp32 rounding sequence stated in the module docstring.
    """
    s = adamw_scalars(hp, step)
    w = np.asarray(w, dtype=F32)
    m = np.asarray(m, dtype=F32)
    v = np.asarray(v, dtype=F32)
    g = np.asarray(g, dtype=F32)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        if hp.weight_decay != 0:
            w = (w * s["decay"]).astype(F32)
        diff = (g - m).astype(F32)
        if s["w1"] < F32(0.5):
            m = fma32(s["w1"], diff, m)
        else:
            m = fma32(F32(s["w1"] - F32(1.0)), diff, g)
        v = (v * s["beta2"]).astype(F32)
        v = fma32((s["omb2"] * g).astype(F32), g, v)
        denom = (np.sqrt(v) / s["bc2_sqrt"]).astype(F32)
        denom = (denom + s["eps"]).astype(F32)
        upd = ((s["neg_step_size"] * m).astype(F32) / denom).astype(F32)
        w = (w + upd).astype(F32)
    return w, m, v


# --------------------------------------------------------------------------------------------
# GradScaler.update, torch._amp_update_scale_ (grad_scaler.py:549)
# --------------------------------------------------------------------------------------------

def scaler_update(scale: np.float32, tracker: int, found_inf: bool, growth_factor: float,
                  backoff_factor: float, growth_interval: int) -> tuple[np.float32, int]:
    """Backoff on a non-finite step, otherwise grow after ``growth_interval`` clean steps.

    The product ``scale * factor`` is formed in double and stored as fp32; growth is applied
    only when the grown scale is finite.
    """
    scale = F32(scale)
    if found_inf:
        return F32(F64(scale) * backoff_factor), 0
    successful = tracker + 1
    if successful == growth_interval:
        with np.errstate(over="ignore"):  # a product past fp32's range rounds to inf: not kept
            grown = F32(F64(scale) * growth_factor)
        return (grown if np.isfinite(grown) else scale), 0
    return scale, successful


# --------------------------------------------------------------------------------------------
# The whole chain over a list of tensors
# --------------------------------------------------------------------------------------------

@dataclass
class TensorState:
    """fp32 master ``w``, moments ``m`` and ``v`` and the per-tensor ``step`` (fp32 in torch)."""
    w: np.ndarray
    m: np.ndarray
    v: np.ndarray
    step: float = 0.0
    group: int = 0


@dataclass
class ScalerState:
    scale: np.float32 = F32(2.0 ** 16)
    tracker: int = 0
    growth_factor: float = 2.0
    backoff_factor: float = 0.5
    growth_interval: int = 2000
    enabled: bool = True


@dataclass
class StepReport:
    found_inf: bool
    norm: np.float32
    clip_coef: np.float32
    skipped: bool
    inv_scale: np.float32
    tensor_norms: list = field(default_factory=list)


def optimizer_step(states: list[TensorState], grads: list[np.ndarray], groups: list[GroupHP],
                   scaler: ScalerState | None, max_norm: float | None,
                   norm: np.float32 | None = None) -> StepReport:
    """One reference step over ``states`` in place, with ``grads`` as fp32 arrays.

    ``grads`` hold the values the backward pass produced (scaled by ``scaler.scale`` when a
    scaler is enabled).  bf16 gradients are passed through ``bf16_bits_to_f32`` first, which
    is exactly the ``.float()`` upcast.  ``norm`` overrides the computed total norm (used to
    replay the reference's own inexact norm).
    """
    use_scaler = scaler is not None and scaler.enabled
    inv = inv_scale_of(scaler.scale) if use_scaler else F32(1.0)
    found_inf = nonfinite_any(grads) if use_scaler else False
    g_eff = [unscale(g, inv) if use_scaler else np.asarray(g, dtype=F32) for g in grads]
    tnorms: list = []
    coef = F32(1.0)
    if max_norm is not None:
        tnorms = [tensor_norm(g) for g in g_eff]
        tot = total_norm(tnorms) if norm is None else F32(norm)
        coef = clip_coefficient(tot, max_norm)
        with np.errstate(over="ignore", invalid="ignore"):
            g_eff = [(g * coef).astype(F32) for g in g_eff]
    else:
        tot = F32(np.nan) if norm is None else F32(norm)
    if not found_inf:
        for st, g in zip(states, g_eff):
            st.step = float(F32(st.step) + F32(1.0))
            st.w, st.m, st.v = adamw_update(st.w, st.m, st.v, g, groups[st.group], st.step)
    if use_scaler:
        scaler.scale, scaler.tracker = scaler_update(
            scaler.scale, scaler.tracker, found_inf, scaler.growth_factor,
            scaler.backoff_factor, scaler.growth_interval)
    return StepReport(found_inf=found_inf, norm=tot, clip_coef=coef, skipped=found_inf,
                      inv_scale=inv, tensor_norms=tnorms)


# --------------------------------------------------------------------------------------------
# ZeRO-1 shard arithmetic (no reference counterpart; restates the build's partition rule)
# --------------------------------------------------------------------------------------------

def shard_bounds(padded_total: int, world_size: int, rank: int) -> tuple[int, int]:
    """Rank ``rank`` owns the contiguous flat range ``[r*S, (r+1)*S)`` with ``S = total/N``."""
    if padded_total % world_size:
        raise ValueError("padded length must divide evenly by the world size")
    s = padded_total // world_size
    return rank * s, (rank + 1) * s

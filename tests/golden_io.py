"""Loader for the golden fixtures written by ``tests/golden/make_golden.py``."""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = ("tiny_minigpt_fp32", "tiny_minigpt_bf16_scaled", "ragged_bf16_scaled")


@dataclass
class Golden:
    name: str
    names: list
    group: np.ndarray          # group index per tensor (0 = decay, 1 = no_decay)
    wd: np.ndarray             # weight decay per group
    lr: float
    beta1: float
    beta2: float
    eps: float
    max_norm: float
    init_scale: float
    growth_interval: int
    grad_dtype: str            # "bf16" (grads stored as uint16 bits) or "fp32"
    w0: list                   # initial fp32 masters
    g: list                    # g[s][i]: gradient of tensor i at step s (uint16 bits or fp32)
    w: list                    # reference state after step s
    m: list
    v: list
    step: np.ndarray           # [steps, tensors] fp32 step counters after each step
    norm: np.ndarray           # total norm returned by clip_grad_norm_ at each step
    found_inf: np.ndarray
    scale: np.ndarray          # loss scale after update() at each step
    tracker: np.ndarray

    @property
    def n_steps(self) -> int:
        return len(self.norm)

    @property
    def n_tensors(self) -> int:
        return len(self.names)

    @property
    def scaler_enabled(self) -> bool:
        return self.grad_dtype == "bf16"


def load(name: str) -> Golden:
    z = np.load(GOLDEN / f"{name}.npz")
    n = len(z["names"])
    hp = z["hp"]
    steps = len(z["norm"])

    def per_step(prefix):
        arrs = [z[f"{prefix}/{i}"] for i in range(n)]
        return [[arrs[i][s] for i in range(n)] for s in range(steps)]

    return Golden(
        name=name, names=[str(x) for x in z["names"]], group=z["group"], wd=z["wd"],
        lr=float(hp[0]), beta1=float(hp[1]), beta2=float(hp[2]), eps=float(hp[3]),
        max_norm=float(hp[4]), init_scale=float(hp[5]), growth_interval=int(hp[6]),
        grad_dtype=str(z["grad_dtype"]), w0=[z[f"w0/{i}"] for i in range(n)],
        g=per_step("g"), w=per_step("w"), m=per_step("m"), v=per_step("v"),
        step=z["step"], norm=z["norm"], found_inf=z["found_inf"], scale=z["scale"],
        tracker=z["tracker"],
    )


def close_rel(a: np.ndarray, b: np.ndarray, rtol: float, floor: float) -> tuple[bool, float]:
    """``|a-b| <= rtol * max(|b|, floor)`` elementwise; NaNs must coincide.

    ``floor`` is the magnitude below which a value is compared absolutely: a moment that is the
    difference of nearly equal terms carries the absolute error of its operands, not of itself.
    Returns (ok, worst ratio of error to allowance).
    """
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    nan_a, nan_b = np.isnan(a), np.isnan(b)
    if not np.array_equal(nan_a, nan_b):
        return False, float("inf")
    mask = ~nan_b
    if not mask.any():
        return True, 0.0
    err = np.abs(a[mask] - b[mask])
    allow = rtol * np.maximum(np.abs(b[mask]), floor)
    worst = float(np.max(err / allow)) if err.size else 0.0
    return worst <= 1.0, worst

"""The reference's own optimizer-step call sequence, executed by PyTorch on the CPU.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  This is the CPU baseline that
``bench.py --impl reference`` times and the generator behind the golden fixtures.

The reference delegates its whole optimizer step to PyTorch; this module drives exactly that
code with the reference's arguments:

* ``torch.optim.AdamW(groups, lr, betas, eps)`` as built at ``train.py:359-365``.  On a CPU
  the reference gets ``fused=False`` (``runtime.py:164`` enables fused AdamW only on CUDA) and
  torch picks the single-tensor loop (``torch/optim/optimizer.py`` ``_default_to_fused_or_foreach``
  returns no foreach for CPU tensors); ``foreach=False`` is passed to make that explicit.
* ``torch.amp.GradScaler("cpu", init_scale, growth_interval, backoff_factor)``
  (``train.py:366-370``).
* per step, ``scaler.unscale_`` -> ``clip_grad_norm_`` -> ``scaler.step`` -> ``scaler.update``
  (``train.py:485-491``).

The parameter grouping is ``build_adamw_param_groups`` (``src/minigpt/optim.py:15-64``): tensors
with ``ndim >= 2`` decay, the rest do not.  Callers pass the groups in; the golden-fixture
generator builds them with the reference's own function.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Sequence

import torch


@dataclass
class ChainConfig:
    lr: float = 6e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    max_norm: float | None = 1.0
    scaler_enabled: bool = True
    init_scale: float = 2.0 ** 16
    growth_interval: int = 2000
    backoff_factor: float = 0.5
    growth_factor: float = 2.0


class ReferenceChain:
    """Holds fp32 CPU parameters (the masters) and runs the reference step on them."""

    def __init__(self, group_params: Sequence[Sequence[torch.Tensor]], group_wd: Sequence[float],
                 cfg: ChainConfig, group_extra: Sequence[dict] | None = None):
        self.cfg = cfg
        groups = []
        self.params: list[torch.nn.Parameter] = []
        for gi, (ps, wd) in enumerate(zip(group_params, group_wd)):
            plist = [torch.nn.Parameter(p.detach().to(torch.float32).clone()) for p in ps]
            self.params.extend(plist)
            entry = {"params": plist, "weight_decay": wd}
            if group_extra is not None:
                entry.update(group_extra[gi])
            groups.append(entry)
        self.opt = torch.optim.AdamW(groups, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                     foreach=False, fused=False)
        self.scaler = torch.amp.GradScaler("cpu", enabled=cfg.scaler_enabled,
                                           init_scale=cfg.init_scale,
                                           growth_factor=cfg.growth_factor,
                                           backoff_factor=cfg.backoff_factor,
                                           growth_interval=cfg.growth_interval)
        if cfg.scaler_enabled:
            # GradScaler creates its scale tensor lazily on the first scale() call.
            self.scaler.scale(torch.ones(()))

    def set_grads(self, grads: Sequence[torch.Tensor]) -> None:
        for p, g in zip(self.params, grads):
            p.grad = g.detach().to(torch.float32).clone()

    def step(self, grads: Sequence[torch.Tensor] | None = None) -> dict:
        """One ``unscale_ -> clip_grad_norm_ -> step -> update``; returns the scalars."""
        if grads is not None:
            self.set_grads(grads)
        self.scaler.unscale_(self.opt)
        norm = None
        if self.cfg.max_norm is not None:
            norm = torch.nn.utils.clip_grad_norm_(self.params, self.cfg.max_norm)
        found = 0.0
        if self.cfg.scaler_enabled:
            st = self.scaler._per_optimizer_states[id(self.opt)]
            found = float(sum(v.item() for v in st["found_inf_per_device"].values()))
        self.scaler.step(self.opt)
        self.scaler.update()
        out = {"found_inf": found, "norm": None if norm is None else float(norm)}
        if self.cfg.scaler_enabled:
            out["scale"] = float(self.scaler._scale.item())
            out["tracker"] = int(self.scaler._growth_tracker.item())
        return out

    def state_of(self, p: torch.Tensor) -> dict:
        return self.opt.state.get(p, {})


def time_reference_chain(chain: ReferenceChain, grads: Sequence[torch.Tensor], steps: int,
                         warmup: int) -> list[float]:
    """Wall-clock seconds of ``steps`` reference steps after ``warmup`` untimed ones.

    The gradient upcast (bf16 -> fp32) and the bf16 parameter copy are part of each timed step,
    as the mixed-precision step needs both (the reference itself keeps fp32 parameters).
    """
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        for p, g in zip(chain.params, grads):
            if p.grad is None:
                p.grad = g.to(torch.float32)
            else:
                p.grad.copy_(g)
        chain.step()
        for p in chain.params:
            p.detach().to(torch.bfloat16)
        t1 = time.perf_counter()
        if i >= warmup:
            times.append(t1 - t0)
    return times

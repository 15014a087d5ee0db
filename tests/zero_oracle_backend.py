"""CPU stand-in for ZeroAdamW's three kernel calls, built on the oracle (test harness only).

``ZeroAdamW(..., _kernels=OracleKernels())`` runs the ZeRO-1 host logic -- shard geometry, the
norm-partial all-gather, the global skip decision, the bf16 parameter all-gather -- on CPU
tensors over gloo, with the per-element arithmetic done by ``oracle/adamw_oracle.py``.
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import torch

from oracle import adamw_oracle as O


def _f32(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return O.bf16_bits_to_f32(t.contiguous().view(torch.int16).numpy().view(np.uint16))
    return t.detach().numpy().astype(np.float32)


class OracleKernels:
    def __init__(self):
        self.calls = []

    def make_plan(self, opt, ranges):
        return SimpleNamespace(opt=opt, ranges=list(ranges))

    def grad_stats(self, plan, loss_scale, exch_local):
        self.calls.append("grad_stats")
        opt = plan.opt
        inv = O.inv_scale_of(float(loss_scale)) if loss_scale is not None else np.float32(1.0)
        exch = np.zeros(opt.n_slots + 1, dtype=np.float64)
        bad = False
        for slot, lo, hi in plan.ranges:
            g = _f32(opt.flat_grad[lo:hi])
            bad |= not bool(np.all(np.isfinite(g)))
            x = O.unscale(g, inv).astype(np.float64)
            with np.errstate(over="ignore", invalid="ignore"):
                exch[slot] = float(np.dot(x, x)) if x.size else 0.0
        exch[-1] = 1.0 if bad else 0.0
        exch_local.copy_(torch.from_numpy(exch))

    def finalize(self, exch_all, n_ranks, n_slots, out):
        self.calls.append("finalize")
        e = exch_all.numpy().reshape(n_ranks, n_slots + 1)
        norms = []
        for s in range(n_slots):
            acc = 0.0
            for r in range(n_ranks):
                acc += float(e[r, s])
            norms.append(np.float32(math.sqrt(acc)) if acc == acc else np.float32(np.nan))
        total = O.total_norm(norms)
        found = 1.0 if float(e[:, -1].sum()) != 0.0 else 0.0
        out.copy_(torch.tensor([found, float(total)], dtype=torch.float32))

    def adamw(self, plan, groups, steps, found_inf, loss_scale, norm, max_norm):
        self.calls.append("adamw")
        if found_inf is not None and float(found_inf) != 0.0:
            return
        opt = plan.opt
        inv = O.inv_scale_of(float(loss_scale)) if loss_scale is not None else np.float32(1.0)
        coef = O.clip_coefficient(np.float32(float(norm)), max_norm) if norm is not None \
            else np.float32(1.0)
        bf16 = opt.flat_param.dtype == torch.bfloat16
        for slot, lo, hi in plan.ranges:
            if hi <= lo:
                continue
            g = (O.unscale(_f32(opt.flat_grad[lo:hi]), inv) * coef).astype(np.float32)
            hp = groups[opt._slot_group[slot]]
            ghp = O.GroupHP(float(hp["lr"]), float(hp["beta1"]), float(hp["beta2"]),
                            float(hp["eps"]), float(hp["weight_decay"]))
            loc = lo - opt.geom.lo
            n = hi - lo
            w = opt.master[loc:loc + n].numpy().copy()
            m = opt.exp_avg[loc:loc + n].numpy().copy()
            v = opt.exp_avg_sq[loc:loc + n].numpy().copy()
            step = float(np.float32(float(steps[slot])) + np.float32(1.0))
            w, m, v = O.adamw_update(w, m, v, g, ghp, step)
            opt.master[loc:loc + n] = torch.from_numpy(w)
            opt.exp_avg[loc:loc + n] = torch.from_numpy(m)
            opt.exp_avg_sq[loc:loc + n] = torch.from_numpy(v)
            if bf16:
                bits = O.f32_to_bf16_bits(w).view(np.int16)
                opt.flat_param[lo:hi] = torch.from_numpy(bits.copy()).view(torch.bfloat16)
        for slot, _, _ in plan.ranges:
            steps[slot] += 1.0

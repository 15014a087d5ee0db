"""The fused step through the public API over the seeded configuration sweep of
``test_oracle_vs_torch_random.py`` (per-group hyper-parameters, clipping off/weak/strong, scaler
off/on with different scales and growth intervals, bf16 or fp32 gradients and parameters,
inf/NaN steps, ragged sizes), four steps each, against the oracle given the kernel's own norm:
flags, loss scale, tracker and step counters exact, every state word and every bf16 bit equal.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import adamw_oracle as O
from test_oracle_vs_torch_random import _case, _grads

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("seed", range(24))
def test_fused_step_matches_oracle_over_the_sweep(seed):
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    shapes, group_of, hp, cfg = _case(seed)
    gen = torch.Generator().manual_seed(seed)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    n_groups = len(hp)
    order = [i for g in range(n_groups) for i in range(len(shapes)) if group_of[i] == g]
    dtype = torch.bfloat16 if cfg["bf16"] else torch.float32
    params = [torch.nn.Parameter(w0[i].to(dtype).to(DEV)) for i in order]
    groups = [{"params": [p for p, i in zip(params, order) if group_of[i] == g],
               "lr": hp[g]["lr"], "betas": hp[g]["betas"], "eps": hp[g]["eps"],
               "weight_decay": hp[g]["weight_decay"]} for g in range(n_groups)]
    opt = FusedAdamW(groups)
    if cfg["bf16"]:
        for p, i in zip(params, order):
            opt.set_master_(p, w0[i].to(DEV))
    scaler = GradScaler("cuda", enabled=cfg["scaler"], init_scale=cfg["scale"],
                        growth_interval=cfg["growth_interval"])
    if cfg["scaler"]:
        scaler.scale(torch.ones((), device=DEV))

    ohp = [O.GroupHP(h["lr"], h["betas"][0], h["betas"][1], h["eps"], h["weight_decay"])
           for h in hp]
    states = [O.TensorState(w=w0[i].numpy().copy(), m=np.zeros(shapes[i], np.float32),
                            v=np.zeros(shapes[i], np.float32), group=group_of[i]) for i in order]
    osc = O.ScalerState(scale=np.float32(cfg["scale"]), growth_interval=cfg["growth_interval"],
                        enabled=cfg["scaler"])
    for step in range(4):
        gs = _grads(seed, step, shapes, cfg)
        for p, i in zip(params, order):
            p.grad = gs[i].to(dtype).to(DEV)
        scaler.unscale_(opt)
        norm = None
        if cfg["max_norm"] is not None:
            norm = np.float32(float(clip_grad_norm_(params, cfg["max_norm"])))
        found = None
        if cfg["scaler"]:
            st = scaler._per_optimizer_states[id(opt)]
            found = float(next(iter(st["found_inf_per_device"].values())))
        scaler.step(opt)
        scaler.update()
        rep = O.optimizer_step(states, [gs[i].numpy() for i in order], ohp,
                               osc if cfg["scaler"] else None, cfg["max_norm"], norm=norm)
        if cfg["scaler"]:
            assert found == (1.0 if rep.found_inf else 0.0), step
            assert float(scaler.get_scale()) == float(osc.scale)
            assert int(scaler._growth_tracker) == osc.tracker
        for p, st in zip(params, states):
            s = opt.state[p]
            assert float(s["step"]) == st.step
            master = s["master_param"] if cfg["bf16"] else p.detach()
            np.testing.assert_array_equal(master.cpu().numpy(), st.w)
            np.testing.assert_array_equal(s["exp_avg"].cpu().numpy(), st.m)
            np.testing.assert_array_equal(s["exp_avg_sq"].cpu().numpy(), st.v)
            if cfg["bf16"]:
                bits = p.detach().view(torch.int16).cpu().numpy().view(np.uint16)
                np.testing.assert_array_equal(bits, O.f32_to_bf16_bits(st.w))

"""The oracle against the reference's own arithmetic -- PyTorch's CPU ``AdamW`` + ``GradScaler``
+ ``clip_grad_norm_`` in the order of ``train.py:485-491`` (``oracle/torch_chain.py``) -- over a
seeded sweep of configurations the golden fixtures do not cover: per-group learning rates,
betas, eps and weight decay; clipping off, weak and strong; scaler off or on with different
initial scales and growth intervals; bf16 or fp32 gradients; an inf or NaN step; ragged sizes.

The bar is the fixtures' bar: flags, scale, tracker and step counters exact; with the
reference's own total norm (torch accumulates the CPU norm in fp32) the moments bit-exact and
the masters within 1e-6 relative to the tensor's largest magnitude (torch's vectorised CPU
``sqrt`` is not always correctly rounded; the oracle's is).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import adamw_oracle as O
from oracle.torch_chain import ChainConfig, ReferenceChain

SHAPE_POOL = [(0,), (1,), (7,), (33, 17), (129,), (4097,), (16, 64), (3, 3, 5)]


def _case(seed):
    rng = np.random.default_rng(seed)
    shapes = [SHAPE_POOL[i] for i in sorted(rng.choice(len(SHAPE_POOL), 5, replace=False))]
    n_groups = int(rng.integers(1, 3))
    group_of = [int(rng.integers(0, n_groups)) for _ in shapes]
    hp = []
    for _ in range(n_groups):
        hp.append(dict(lr=float(10 ** rng.uniform(-5, -2)),
                       betas=(float(rng.choice([0.8, 0.9, 0.95])),
                              float(rng.choice([0.95, 0.99, 0.999]))),
                       eps=float(rng.choice([1e-8, 1e-6])),
                       weight_decay=float(rng.choice([0.0, 0.01, 0.1]))))
    cfg = dict(max_norm=[None, 0.1, 1.0, 1e3][int(rng.integers(0, 4))],
               scaler=bool(rng.integers(0, 2)), scale=float(2.0 ** int(rng.choice([8, 12, 16]))),
               growth_interval=int(rng.choice([1, 2, 2000])),
               bf16=bool(rng.integers(0, 2)), bad_step=int(rng.integers(-1, 3)),
               bad_value=float(rng.choice([np.inf, -np.inf, np.nan])))
    return shapes, group_of, hp, cfg


def _grads(seed, step, shapes, cfg):
    gen = torch.Generator().manual_seed(10_000 * seed + step)
    mult = cfg["scale"] if cfg["scaler"] else 1.0
    gs = [torch.randn(s, generator=gen) * 0.05 * mult for s in shapes]
    if cfg["bf16"]:
        gs = [g.to(torch.bfloat16).float() for g in gs]
    if step == cfg["bad_step"] and cfg["scaler"]:
        big = max(range(len(shapes)), key=lambda i: gs[i].numel())
        gs[big].view(-1)[gs[big].numel() // 2] = cfg["bad_value"]
    return gs


def _normwise(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if a.size == 0:
        return 0.0
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.mark.parametrize("seed", range(24))
def test_oracle_matches_torch_chain(seed):
    shapes, group_of, hp, cfg = _case(seed)
    gen = torch.Generator().manual_seed(seed)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    n_groups = len(hp)
    order = [i for g in range(n_groups) for i in range(len(shapes)) if group_of[i] == g]
    chain = ReferenceChain([[w0[i] for i in order if group_of[i] == g] for g in range(n_groups)],
                           [h["weight_decay"] for h in hp],
                           ChainConfig(lr=hp[0]["lr"], betas=hp[0]["betas"], eps=hp[0]["eps"],
                                       max_norm=cfg["max_norm"], scaler_enabled=cfg["scaler"],
                                       init_scale=cfg["scale"],
                                       growth_interval=cfg["growth_interval"]),
                           group_extra=[dict(lr=h["lr"], betas=h["betas"], eps=h["eps"])
                                        for h in hp])
    groups = [O.GroupHP(h["lr"], h["betas"][0], h["betas"][1], h["eps"], h["weight_decay"])
              for h in hp]
    states = [O.TensorState(w=w0[i].numpy().copy(), m=np.zeros(shapes[i], np.float32),
                            v=np.zeros(shapes[i], np.float32), group=group_of[i]) for i in order]
    scaler = O.ScalerState(scale=np.float32(cfg["scale"]), growth_interval=cfg["growth_interval"],
                           enabled=cfg["scaler"])
    for step in range(4):
        gs = _grads(seed, step, shapes, cfg)
        ref = chain.step([gs[i] for i in order])
        ref_norm = None if ref["norm"] is None else np.float32(ref["norm"])
        rep = O.optimizer_step(states, [gs[i].numpy() for i in order], groups,
                               scaler if cfg["scaler"] else None, cfg["max_norm"], norm=ref_norm)
        assert bool(rep.found_inf) == bool(ref["found_inf"]), step
        if cfg["scaler"]:
            assert scaler.scale == np.float32(ref["scale"]) and scaler.tracker == ref["tracker"]
        for st, p in zip(states, chain.params):
            s = chain.state_of(p)
            torch_step = float(s["step"]) if "step" in s else 0.0
            assert st.step == torch_step
            if "exp_avg" in s:
                np.testing.assert_array_equal(st.m, s["exp_avg"].numpy())
                np.testing.assert_array_equal(st.v, s["exp_avg_sq"].numpy())
            assert _normwise(st.w, p.detach().numpy()) <= 1e-6, (step, "w")


def test_sweep_covers_the_cases():
    cases = [_case(s) for s in range(24)]
    cfgs = [c[3] for c in cases]
    assert sum(c["scaler"] and c["bad_step"] >= 0 for c in cfgs) >= 3       # skipped steps
    assert sum(not c["scaler"] for c in cfgs) >= 3                          # scaler off
    assert {c["max_norm"] for c in cfgs} == {None, 0.1, 1.0, 1e3}           # clip off/on/idle
    assert {c["bf16"] for c in cfgs} == {True, False}
    assert sum(len(c[2]) == 2 for c in cases) >= 3                          # two param groups
    assert {c["growth_interval"] for c in cfgs} >= {1, 2}                   # growth happens


@pytest.mark.parametrize("start_step", [999.0, 123456.0])
def test_oracle_matches_torch_chain_from_a_late_step(start_step):
    """Bias corrections far from step 1 (BASELINE config 2 stores step 999): the state is loaded
    into torch's AdamW at ``start_step`` with non-zero moments, then two steps run on both."""
    shapes = [(257,), (64, 33), (5,)]
    gen = torch.Generator().manual_seed(99)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    m0 = [torch.randn(s, generator=gen) * 1e-3 for s in shapes]
    v0 = [torch.randn(s, generator=gen).abs() * 1e-6 for s in shapes]
    chain = ReferenceChain([w0], [0.1], ChainConfig(lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                                                    max_norm=1.0, scaler_enabled=True,
                                                    init_scale=2.0 ** 16))
    sd = chain.opt.state_dict()
    sd["state"] = {i: {"step": torch.tensor(start_step), "exp_avg": m0[i].clone(),
                       "exp_avg_sq": v0[i].clone()} for i in range(len(shapes))}
    chain.opt.load_state_dict(sd)
    states = [O.TensorState(w=w0[i].numpy().copy(), m=m0[i].numpy().copy(),
                            v=v0[i].numpy().copy(), step=start_step) for i in range(len(shapes))]
    scaler = O.ScalerState(scale=np.float32(2.0 ** 16))
    hp = [O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.1)]
    for step in range(2):
        g = torch.Generator().manual_seed(500 + step)
        gs = [(torch.randn(s, generator=g) * 1e-2 * 2.0 ** 16).to(torch.bfloat16).float()
              for s in shapes]
        ref = chain.step(gs)
        O.optimizer_step(states, [x.numpy() for x in gs], hp, scaler, 1.0,
                         norm=np.float32(ref["norm"]))
        for st, p in zip(states, chain.params):
            s = chain.state_of(p)
            assert st.step == float(s["step"]) == start_step + step + 1
            np.testing.assert_array_equal(st.m, s["exp_avg"].numpy())
            np.testing.assert_array_equal(st.v, s["exp_avg_sq"].numpy())
            assert _normwise(st.w, p.detach().numpy()) <= 1e-6


@pytest.mark.parametrize("scale,growth", [(2.0 ** 127, 2.0), (3.0e38, 1.1), (1.7e38, 2.0),
                                          (2.0 ** 126, 2.0), (2.0 ** -100, 0.5)])
@pytest.mark.parametrize("found", [0.0, 1.0, float("nan")])
def test_scaler_update_matches_torch_at_the_edges(scale, growth, found):
    """torch._amp_update_scale_ (grad_scaler.py:549) against the oracle: growth that would
    overflow fp32 is not applied, a NaN flag counts as found, backoff rounds through double."""
    s = torch.tensor([scale], dtype=torch.float32)
    t = torch.tensor([0], dtype=torch.int32)
    torch._amp_update_scale_(s, t, torch.tensor([found]), growth, 0.5, 1)
    o_scale, o_tracker = O.scaler_update(np.float32(scale), 0, found != 0.0, growth, 0.5, 1)
    assert np.float32(s.item()) == o_scale and int(t.item()) == o_tracker


@pytest.mark.parametrize("max_norm", [1.0, 0.25, 1e-3])
@pytest.mark.parametrize("kind", ["zero", "tiny", "at_max", "large", "inf", "nan"])
def test_clip_coefficient_matches_torch(kind, max_norm):
    """torch.nn.utils.clip_grad_norm_ (clip_grad.py:165-174) multiplies every gradient by its
    clamped coefficient; the oracle's coefficient times the same gradients must give the same
    bits, including for a zero, inf or NaN total norm."""
    g = torch.tensor([3.0, -4.0, 0.5, 1e-20], dtype=torch.float32)
    g = {"zero": g * 0.0, "tiny": g * 1e-30, "at_max": g / float(torch.linalg.vector_norm(g)) *
         max_norm, "large": g * 1e10,
         "inf": torch.cat([g, torch.tensor([float("inf")])]),
         "nan": torch.cat([g, torch.tensor([float("nan")])])}[kind]
    p = torch.nn.Parameter(torch.zeros_like(g))
    p.grad = g.clone()
    norm = torch.nn.utils.clip_grad_norm_([p], max_norm)
    coef = O.clip_coefficient(np.float32(norm.item()), max_norm)
    with np.errstate(invalid="ignore", over="ignore"):
        want = (g.numpy() * coef).astype(np.float32)
    got = p.grad.numpy()
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    np.testing.assert_array_equal(got[~np.isnan(got)], want[~np.isnan(want)])

"""GPU parity of the fused step against the reference's path (golden fixtures) and the oracle.

Every case calls through the package's public API (``FusedAdamW``, ``GradScaler``,
``clip_grad_norm_``), which binds the C ABI of ``include/b200_optim.h``.

Bars (stated for this path): ``found_inf``/skip, ``step``, loss scale and growth tracker
bit-exact; fp32 master/``exp_avg``/``exp_avg_sq`` within 1e-6 relative (per tensor, against its
largest magnitude) of the reference; bf16 parameters within 1 ulp.  Against the CPU oracle fed
the kernel's own norm, the results must be bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_io as G
from oracle import adamw_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-6


def _normwise(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if a.size == 0:
        return 0.0
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def _bf16_ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray) -> int:
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # map sign-magnitude to a monotone integer line
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), 0x8000 + a)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + b)
    return int(np.max(np.abs(a - b))) if a.size else 0


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _to_bf16_tensor(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16).copy()).view(
        torch.bfloat16).to(device)


def _build(gd: G.Golden, device, chunk_elems=1 << 16):
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler
    bf16 = gd.grad_dtype == "bf16"
    params = []
    for w0 in gd.w0:
        t = torch.from_numpy(w0.copy()).to(device)
        params.append(torch.nn.Parameter(t.to(torch.bfloat16) if bf16 else t))
    groups = []
    for gi in range(len(gd.wd)):
        groups.append({"params": [p for p, g in zip(params, gd.group) if g == gi],
                       "weight_decay": float(gd.wd[gi])})
    opt = FusedAdamW(groups, lr=gd.lr, betas=(gd.beta1, gd.beta2), eps=gd.eps,
                     chunk_elems=chunk_elems)
    # order of the fixture == order of the groups (decay first), as make_golden wrote it
    order = [p for g in groups for p in g["params"]]
    assert [id(p) for p in order] == [id(p) for p in params]
    if bf16:
        for p, w0 in zip(params, gd.w0):
            opt.set_master_(p, torch.from_numpy(w0.copy()).to(device))
    scaler = GradScaler("cuda", init_scale=gd.init_scale, growth_interval=gd.growth_interval,
                        enabled=gd.scaler_enabled)
    scaler.scale(torch.ones((), device=device))  # creates the scale tensor, as loss scaling does
    return params, opt, scaler


def _set_grads(gd, params, s, device):
    for p, g in zip(params, gd.g[s]):
        if gd.grad_dtype == "bf16":
            p.grad = _to_bf16_tensor(g, device).view(p.shape)
        else:
            p.grad = torch.from_numpy(g.copy()).to(device).view(p.shape)


def _step(params, opt, scaler, max_norm):
    from minigpt_train_infra_b200 import clip_grad_norm_
    scaler.unscale_(opt)
    norm = clip_grad_norm_(params, max_norm)
    found = None
    if scaler.is_enabled():
        st = scaler._per_optimizer_states[id(opt)]
        found = float(next(iter(st["found_inf_per_device"].values())).item())
    norm_v = float(norm.item())
    scaler.step(opt)
    scaler.update()
    return norm_v, found


@pytest.mark.parametrize("name", G.FIXTURES)
@pytest.mark.parametrize("chunk_elems", [1 << 16, 64])
def test_fused_step_matches_reference_fixture(name, chunk_elems):
    device = torch.device("cuda", 0)
    gd = G.load(name)
    params, opt, scaler = _build(gd, device, chunk_elems)
    for s in range(gd.n_steps):
        _set_grads(gd, params, s, device)
        norm, found = _step(params, opt, scaler, gd.max_norm)
        torch.cuda.synchronize()
        if gd.scaler_enabled:
            assert found == gd.found_inf[s], s
            assert float(scaler._scale.item()) == gd.scale[s]
            assert int(scaler._growth_tracker.item()) == gd.tracker[s]
        if np.isfinite(gd.norm[s]):
            assert abs(norm - gd.norm[s]) <= RTOL * gd.norm[s], (s, norm, gd.norm[s])
        else:
            assert np.isnan(norm) == np.isnan(gd.norm[s]) and not np.isfinite(norm)
        for i, p in enumerate(params):
            st = opt.state[p]
            assert float(st["step"].item()) == gd.step[s][i]
            master = st["master_param"] if "master_param" in st else p.detach()
            w = master.float().cpu().numpy()
            assert _normwise(w, gd.w[s][i]) <= RTOL, (s, i, "w")
            assert _normwise(st["exp_avg"].cpu().numpy(), gd.m[s][i]) <= RTOL, (s, i, "m")
            assert _normwise(st["exp_avg_sq"].cpu().numpy(), gd.v[s][i]) <= RTOL, (s, i, "v")
            if p.dtype == torch.bfloat16:
                ref_bits = O.f32_to_bf16_bits(gd.w[s][i].astype(np.float32))
                assert _bf16_ulp_diff(_bits(p), ref_bits) <= 1, (s, i, "bf16")


@pytest.mark.parametrize("name", G.FIXTURES)
def test_fused_step_bit_exact_vs_oracle_given_kernel_norm(name):
    """With the oracle fed the kernel's own norm, every state word must agree bit for bit."""
    device = torch.device("cuda", 0)
    gd = G.load(name)
    params, opt, scaler = _build(gd, device, 1 << 16)
    groups = [O.GroupHP(gd.lr, gd.beta1, gd.beta2, gd.eps, float(gd.wd[k]))
              for k in range(len(gd.wd))]
    states = [O.TensorState(w=gd.w0[i].astype(np.float32).copy(),
                            m=np.zeros(gd.w0[i].shape, np.float32),
                            v=np.zeros(gd.w0[i].shape, np.float32), group=int(gd.group[i]))
              for i in range(gd.n_tensors)]
    osc = O.ScalerState(scale=np.float32(gd.init_scale), growth_interval=gd.growth_interval,
                        enabled=gd.scaler_enabled)
    for s in range(gd.n_steps):
        _set_grads(gd, params, s, device)
        norm, found = _step(params, opt, scaler, gd.max_norm)
        grads = [O.bf16_bits_to_f32(g) if gd.grad_dtype == "bf16" else g for g in gd.g[s]]
        rep = O.optimizer_step(states, grads, groups, osc if gd.scaler_enabled else None,
                               gd.max_norm, norm=np.float32(norm))
        # the kernel's norm itself: within 2 ulp of the oracle's exact-then-rounded norm
        exact = O.total_norm([O.tensor_norm(O.unscale(g, rep.inv_scale)) for g in grads])
        if np.isfinite(exact):
            assert abs(np.float32(norm) - exact) <= 2 * np.spacing(np.float32(exact))
        for i, p in enumerate(params):
            st = opt.state[p]
            master = st["master_param"] if "master_param" in st else p.detach()
            np.testing.assert_array_equal(master.float().cpu().numpy(), states[i].w)
            np.testing.assert_array_equal(st["exp_avg"].cpu().numpy(), states[i].m)
            np.testing.assert_array_equal(st["exp_avg_sq"].cpu().numpy(), states[i].v)
            if p.dtype == torch.bfloat16:
                np.testing.assert_array_equal(_bits(p), O.f32_to_bf16_bits(states[i].w))


def test_misaligned_views_take_the_scalar_path_and_match():
    """Parameters that are 2-byte-offset views cannot use 128-bit loads; results must agree."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    device = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(5)
    base = torch.randn(20001, generator=gen) * 0.02
    sizes = [(0, 4096), (4096, 4104), (4104, 11104), (11104, 20000)]
    outs = []
    for misalign in (False, True):
        store = torch.zeros(20002, dtype=torch.bfloat16, device=device)
        off = 1 if misalign else 0
        store[off:off + 20001] = base.to(torch.bfloat16).to(device)
        params = [torch.nn.Parameter(store[off + a:off + b]) for a, b in sizes]
        opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)
        sc = GradScaler("cuda", init_scale=2.0 ** 10)
        sc.scale(torch.ones((), device=device))
        g_gen = torch.Generator().manual_seed(9)
        for _ in range(3):
            gstore = torch.zeros(20002, dtype=torch.bfloat16, device=device)
            gstore[off:off + 20001] = (torch.randn(20001, generator=g_gen) * 2.0 ** 10
                                       ).to(torch.bfloat16).to(device)
            for p, (a, b) in zip(params, sizes):
                p.grad = gstore[off + a:off + b]
            sc.unscale_(opt)
            clip_grad_norm_(params, 1.0)
            sc.step(opt)
            sc.update()
        vec = [pl.vector_fraction() for pl in opt._plans]
        assert (min(vec) < 1.0) if misalign else (min(vec) == 1.0)
        outs.append([torch.cat([opt.state[p][k].flatten().cpu() for p in params])
                     for k in ("master_param", "exp_avg", "exp_avg_sq")])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_skipped_step_moves_nothing():
    """An inf anywhere skips the update: state, params and step counters bit-identical."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    device = torch.device("cuda", 0)
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(n, device=device).to(torch.bfloat16))
              for n in (1 << 20, 3, 77777)]
    opt = FusedAdamW(params, lr=1e-3)
    sc = GradScaler("cuda", init_scale=2.0 ** 16)
    sc.scale(torch.ones((), device=device))
    for p in params:
        p.grad = torch.randn_like(p)
    sc.unscale_(opt); clip_grad_norm_(params, 1.0); sc.step(opt); sc.update()
    before = {k: torch.cat([opt.state[p][k].flatten() for p in params]).clone()
              for k in ("master_param", "exp_avg", "exp_avg_sq")}
    pbefore = torch.cat([p.detach().flatten() for p in params]).clone()
    steps_before = [float(opt.state[p]["step"]) for p in params]
    params[2].grad[12345] = float("nan")
    sc.unscale_(opt); clip_grad_norm_(params, 1.0); sc.step(opt); sc.update()
    torch.cuda.synchronize()
    for k, v in before.items():
        assert torch.equal(v, torch.cat([opt.state[p][k].flatten() for p in params]))
    assert torch.equal(pbefore, torch.cat([p.detach().flatten() for p in params]))
    assert [float(opt.state[p]["step"]) for p in params] == steps_before
    assert float(sc.get_scale()) == 2.0 ** 15


def test_fp32_params_without_scaler_match_oracle():
    """The reference's own configuration: fp32 params, fp32 grads, scaler off, clip on."""
    from minigpt_train_infra_b200 import FusedAdamW, clip_grad_norm_
    device = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(3)
    shapes = [(300, 129), (129,), (5,), (64, 64, 3)]
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    params = [torch.nn.Parameter(w.clone().to(device)) for w in w0]
    groups = [{"params": [params[0], params[3]], "weight_decay": 0.1},
              {"params": [params[1], params[2]], "weight_decay": 0.0, "lr": 2e-3}]
    opt = FusedAdamW(groups, lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    order = [0, 3, 1, 2]
    ohp = [O.GroupHP(6e-4, 0.9, 0.95, 1e-8, 0.1), O.GroupHP(2e-3, 0.9, 0.95, 1e-8, 0.0)]
    states = [O.TensorState(w=w0[i].numpy().copy(), m=np.zeros(shapes[i], np.float32),
                            v=np.zeros(shapes[i], np.float32), group=0 if i in (0, 3) else 1)
              for i in order]
    for s in range(5):
        grads = [torch.randn(shapes[i], generator=gen) * 0.3 for i in order]
        for i, g in zip(order, grads):
            params[i].grad = g.to(device)
        norm = clip_grad_norm_(params, 1.0)
        opt.step()
        O.optimizer_step(states, [g.numpy() for g in grads], ohp, None, 1.0,
                         norm=np.float32(norm.item()))
        for k, i in enumerate(order):
            np.testing.assert_array_equal(params[i].detach().cpu().numpy(), states[k].w)
            np.testing.assert_array_equal(opt.state[params[i]]["exp_avg"].cpu().numpy(),
                                          states[k].m)

"""Drop-in behaviour of FusedAdamW / GradScaler / clip_grad_norm_ on a GPU.

What the reference's training loop and checkpoint code rely on (``train.py:162-176,359-370,
464-491``, ``checkpoint.py:41-42``, ``src/minigpt/optim.py:67-71,124-251``): per-step lr writes,
step accounting, state_dict round trips, loading torch AdamW state, loaders that assign
``optimizer.state[p]`` directly, and the stock torch GradScaler / clip.  Numbers are checked against
the CPU oracle (``oracle/adamw_oracle.py``) or against an uninterrupted run.
"""

from __future__ import annotations

import io

import numpy as np
import pytest
import torch

from oracle import adamw_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _normwise(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return 0.0 if a.size == 0 else float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _params(shapes, dtype, seed=0):
    gen = torch.Generator().manual_seed(seed)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    return w0, [torch.nn.Parameter(w.to(dtype).to(DEV)) for w in w0]


def _grads(shapes, step, dtype, scale=1.0):
    gen = torch.Generator().manual_seed(100 + step)
    return [(torch.randn(s, generator=gen) * 0.1 * scale).to(dtype) for s in shapes]


def test_lr_written_each_step_is_used():
    """cosine_lr + set_optimizer_lr write group["lr"] every step (optim.py:67-71)."""
    from minigpt_train_infra_b200 import FusedAdamW, clip_grad_norm_
    shapes = [(64, 33), (33,)]
    w0, params = _params(shapes, torch.float32)
    opt = FusedAdamW([{"params": [params[0]], "weight_decay": 0.1},
                      {"params": [params[1]], "weight_decay": 0.0}], lr=1.0, betas=(0.9, 0.95))
    states = [O.TensorState(w=w.numpy().copy(), m=np.zeros(w.shape, np.float32),
                            v=np.zeros(w.shape, np.float32), group=i) for i, w in enumerate(w0)]
    for s, lr in enumerate([1e-4, 6e-4, 3e-4, 0.0]):
        for g in opt.param_groups:
            g["lr"] = lr
        gs = _grads(shapes, s, torch.float32)
        for p, g in zip(params, gs):
            p.grad = g.to(DEV)
        norm = clip_grad_norm_(params, 1.0)
        opt.step()
        hp = [O.GroupHP(lr, 0.9, 0.95, 1e-8, 0.1), O.GroupHP(lr, 0.9, 0.95, 1e-8, 0.0)]
        O.optimizer_step(states, [g.numpy() for g in gs], hp, None, 1.0,
                         norm=np.float32(norm.item()))
        for p, st in zip(params, states):
            np.testing.assert_array_equal(p.detach().cpu().numpy(), st.w)


def test_mixed_bf16_and_fp32_parameters_share_one_norm():
    """Two dtype buckets: two statistics launches folded by the finalize kernel."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    shapes = [(128, 40), (40,), (7,), (300,)]
    gen = torch.Generator().manual_seed(4)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    dts = [torch.bfloat16, torch.float32, torch.bfloat16, torch.float32]
    params = [torch.nn.Parameter(w.to(d).to(DEV)) for w, d in zip(w0, dts)]
    opt = FusedAdamW(params, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.05)
    for p, w in zip(params, w0):
        opt.set_master_(p, w.to(DEV))
    sc = GradScaler("cuda", init_scale=2.0 ** 8)
    sc.scale(torch.ones((), device=DEV))
    states = [O.TensorState(w=w.numpy().copy(), m=np.zeros(w.shape, np.float32),
                            v=np.zeros(w.shape, np.float32)) for w in w0]
    osc = O.ScalerState(scale=np.float32(2.0 ** 8))
    hp = [O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.05)]
    for s in range(4):
        gs = [g.to(d) for g, d in zip(_grads(shapes, s, torch.float32, 2.0 ** 8), dts)]
        for p, g in zip(params, gs):
            p.grad = g.to(DEV)
        sc.unscale_(opt)
        norm = clip_grad_norm_(params, 1.0)
        sc.step(opt)
        sc.update()
        assert len(opt._plans) == 2
        rep = O.optimizer_step(states, [g.float().numpy() for g in gs], hp, osc, 1.0,
                               norm=np.float32(norm.item()))
        exact = O.total_norm([O.tensor_norm(O.unscale(g.float().numpy(), rep.inv_scale))
                              for g in gs])
        assert abs(np.float32(norm.item()) - exact) <= 2 * np.spacing(exact)
        for p, st in zip(params, states):
            master = opt.state[p].get("master_param", p.detach())
            np.testing.assert_array_equal(master.float().cpu().numpy(), st.w)


def _run(opt, sc, params, shapes, steps, start=0):
    from minigpt_train_infra_b200 import clip_grad_norm_
    for s in range(start, start + steps):
        for p, g in zip(params, _grads(shapes, s, torch.bfloat16, 2.0 ** 10)):
            p.grad = g.to(DEV)
        sc.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        sc.step(opt)
        sc.update()


def test_state_dict_round_trip_resumes_bit_exactly():
    """checkpoint.py:41-42 saves state_dict(); resuming must equal an uninterrupted run
    (the property tests/test_resume_consistency.py pins for the reference on CPU)."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler
    shapes = [(96, 64), (64,), (1000,)]

    def fresh():
        w0, params = _params(shapes, torch.bfloat16, seed=9)
        opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.95))
        for p, w in zip(params, w0):
            opt.set_master_(p, w.to(DEV))
        sc = GradScaler("cuda", init_scale=2.0 ** 10, growth_interval=3)
        sc.scale(torch.ones((), device=DEV))
        return params, opt, sc

    p1, o1, s1 = fresh()
    _run(o1, s1, p1, shapes, 6)
    p2, o2, s2 = fresh()
    _run(o2, s2, p2, shapes, 3)
    buf = io.BytesIO()
    torch.save({"opt": o2.state_dict(), "sc": s2.state_dict(),
                "model": [p.detach().clone() for p in p2]}, buf)
    buf.seek(0)
    ck = torch.load(buf, weights_only=False)
    sd = ck["opt"]
    assert set(sd["state"][0]) == {"step", "exp_avg", "exp_avg_sq", "master_param"}
    assert sd["state"][0]["exp_avg"].dtype == torch.float32
    p3, o3, s3 = fresh()
    with torch.no_grad():
        for p, saved in zip(p3, ck["model"]):
            p.copy_(saved)
    o3.load_state_dict(sd)
    s3.load_state_dict(ck["sc"])
    _run(o3, s3, p3, shapes, 3, start=3)
    torch.cuda.synchronize()
    for a, b in zip(p1, p3):
        assert torch.equal(a, b)
    for a, b in zip(p1, p3):
        for k in ("exp_avg", "exp_avg_sq", "master_param", "step"):
            assert torch.equal(o1.state[a][k], o3.state[b][k]), k
    assert s1.get_scale() == s3.get_scale()


def test_loads_torch_adamw_state_and_continues_like_it():
    """A torch.optim.AdamW checkpoint (fp32 params) loads into FusedAdamW and continues within
    the parity tolerance of torch's own CPU AdamW."""
    from minigpt_train_infra_b200 import FusedAdamW
    shapes = [(50, 20), (20,)]
    gen = torch.Generator().manual_seed(12)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    cpu_params = [torch.nn.Parameter(w.clone()) for w in w0]
    ref = torch.optim.AdamW(cpu_params, lr=1e-3, betas=(0.9, 0.95), foreach=False, fused=False)
    for s in range(3):
        for p, g in zip(cpu_params, _grads(shapes, s, torch.float32)):
            p.grad = g
        ref.step()
    gpu_params = [torch.nn.Parameter(p.detach().clone().to(DEV)) for p in cpu_params]
    opt = FusedAdamW(gpu_params, lr=1e-3, betas=(0.9, 0.95))
    opt.load_state_dict(ref.state_dict())
    assert float(opt.state[gpu_params[0]]["step"]) == 3.0
    for s in range(3, 6):
        gs = _grads(shapes, s, torch.float32)
        for p, q, g in zip(cpu_params, gpu_params, gs):
            p.grad = g
            q.grad = g.to(DEV)
        ref.step()
        opt.step()
    for p, q in zip(cpu_params, gpu_params):
        assert _normwise(q.detach().cpu().numpy(), p.detach().numpy()) <= 1e-6
        assert _normwise(opt.state[q]["exp_avg"].cpu().numpy(),
                         ref.state[p]["exp_avg"].numpy()) <= 1e-6


def test_direct_state_assignment_is_ingested():
    """The reference's legacy loader clears optimizer.state and assigns per-param dicts cast to
    the param dtype (src/minigpt/optim.py:124-133,242-251); the next step must use them."""
    from minigpt_train_infra_b200 import FusedAdamW
    shapes = [(40, 40), (40,)]
    w0, params = _params(shapes, torch.float32, seed=21)
    opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0)
    m_in = [torch.full(s, 1e-3) for s in shapes]
    v_in = [torch.full(s, 4e-6) for s in shapes]
    opt.state.clear()
    for p, m, v in zip(params, m_in, v_in):
        opt.state[p] = {"step": torch.tensor(7.0), "exp_avg": m.to(DEV), "exp_avg_sq": v.to(DEV)}
    gs = _grads(shapes, 0, torch.float32)
    for p, g in zip(params, gs):
        p.grad = g.to(DEV)
    opt.step()
    hp = [O.GroupHP(1e-3, 0.9, 0.95, 1e-8, 0.0)]
    for p, w, m, v, g in zip(params, w0, m_in, v_in, gs):
        st = O.TensorState(w=w.numpy().copy(), m=m.numpy().copy(), v=v.numpy().copy(), step=7.0)
        O.optimizer_step([st], [g.numpy()], hp, None, None)
        np.testing.assert_array_equal(p.detach().cpu().numpy(), st.w)
        assert float(opt.state[p]["step"]) == 8.0


@pytest.mark.parametrize("call_unscale", [True, False])
def test_stock_torch_gradscaler_and_clip_work_with_fused_adamw(call_unscale):
    """torch's own GradScaler/clip rewrite the gradients; with unscale_ skipped, GradScaler.step
    hands over grad_scale and found_inf (grad_scaler.py:418-470).  Both paths must match."""
    from minigpt_train_infra_b200 import FusedAdamW
    shapes = [(64, 64), (64,)]
    w0, params = _params(shapes, torch.float32, seed=5)
    opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)
    sc = torch.amp.GradScaler("cuda", init_scale=2.0 ** 12)
    sc.scale(torch.ones((), device=DEV))
    states = [O.TensorState(w=w.numpy().copy(), m=np.zeros(w.shape, np.float32),
                            v=np.zeros(w.shape, np.float32)) for w in w0]
    osc = O.ScalerState(scale=np.float32(2.0 ** 12))
    hp = [O.GroupHP(1e-3, 0.9, 0.95, 1e-8, 0.1)]
    for s in range(4):
        gs = _grads(shapes, s, torch.float32, 2.0 ** 12)
        if s == 2:
            gs[1][3] = float("inf")
        for p, g in zip(params, gs):
            p.grad = g.to(DEV)
        norm = None
        if call_unscale:
            sc.unscale_(opt)
            norm = torch.nn.utils.clip_grad_norm_(params, 1.0)
        sc.step(opt)
        sc.update()
        O.optimizer_step(states, [g.numpy() for g in gs], hp, osc, 1.0 if call_unscale else None,
                         norm=None if norm is None else np.float32(norm.item()))
        assert float(sc.get_scale()) == float(osc.scale)
        for p, st in zip(params, states):
            assert _normwise(p.detach().cpu().numpy(), st.w) <= 1e-6
            assert float(opt.state[p]["step"]) == st.step


@pytest.mark.parametrize("combo", ["ours+ours", "stock+ours", "ours+torch", "ours+mutate",
                                   "ours+replace"])
def test_scaler_and_clip_combinations(combo):
    """train.py:485-486 calls ``scaler.unscale_`` and ``torch.nn.utils.clip_grad_norm_`` by
    their full names, so a half-applied swap is easy to make.  This package's scaler leaves the
    gradients scaled; torch's clip would then rescale them in place by max_norm/(S*norm) and the
    update would apply 1/S again.  The supported pairs must match the oracle; a gradient written
    (or replaced) after this package's statistics pass must make the step raise, before any
    kernel runs."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    shapes = [(96, 64), (64,), (5,)]
    scaler_name, clip_name = combo.split("+")
    # torch's own unscale_ has no bf16 CUDA kernel, so its pairing runs on fp32 parameters (the
    # reference's fp16-autocast mode keeps fp32 parameters too)
    dtype = torch.float32 if scaler_name == "stock" else torch.bfloat16
    w0, params = _params(shapes, dtype, seed=11)
    opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)
    for p, w in zip(params, w0):
        opt.set_master_(p, w.to(DEV))
    S = 2.0 ** 12
    sc = (GradScaler if scaler_name == "ours" else torch.amp.GradScaler)("cuda", init_scale=S)
    sc.scale(torch.ones((), device=DEV))
    states = [O.TensorState(w=w.numpy().copy(), m=np.zeros(w.shape, np.float32),
                            v=np.zeros(w.shape, np.float32)) for w in w0]
    osc = O.ScalerState(scale=np.float32(S))
    hp = [O.GroupHP(1e-3, 0.9, 0.95, 1e-8, 0.1)]
    store = opt._ensure_store()
    before = [v.get("master_param", q).detach().clone()
              for v, q in zip(store.views, store.params)]
    for s in range(3):
        gs = _grads(shapes, s, dtype, S)
        for p, g in zip(params, gs):
            p.grad = g.to(DEV)
        sc.unscale_(opt)
        if clip_name == "torch":
            norm = torch.nn.utils.clip_grad_norm_(params, 1.0)
        else:
            norm = clip_grad_norm_(params, 1.0)
        if clip_name == "mutate":
            params[2].grad.mul_(2.0)
        if clip_name == "replace":
            params[1].grad = params[1].grad.clone()
        if clip_name in ("torch", "mutate", "replace"):
            with pytest.raises(RuntimeError, match="modified after"):
                sc.step(opt)
            torch.cuda.synchronize()
            for v, b in zip(store.views, before):  # nothing was launched: state untouched
                assert torch.equal(v["master_param"], b)
            assert not bool(store.steps.any())
            return
        sc.step(opt)
        sc.update()
        O.optimizer_step(states, [g.float().numpy() for g in gs], hp, osc, 1.0,
                         norm=np.float32(norm.item()))
        assert float(sc.get_scale()) == float(osc.scale)
        for p, st in zip(params, states):
            m = opt.state[p].get("master_param", p.detach()).float().cpu().numpy()
            if scaler_name == "ours":
                np.testing.assert_array_equal(m, st.w)
            else:  # torch's unscale_ rewrote the gradients first; the same values within 1e-6
                assert _normwise(m, st.w) <= 1e-6
            assert float(opt.state[p]["step"]) == st.step


def test_parameters_without_grads_are_left_alone():
    from minigpt_train_infra_b200 import FusedAdamW
    shapes = [(32, 32), (32,)]
    _, params = _params(shapes, torch.float32, seed=8)
    opt = FusedAdamW(params, lr=1e-3)
    params[0].grad = torch.randn(32, 32, device=DEV)
    before = params[1].detach().clone()
    opt.step()
    opt.step()
    assert torch.equal(params[1].detach(), before)
    assert params[1] not in opt.state
    assert float(opt.state[params[0]]["step"]) == 2.0
    sd = opt.state_dict()
    assert list(sd["state"]) == [0]


def test_rejected_configurations():
    from minigpt_train_infra_b200 import FusedAdamW
    p = torch.nn.Parameter(torch.zeros(4))
    with pytest.raises(RuntimeError, match="CUDA"):
        opt = FusedAdamW([p])
        p.grad = torch.zeros(4)
        opt.step()
    q = torch.nn.Parameter(torch.zeros(4, device=DEV))
    with pytest.raises(NotImplementedError):
        FusedAdamW([q], amsgrad=True)
    with pytest.raises(NotImplementedError):
        FusedAdamW([q], maximize=True)
    h = torch.nn.Parameter(torch.zeros(4, device=DEV, dtype=torch.float16))
    with pytest.raises(TypeError):
        opt = FusedAdamW([h])
        h.grad = torch.zeros_like(h)
        opt.step()
    with pytest.raises(ValueError):
        FusedAdamW([q], lr=-1.0)


def test_step_hooks_and_profiler_range_as_torch_provides_them():
    """torch.optim.Optimizer wraps every step with pre/post hooks and a profiler range; the
    fused optimizer keeps both (it skips the wrapper's cost only when neither is in use)."""
    from minigpt_train_infra_b200 import FusedAdamW
    shapes = [(32, 16), (16,)]
    _, params = _params(shapes, torch.float32, seed=3)
    opt = FusedAdamW(params, lr=1e-3)
    calls = []
    pre = opt.register_step_pre_hook(lambda o, a, k: calls.append(("pre", o is opt)))
    post = opt.register_step_post_hook(lambda o, a, k: calls.append(("post", o is opt)))
    for p, g in zip(params, _grads(shapes, 0, torch.float32)):
        p.grad = g.to(DEV)
    opt.step()
    assert calls == [("pre", True), ("post", True)]
    pre.remove()
    post.remove()
    opt.step()
    assert len(calls) == 2
    from torch.optim.optimizer import register_optimizer_step_pre_hook
    glob = register_optimizer_step_pre_hook(lambda o, a, k: calls.append(("global", o is opt)))
    try:
        opt.step()
    finally:
        glob.remove()
    assert calls[-1] == ("global", True)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        opt.step()
    names = {e.key for e in prof.key_averages()}
    assert "Optimizer.step#FusedAdamW.step" in names
    torch.cuda.synchronize()
    assert float(opt.state[params[0]]["step"]) == 4.0


def test_no_gradient_is_held_after_the_step():
    """A loop that frees its gradients (zero_grad(set_to_none=True), train.py:465) must get their
    memory back before the next backward: nothing of the optimizer, scaler or clip keeps a
    reference to a gradient once the step is done."""
    import gc
    import weakref
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    shapes = [(64, 32), (32,)]
    _, params = _params(shapes, torch.bfloat16, seed=8)
    opt = FusedAdamW(params, lr=1e-3)
    sc = GradScaler("cuda", init_scale=2.0 ** 8)
    sc.scale(torch.ones((), device=DEV))
    refs = []
    for s in range(3):
        for p, g in zip(params, _grads(shapes, s, torch.bfloat16, 2.0 ** 8)):
            p.grad = g.to(DEV)
        refs.append([weakref.ref(p.grad) for p in params])
        sc.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        sc.step(opt)
        sc.update()
        opt.zero_grad(set_to_none=True)
        gc.collect()
        assert all(r() is None for r in refs[-1])

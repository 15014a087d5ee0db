"""The whole optimizer step captured in a CUDA graph (``FusedAdamW(capturable=True)``).

``GradScaler.unscale_`` -> ``clip_grad_norm_`` -> ``GradScaler.step`` -> ``update`` is captured once
and replayed with a changing learning rate and new gradient values each time; the replays must
reproduce eager steps bit for bit (parameters, masters, moments, step counters, loss scale).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SHAPES = [(256, 96), (96,), (13,), (4099,)]


def _setup():
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler
    gen = torch.Generator().manual_seed(3)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in SHAPES]
    params = [torch.nn.Parameter(w.to(torch.bfloat16).to(DEV)) for w in w0]
    groups = [{"params": [params[0]], "weight_decay": 0.1},
              {"params": params[1:], "weight_decay": 0.0}]
    opt = FusedAdamW(groups, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, capturable=True)
    for p, w in zip(params, w0):
        opt.set_master_(p, w.to(DEV))
    sc = GradScaler("cuda", init_scale=2.0 ** 12, growth_interval=3)
    sc.scale(torch.ones((), device=DEV))
    grads = [torch.zeros(s, dtype=torch.bfloat16, device=DEV) for s in SHAPES]
    for p, g in zip(params, grads):
        p.grad = g
    return params, grads, opt, sc


def _new_grads(step):
    gen = torch.Generator().manual_seed(50 + step)
    gs = [(torch.randn(s, generator=gen) * 0.05 * 2.0 ** 12).to(torch.bfloat16) for s in SHAPES]
    if step == 4:
        gs[3][11] = float("inf")
    return gs


def _lr(step):
    return 1e-3 * (0.8 ** step)


def _step(params, opt, sc):
    from minigpt_train_infra_b200 import clip_grad_norm_
    sc.unscale_(opt)
    norm = clip_grad_norm_(params, 1.0)
    sc.step(opt)
    sc.update()
    return norm


def test_graph_replay_matches_eager_steps():
    pe, ge, oe, se = _setup()   # eager twin
    pg, gg, og, sg = _setup()   # graph-replayed
    # one eager step on both builds the plans (a graph cannot build them)
    for gs, grads in ((pe, ge), (pg, gg)):
        for g, v in zip(grads, _new_grads(0)):
            g.copy_(v.to(DEV))
    for g in oe.param_groups + og.param_groups:
        g["lr"] = _lr(0)
    _step(pe, oe, se)
    _step(pg, og, sg)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            norm_out = _step(pg, og, sg)
    torch.cuda.current_stream().wait_stream(side)
    norms_graph, norms_eager = [], []
    for step in range(1, 8):
        vals = _new_grads(step)
        for g, v in zip(ge, vals):
            g.copy_(v.to(DEV))
        for g, v in zip(gg, vals):
            g.copy_(v.to(DEV))
        for g in oe.param_groups + og.param_groups:
            g["lr"] = _lr(step)
        norms_eager.append(float(_step(pe, oe, se)))
        og.prepare_replay()
        graph.replay()
        norms_graph.append(float(norm_out))
    torch.cuda.synchronize()
    assert norms_graph == norms_eager
    assert float(sg.get_scale()) == float(se.get_scale())
    for a, b in zip(pe, pg):
        assert torch.equal(a, b)
        for k in ("master_param", "exp_avg", "exp_avg_sq", "step"):
            assert torch.equal(oe.state[a][k], og.state[b][k]), k
    assert float(og.state[pg[0]]["step"]) == 7.0  # 8 steps, one skipped on inf


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")  # the capture raises before launching
def test_capture_requires_a_prior_eager_step():
    params, grads, opt, sc = _setup()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with pytest.raises(RuntimeError, match="eager step"):
            with torch.cuda.graph(graph):
                _step(params, opt, sc)

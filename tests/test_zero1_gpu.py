"""ZeroAdamW on GPUs: one rank must reproduce FusedAdamW bit for bit; 2, 4 or 8 NCCL ranks (as
many as the box has GPUs) must reproduce the one-GPU result."""

from __future__ import annotations

import datetime
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(300, 129), (129,), (5,), (1024, 64), (3, 3, 3), (70001,), (0,), (4096, 33)]
# world sizes to run: every one of 2, 4, 8 that the visible GPUs allow (2 -> skipped on one GPU)
WORLDS = [w for w in (2, 4, 8) if w <= torch.cuda.device_count()] or [2]
needs_world = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


def _init(device, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(77)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in SHAPES]
    params = [torch.nn.Parameter(w.to(dtype).to(device)) for w in w0]
    groups = [{"params": [p for p, s in zip(params, SHAPES) if len(s) >= 2], "weight_decay": 0.1},
              {"params": [p for p, s in zip(params, SHAPES) if len(s) < 2], "weight_decay": 0.0,
               "lr": 1e-3}]
    return w0, params, groups


def _grads(step, dtype, device):
    gen = torch.Generator().manual_seed(500 + step)
    gs = [(torch.randn(s, generator=gen) * 0.05 * 2.0 ** 14).to(dtype) for s in SHAPES]
    if step == 3:
        gs[5][60000] = float("nan")
    return [g.to(device) for g in gs]


def _run(opt, params, scaler, device, dtype, steps=6, copy_grads=False):
    from minigpt_train_infra_b200 import clip_grad_norm_
    norms = []
    for s in range(steps):
        for p, g in zip(params, _grads(s, dtype, device)):
            if copy_grads:
                p.grad.copy_(g)
            else:
                p.grad = g
        scaler.unscale_(opt)
        norms.append(clip_grad_norm_(params, 1.0))
        scaler.step(opt)
        scaler.update()
    return [float(n) for n in norms]


def test_zero_world1_matches_fused_bit_for_bit():
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, ZeroAdamW
    device = torch.device("cuda", 0)
    results = []
    for cls in (FusedAdamW, ZeroAdamW):
        _, params, groups = _init(device)
        opt = cls(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
        sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
        sc.scale(torch.ones((), device=device))
        norms = _run(opt, params, sc, device, torch.bfloat16)
        torch.cuda.synchronize()
        results.append((norms, [p.detach().clone() for p in params], float(sc.get_scale())))
    (n0, p0, s0), (n1, p1, s1) = results
    assert s0 == s1
    np.testing.assert_array_equal(np.array(n0), np.array(n1))
    for a, b in zip(p0, p1):
        assert torch.equal(a, b)


def _nccl_worker(rank, world, port, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    import torch.distributed as dist
    from minigpt_train_infra_b200 import GradScaler, ZeroAdamW
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=device)
    try:
        _, params, groups = _init(device)
        opt = ZeroAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
        sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
        sc.scale(torch.ones((), device=device))
        norms = _run(opt, params, sc, device, torch.bfloat16, copy_grads=True)
        torch.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"nccl{rank}.npz"), norms=np.array(norms),
                 scale=float(sc.get_scale()),
                 flat=opt.flat_param.float().cpu().numpy(), steps=opt.steps.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@needs_world
@pytest.mark.parametrize("world", WORLDS)
def test_zero_nccl_ranks_match_one_gpu(tmp_path, world):
    from minigpt_train_infra_b200 import GradScaler, ZeroAdamW
    port = 29500 + os.getpid() % 1000 + world
    mp.start_processes(_nccl_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    device = torch.device("cuda", 0)
    _, params, groups = _init(device)
    opt = ZeroAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
    sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
    sc.scale(torch.ones((), device=device))
    norms = _run(opt, params, sc, device, torch.bfloat16, copy_grads=True)
    flat1 = opt.flat_param.float().cpu().numpy()
    for r in range(world):
        z = np.load(tmp_path / f"nccl{r}.npz")
        assert float(z["scale"]) == float(sc.get_scale())
        np.testing.assert_array_equal(z["steps"], opt.steps.cpu().numpy())
        for a, b in zip(z["norms"], norms):
            assert (np.isnan(a) and np.isnan(b)) or abs(a - b) <= 2 * np.spacing(np.float32(b))
        n = min(len(flat1), len(z["flat"]))
        # same values everywhere both layouts hold parameters (padding differs with the world)
        for p, off in zip(opt.params, opt.geom.offsets):
            np.testing.assert_array_equal(z["flat"][off:off + p.numel()],
                                          flat1[off:off + p.numel()])


def _local_grads(step, rank, device):
    """Per-rank gradients (different on every rank), bf16, loss-scaled."""
    gen = torch.Generator().manual_seed(900 + 17 * step + rank)
    gs = [(torch.randn(s, generator=gen) * 0.05 * 2.0 ** 14).to(torch.bfloat16) for s in SHAPES]
    if step == 2 and rank == 1:
        gs[0][3, 7] = float("nan")
    return [g.to(device) for g in gs]


def _reduced_grads(step, world, device):
    """bf16((g_0 + g_1 + ...) * (1/world)) summed in fp32 in rank order: the fused kernel's
    rule."""
    per_rank = [_local_grads(step, r, "cpu") for r in range(world)]
    out = []
    for t in range(len(SHAPES)):
        acc = per_rank[0][t].float()
        for r in range(1, world):
            acc = acc + per_rank[r][t].float()
        out.append((acc * (1.0 / world)).to(torch.bfloat16).to(device))
    return out


GAP_SENTINEL = 0x7FC1  # a bf16 NaN


def _dp_worker(rank, world, port, out_dir, peer_memory):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    import torch.distributed as dist
    from minigpt_train_infra_b200 import GradScaler, ZeroAdamW, clip_grad_norm_
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=device)
    try:
        _, params, groups = _init(device)
        opt = ZeroAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, peer_memory=peer_memory,
                        reduce_grads=True)
        # guard bands: the alignment gaps and the tail padding of both flat buffers hold a bf16
        # NaN; with peer memory no kernel may read them (the NaN would raise the inf flag) or
        # write them (they are compared afterwards), on this rank or through a peer mapping
        covered = torch.zeros(opt.geom.padded, dtype=torch.bool)
        for p, off in zip(opt.params, opt.geom.offsets):
            covered[off:off + p.numel()] = True
        gaps = (~covered).nonzero().squeeze(1).to(device)
        if peer_memory:
            opt.flat_grad.view(torch.int16)[gaps] = GAP_SENTINEL
            opt.flat_param.view(torch.int16)[gaps] = GAP_SENTINEL
            dist.barrier()
        sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
        sc.scale(torch.ones((), device=device))
        norms = []
        for s in range(5):
            for p, g in zip(params, _local_grads(s, rank, device)):
                p.grad.copy_(g)
            sc.unscale_(opt)
            norms.append(float(clip_grad_norm_(params, 1.0)))
            sc.step(opt)
            sc.update()
        torch.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"dp{rank}.npz"), norms=np.array(norms),
                 scale=float(sc.get_scale()), flat=opt.flat_param.float().cpu().numpy(),
                 steps=opt.steps.cpu().numpy(), n_gaps=gaps.numel(),
                 grad_gaps=opt.flat_grad.view(torch.int16)[gaps].cpu().numpy(),
                 param_gaps=opt.flat_param.view(torch.int16)[gaps].cpu().numpy())
        opt.close()
        if peer_memory:
            # every rank raises at the same point, before any collective of the step
            try:
                sc.unscale_(opt)
            except RuntimeError as e:
                assert "closed" in str(e)
            else:
                raise AssertionError("a step after close() must raise")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@needs_world
@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("peer_memory", [True, False])
def test_dp_reduce_scatter_step_matches_one_gpu_on_mean_grads(tmp_path, peer_memory, world):
    """Ranks with different local gradients: the fused peer-memory reduce-scatter (or NCCL's)
    plus the step must equal one GPU stepping on the averaged gradients; with peer memory the
    updated parameters reach every rank through the fused broadcast."""
    from minigpt_train_infra_b200 import GradScaler, FusedAdamW, clip_grad_norm_
    port = 29700 + os.getpid() % 1000 + 16 * world + (0 if peer_memory else 1)
    mp.start_processes(_dp_worker, args=(world, port, str(tmp_path), peer_memory), nprocs=world,
                       join=True, start_method="spawn")
    device = torch.device("cuda", 0)
    _, params, groups = _init(device)
    opt = FusedAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
    sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
    sc.scale(torch.ones((), device=device))
    norms = []
    for s in range(5):
        for p, g in zip(params, _reduced_grads(s, world, device)):
            p.grad = g
        sc.unscale_(opt)
        norms.append(float(clip_grad_norm_(params, 1.0)))
        sc.step(opt)
        sc.update()
    # the flat buffer holds the tensors in param-group order (decay group first)
    ref_flat = [p.detach().float().cpu().numpy().ravel() for g in groups for p in g["params"]]
    for r in range(world):
        z = np.load(tmp_path / f"dp{r}.npz")
        assert float(z["scale"]) == float(sc.get_scale())
        if peer_memory:
            assert int(z["n_gaps"]) > 0
            assert (z["grad_gaps"] == GAP_SENTINEL).all(), "a gradient gap was written"
            assert (z["param_gaps"] == GAP_SENTINEL).all(), "a parameter gap was written"
        # NCCL sums more than two bf16 addends with a bf16 rounding per partial sum, so its
        # reduced gradients (and the norm) differ from the fp32 rule by bf16 roundings
        loose = not peer_memory and world > 2
        for a, b in zip(z["norms"], norms):
            tol = 1e-4 * abs(b) if loose else 2 * np.spacing(np.float32(b))
            assert (np.isnan(a) and np.isnan(b)) or abs(a - b) <= tol
        off = 0
        for t, w in enumerate(ref_flat):
            n = w.size
            got = z["flat"][off:off + n]
            if peer_memory:
                np.testing.assert_array_equal(got, w)
            elif n and not loose:
                # two bf16 addends: NCCL's sum is their exact sum rounded once, as in the rule
                assert np.max(np.abs(got - w)) <= 2 ** -7 * np.max(np.abs(w)) + 1e-12
            elif n:
                # a gradient sum near zero can change sign under NCCL's roundings; four applied
                # steps (one skipped) move an element by at most about 1.5 lr each, and almost
                # every element must agree to bf16 rounding
                d = np.abs(got - w)
                assert np.max(d) <= 2 * 4 * 1.5e-3 + 1e-3
                assert np.mean(d <= 2 ** -7 * np.max(np.abs(w)) + 1e-12) >= 0.98
            off += (n + 63) // 64 * 64


@needs_world
def test_rank_leaving_between_steps_ends_the_survivors_next_step_with_an_error(tmp_path):
    """Failure detection over NCCL without a GPU fault.  Two child processes on two GPUs run
    ZeroAdamW steps with NVLS off and no peer memory.  After two completed steps the second rank
    announces in the rendezvous store that it leaves, joins a barrier (nothing of either rank in
    flight), destroys its process group and exits.  The survivor's third step must end with an
    error at once -- raised by the membership check before any collective or kernel -- rather
    than wait in a collective that can never complete."""
    import re
    import socket
    import subprocess
    import sys
    import time
    from pathlib import Path

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    worker = Path(__file__).with_name("zero_leave_worker.py")
    timeout_s = 10
    procs = [subprocess.Popen([sys.executable, str(worker), str(r), "2", str(port), str(tmp_path),
                               str(timeout_s)], env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    deadline = time.time() + 150
    outs, ended = [], []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=max(1.0, deadline - time.time()))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            logs = {f.name: f.read_text() for f in sorted(tmp_path.glob("rank*.log"))}
            pytest.fail(f"a rank was still running at the test's deadline (hang): {logs}")
        outs.append(out)
        ended.append(time.time())
    log0 = (tmp_path / "rank0.log").read_text()
    log1 = (tmp_path / "rank1.log").read_text()
    assert procs[1].returncode == 0 and "left" in log1, outs[1][-2000:]
    assert "step 1 done" in log0 and "step 2 start" in log0, log0
    assert "step 2 done" not in log0 and "all steps done" not in log0, (log0, outs[0][-3000:])
    assert procs[0].returncode == 3, (procs[0].returncode, outs[0][-3000:])
    err = next(ln for ln in log0.splitlines() if " step 2 error " in ln)
    assert re.search(r"announced that they left", err), err
    started = float(next(ln.split()[0] for ln in log0.splitlines() if ln.endswith("step 2 start")))
    assert float(err.split()[0]) - started <= 5.0, (err, started)
    assert "announced" in log1


def _reshard_worker(rank, world, port, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    import torch.distributed as dist
    from minigpt_train_infra_b200 import GradScaler, ZeroAdamW
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=device)
    try:
        _, params, groups = _init(device)
        opt = ZeroAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
        sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
        sc.scale(torch.ones((), device=device))
        _run(opt, params, sc, device, torch.bfloat16, steps=3, copy_grads=True)
        sd = opt.consolidated_state_dict()
        if rank == 0:
            torch.save({"optimizer": sd, "scaler": sc.state_dict(),
                        "params": [p.detach().cpu() for p in params]},
                       os.path.join(out_dir, "zero_ckpt.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@needs_world
def test_zero_checkpoint_from_n_ranks_resumes_on_one_gpu_bit_exactly(tmp_path):
    """The sharded checkpoint path (consolidated_state_dict) across an N -> 1 reshard on GPUs:
    N NCCL ranks take three steps (one with a NaN: skipped) and save the consolidated state in
    FusedAdamW's per-parameter layout; one GPU loads it into FusedAdamW and takes three more.
    The result equals one GPU taking all six steps, word for word."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler
    world = WORLDS[0]
    port = 29700 + os.getpid() % 1000
    mp.start_processes(_reshard_worker, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    device = torch.device("cuda", 0)
    ck = torch.load(tmp_path / "zero_ckpt.pt", weights_only=False)

    def fresh():
        _, params, groups = _init(device)
        opt = FusedAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
        sc = GradScaler("cuda", init_scale=2.0 ** 14, growth_interval=2)
        sc.scale(torch.ones((), device=device))
        return params, opt, sc

    def continue_from(params, opt, sc, start, steps):
        for s in range(start, start + steps):
            for p, g in zip(params, _grads(s, torch.bfloat16, device)):
                p.grad = g
            sc.unscale_(opt)
            from minigpt_train_infra_b200 import clip_grad_norm_
            clip_grad_norm_(params, 1.0)
            sc.step(opt)
            sc.update()

    p1, o1, s1 = fresh()
    continue_from(p1, o1, s1, 0, 6)
    p2, o2, s2 = fresh()
    with torch.no_grad():
        for p, saved in zip(p2, ck["params"]):
            p.copy_(saved)
    o2.load_state_dict(ck["optimizer"])
    s2.load_state_dict(ck["scaler"])
    s2.scale(torch.ones((), device=device))
    continue_from(p2, o2, s2, 3, 3)
    torch.cuda.synchronize()
    assert s1.get_scale() == s2.get_scale()
    for a, b in zip(p1, p2):
        assert torch.equal(a, b)
    for a, b in zip(p1, p2):
        for k in ("step", "exp_avg", "exp_avg_sq", "master_param"):
            assert torch.equal(o1.state[a][k], o2.state[b][k]), k

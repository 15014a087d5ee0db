"""ZeRO-1 host logic on gloo CPU ranks (world size 2), with the kernel math from the oracle.

Covers what the multi-GPU path adds on top of the single-GPU step: the shard geometry, the
exchange of per-slot norm partials (summed in rank order), the global skip decision when only one
rank's shard holds an inf, the in-place all-gather of the updated bf16 parameters, and a rank that
fails before the exchange (the survivor must get an error from the process-group timeout, not
hang).  The pattern -- ``torch.multiprocessing.spawn`` with a ``file://`` rendezvous -- is the one
the reference uses for its own gloo tests (``tests/test_qwen3_tp.py:207-250``).
"""

from __future__ import annotations

import datetime
import os
import tempfile
import time
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from minigpt_train_infra_b200.zero1 import ShardGeometry
from oracle import adamw_oracle as O

SHAPES = [(37, 11), (5,), (1,), (64, 40), (3, 3, 3), (130,), (0,), (2049,)]
HP = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8)


# --------------------------------------------------------------------------------------------
# pure geometry (no processes)
# --------------------------------------------------------------------------------------------

@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_every_element_exactly_once(world):
    numels = [int(np.prod(s)) for s in SHAPES] + [1 << 20, 7, 0]
    owned = np.zeros(sum(numels), dtype=np.int64)
    for r in range(world):
        g = ShardGeometry(numels, world, r)
        assert g.shard % 64 == 0 and g.lo % 64 == 0
        ranges = g.local_ranges()
        assert [s for s, _, _ in ranges] == list(range(len(numels)))  # every slot listed
        for slot, lo, hi in ranges:
            assert g.lo <= lo <= hi <= g.hi
            if hi > lo:
                off = g.offsets[slot]
                assert off <= lo and hi <= off + numels[slot]
                base = sum(numels[:slot])
                owned[base + lo - off: base + hi - off] += 1
    assert (owned == 1).all()


# --------------------------------------------------------------------------------------------
# multi-process runs
# --------------------------------------------------------------------------------------------

def _make(rank, world, dtype, init_file, timeout_s=60):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    gen = torch.Generator().manual_seed(123)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in SHAPES]
    params = [torch.nn.Parameter(w.to(dtype).clone()) for w in w0]
    return w0, params


def _grads(step, dtype, scale, inf_at=None):
    gen = torch.Generator().manual_seed(1000 + step)
    gs = [(torch.randn(s, generator=gen) * 0.05 * scale).to(dtype) for s in SHAPES]
    if inf_at is not None:
        t, i = inf_at
        gs[t].view(-1)[i] = float("inf")
    return gs


def _worker_equivalence(rank, world, init_file, out_dir, dtype_name):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    from zero_oracle_backend import OracleKernels
    from minigpt_train_infra_b200 import GradScaler, clip_grad_norm_
    from minigpt_train_infra_b200.zero1 import ZeroAdamW
    try:
        dtype = getattr(torch, dtype_name)
        w0, params = _make(rank, world, dtype, init_file)
        groups = [{"params": [p for p, s in zip(params, SHAPES) if len(s) >= 2],
                   "weight_decay": 0.1},
                  {"params": [p for p, s in zip(params, SHAPES) if len(s) < 2],
                   "weight_decay": 0.0}]
        kern = OracleKernels()
        opt = ZeroAdamW(groups, **HP, _kernels=kern)
        if dtype == torch.bfloat16:
            # masters start from the fp32 values, as a mixed-precision trainer would seed them
            for p, w in zip(params, w0):
                off = opt.geom.offsets[next(i for i, q in enumerate(opt.params) if q is p)]
                loc_lo, loc_hi = max(off, opt.geom.lo), min(off + p.numel(), opt.geom.hi)
                if loc_lo < loc_hi:
                    opt.master[loc_lo - opt.geom.lo:loc_hi - opt.geom.lo] = \
                        w.flatten()[loc_lo - off:loc_hi - off]
        scaler = GradScaler("cpu", init_scale=2.0 ** 12, growth_interval=3)
        scaler.scale(torch.ones(()))
        order = [p for g in groups for p in g["params"]]
        idx = [next(i for i, q in enumerate(params) if q is p) for p in order]
        # an inf at step 2 in the last tensor, inside the last rank's shard
        found, norms, scales = [], [], []
        for step in range(5):
            inf_at = (len(SHAPES) - 1, 2040) if step == 2 else None
            gs = _grads(step, dtype, 2.0 ** 12, inf_at)
            for p, g in zip(params, gs):
                p.grad = g
            scaler.unscale_(opt)
            norm = clip_grad_norm_(opt.managed_params(), 1.0)
            f = next(iter(scaler._per_optimizer_states[id(opt)]["found_inf_per_device"].values()))
            found.append(float(f))
            norms.append(float(norm))
            scaler.step(opt)
            scaler.update()
            scales.append(float(scaler.get_scale()))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"),
                 flat_param=opt.flat_param.float().numpy(), lo=opt.geom.lo, hi=opt.geom.hi,
                 master=opt.master.float().numpy(), exp_avg=opt.exp_avg.numpy(),
                 steps=opt.steps.numpy(), found=np.array(found), norms=np.array(norms),
                 scales=np.array(scales), idx=np.array(idx),
                 offsets=np.array(opt.geom.offsets), calls=np.array(kern.calls))
        dist.barrier()
    except Exception:
        traceback.print_exc()
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _single_process_oracle(dtype):
    """The same five steps on one process with the plain oracle chain."""
    gen = torch.Generator().manual_seed(123)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in SHAPES]
    dec = [i for i, s in enumerate(SHAPES) if len(s) >= 2]
    nod = [i for i, s in enumerate(SHAPES) if len(s) < 2]
    order = dec + nod
    groups = [O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.1), O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.0)]
    states = [O.TensorState(w=(w0[i] if dtype == torch.bfloat16 else w0[i]).numpy().copy(),
                            m=np.zeros(SHAPES[i], np.float32), v=np.zeros(SHAPES[i], np.float32),
                            group=0 if i in dec else 1) for i in order]
    sc = O.ScalerState(scale=np.float32(2.0 ** 12), growth_interval=3)
    reports = []
    for step in range(5):
        inf_at = (len(SHAPES) - 1, 2040) if step == 2 else None
        gs = _grads(step, dtype, 2.0 ** 12, inf_at)
        g32 = [gs[i].float().numpy() for i in order]
        reports.append((O.optimizer_step(states, g32, groups, sc, 1.0), float(sc.scale)))
    return order, states, reports


@pytest.mark.slow
@pytest.mark.parametrize("dtype_name,world", [("bfloat16", 2), ("float32", 2), ("bfloat16", 3)])
def test_zero1_ranks_match_single_process_oracle(tmp_path, dtype_name, world):
    init_file = tmp_path / "rdzv"
    mp.spawn(_worker_equivalence, args=(world, str(init_file), str(tmp_path), dtype_name),
             nprocs=world, join=True)
    dtype = getattr(torch, dtype_name)
    order, states, reports = _single_process_oracle(dtype)
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for r in ranks:
        # identical global decisions on every rank
        assert list(r["found"]) == [1.0 if rep.found_inf else 0.0 for rep, _ in reports]
        assert list(r["scales"]) == [s for _, s in reports]
        for (rep, _), n in zip(reports, r["norms"]):
            if np.isfinite(rep.norm):
                assert abs(n - rep.norm) <= 2 * np.spacing(np.float32(rep.norm))
            else:
                assert not np.isfinite(n)
        assert list(r["calls"][:3]) == ["grad_stats", "finalize", "adamw"]
    # every rank's gathered parameters equal the single-process result
    for r in ranks:
        offsets = r["offsets"]
        for slot, st in enumerate(states):
            off = offsets[slot]
            got = r["flat_param"][off:off + st.w.size]
            want = O.bf16_bits_to_f32(O.f32_to_bf16_bits(st.w.ravel())) \
                if dtype == torch.bfloat16 else st.w.ravel()
            np.testing.assert_array_equal(got, want)
            assert r["steps"][slot] == st.step
    # each rank's owned master / exp_avg equal the oracle's slice
    for r in ranks:
        lo, hi = int(r["lo"]), int(r["hi"])
        for slot, st in enumerate(states):
            off = int(r["offsets"][slot])
            a, b = max(off, lo), min(off + st.w.size, hi)
            if a < b:
                np.testing.assert_array_equal(r["master"][a - lo:b - lo],
                                              st.w.ravel()[a - off:b - off])
                np.testing.assert_array_equal(r["exp_avg"][a - lo:b - lo],
                                              st.m.ravel()[a - off:b - off])


def _worker_dead_peer(rank, world, init_file, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    from zero_oracle_backend import OracleKernels
    from minigpt_train_infra_b200 import GradScaler
    from minigpt_train_infra_b200.zero1 import ZeroAdamW
    _, params = _make(rank, world, torch.float32, init_file, timeout_s=5)
    opt = ZeroAdamW(params, **HP, _kernels=OracleKernels())
    scaler = GradScaler("cpu", init_scale=2.0 ** 12)
    scaler.scale(torch.ones(()))
    for p, g in zip(params, _grads(0, torch.float32, 1.0)):
        p.grad = g
    if rank == 1:
        # this rank fails before the norm exchange and never joins it
        open(os.path.join(out_dir, "rank1_failed"), "w").close()
        os._exit(3)
    t0 = time.time()
    err = ""
    try:
        scaler.unscale_(opt)  # the exchange all-gather waits for the dead rank
    except Exception as e:  # gloo raises once the process-group timeout expires
        err = f"{type(e).__name__}: {e}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{time.time() - t0:.2f}\n{err}\n")
    os._exit(0)


@pytest.mark.slow
def test_rank_failing_before_exchange_gives_bounded_error(tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, 2, str(tmp_path / "rdzv"),
                                                         str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung past the process-group timeout")
    assert (tmp_path / "rank1_failed").exists()
    secs, err = (tmp_path / "rank0.txt").read_text().split("\n", 1)
    assert err.strip(), "the surviving rank returned from the exchange without an error"
    assert float(secs) < 60.0


def _worker_announced_leave(rank, world, init_file, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    from zero_oracle_backend import OracleKernels
    from minigpt_train_infra_b200 import GradScaler, clip_grad_norm_
    from minigpt_train_infra_b200.zero1 import ZeroAdamW
    _, params = _make(rank, world, torch.float32, init_file, timeout_s=30)
    store = dist.FileStore(str(init_file) + ".members", world)
    opt = ZeroAdamW(params, **HP, membership_store=store, _kernels=OracleKernels())
    scaler = GradScaler("cpu", init_scale=2.0 ** 12)
    scaler.scale(torch.ones(()))
    for step in range(3):
        if step == 2 and rank == world - 1:
            dist.destroy_process_group()
            os._exit(0)
        for p, g in zip(params, _grads(step, torch.float32, 2.0 ** 12)):
            p.grad = g
        t0 = time.time()
        try:
            scaler.unscale_(opt)
            clip_grad_norm_(opt.managed_params(), 1.0)
            scaler.step(opt)
            scaler.update()
        except RuntimeError as e:
            with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
                f.write(f"{step}\n{time.time() - t0:.3f}\n{e}\n")
            os._exit(0)
        if step == 1:
            if rank == world - 1:
                opt.announce_leave()
            dist.barrier()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write("no error\n")
    os._exit(0)


@pytest.mark.slow
def test_announced_leave_makes_the_next_step_raise_before_any_collective(tmp_path):
    """A rank that leaves between steps announces it in the membership store before the last
    barrier; the other ranks' next step raises at once (no collective issued), at 3 ranks."""
    ctx = mp.get_context("spawn")
    world = 3
    procs = [ctx.Process(target=_worker_announced_leave,
                         args=(r, world, str(tmp_path / "rdzv"), str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    for r in range(world - 1):
        step, secs, msg = (tmp_path / f"rank{r}.txt").read_text().split("\n", 2)
        assert step == "2" and float(secs) < 5.0, (step, secs, msg)
        assert "announced that they left" in msg


# --------------------------------------------------------------------------------------------
# consolidated checkpoints and resharding (world 2 -> world 3)
# --------------------------------------------------------------------------------------------

def _worker_ckpt(rank, world, init_file, out_dir, phase):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    from zero_oracle_backend import OracleKernels
    from minigpt_train_infra_b200 import GradScaler, clip_grad_norm_
    from minigpt_train_infra_b200.zero1 import ZeroAdamW
    try:
        w0, params = _make(rank, world, torch.bfloat16, init_file)
        groups = [{"params": [p for p, s in zip(params, SHAPES) if len(s) >= 2],
                   "weight_decay": 0.1},
                  {"params": [p for p, s in zip(params, SHAPES) if len(s) < 2],
                   "weight_decay": 0.0}]
        opt = ZeroAdamW(groups, **HP, _kernels=OracleKernels())
        scaler = GradScaler("cpu", init_scale=2.0 ** 12, growth_interval=3)
        scaler.scale(torch.ones(()))
        ck_path = os.path.join(out_dir, "ckpt.pt")
        if phase == "save":
            # masters from the fp32 values (the oracle starts from them too)
            opt.load_consolidated_state_dict({
                "state": {i: {"master_param": w} for i, w in
                          enumerate([w0[j] for j in _group_order()])},
                "param_groups": [{"params": list(range(len(groups[0]["params"])))},
                                 {"params": list(range(len(groups[0]["params"]),
                                                       len(SHAPES)))}]})
            steps = range(0, 3)
        else:
            ck = torch.load(ck_path, weights_only=False)
            opt.load_consolidated_state_dict(ck["optimizer"])
            scaler.load_state_dict(ck["scaler"])  # bf16 params come from the loaded masters
            steps = range(3, 5)
        for step in steps:
            for p, g in zip(params, _grads(step, torch.bfloat16, 2.0 ** 12)):
                p.grad = g
            scaler.unscale_(opt)
            clip_grad_norm_(opt.managed_params(), 1.0)
            scaler.step(opt)
            scaler.update()
        sd = opt.consolidated_state_dict()
        if rank == 0:
            torch.save({"optimizer": sd, "scaler": scaler.state_dict()},
                       ck_path if phase == "save" else os.path.join(out_dir, "final.pt"))
        dist.barrier()
    except Exception:
        traceback.print_exc()
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _group_order():
    dec = [i for i, s in enumerate(SHAPES) if len(s) >= 2]
    nod = [i for i, s in enumerate(SHAPES) if len(s) < 2]
    return dec + nod


def _oracle_steps(n_steps):
    gen = torch.Generator().manual_seed(123)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in SHAPES]
    order = _group_order()
    groups = [O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.1), O.GroupHP(3e-4, 0.9, 0.95, 1e-8, 0.0)]
    states = [O.TensorState(w=w0[i].numpy().copy(), m=np.zeros(SHAPES[i], np.float32),
                            v=np.zeros(SHAPES[i], np.float32), group=0 if len(SHAPES[i]) >= 2
                            else 1) for i in order]
    sc = O.ScalerState(scale=np.float32(2.0 ** 12), growth_interval=3)
    for step in range(n_steps):
        gs = _grads(step, torch.bfloat16, 2.0 ** 12)
        O.optimizer_step(states, [gs[i].float().numpy() for i in order], groups, sc, 1.0)
    return states, sc


@pytest.mark.slow
def test_consolidated_checkpoint_reshards_from_two_to_three_ranks(tmp_path):
    mp.spawn(_worker_ckpt, args=(2, str(tmp_path / "rdzv2"), str(tmp_path), "save"),
             nprocs=2, join=True)
    ck = torch.load(tmp_path / "ckpt.pt", weights_only=False)["optimizer"]
    states3, _ = _oracle_steps(3)
    for slot, st in enumerate(states3):
        saved = ck["state"][slot]
        np.testing.assert_array_equal(saved["master_param"].numpy(), st.w)
        np.testing.assert_array_equal(saved["exp_avg"].numpy(), st.m)
        np.testing.assert_array_equal(saved["exp_avg_sq"].numpy(), st.v)
        assert float(saved["step"]) == st.step
    mp.spawn(_worker_ckpt, args=(3, str(tmp_path / "rdzv3"), str(tmp_path), "load"),
             nprocs=3, join=True)
    final = torch.load(tmp_path / "final.pt", weights_only=False)
    states5, sc5 = _oracle_steps(5)
    for slot, st in enumerate(states5):
        saved = final["optimizer"]["state"][slot]
        np.testing.assert_array_equal(saved["master_param"].numpy(), st.w)
        np.testing.assert_array_equal(saved["exp_avg"].numpy(), st.m)
        assert float(saved["step"]) == st.step
    assert final["scaler"]["scale"] == float(sc5.scale)

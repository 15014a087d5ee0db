"""The benchmark's multi-GPU parity leg (``bench.parity_check``), run on CPU ranks over gloo.

On the GPU box the leg checks the ZeRO-1 kernels on every rank after the timed steps.  Here the
same host logic -- sampling every owned tensor range, the oracle comparison fed the global norm,
the cross-rank check of the gathered bf16 parameters, the fp64 norm on rank 0, the +inf skip on
the last rank -- runs on two gloo ranks with the oracle standing in for the kernels, once as is
(the leg must report ok) and with a mistake planted in that stand-in (the leg must report it).
"""

from __future__ import annotations

import datetime
import json
import os
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHAPES = [(40, 24), (24,), (300,), (7,), (96, 10)]


def _worker(rank, world, init_file, out_dir, plant):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.dirname(here)]
    import bench
    from minigpt_train_infra_b200 import GradScaler
    from minigpt_train_infra_b200.zero1 import ZeroAdamW
    from zero_oracle_backend import OracleKernels

    class Planted(OracleKernels):
        def adamw(self, plan, groups, steps, found_inf, loss_scale, norm, max_norm):
            if plant == "noskip":
                found_inf = None  # update even when a gradient is not finite
            super().adamw(plan, groups, steps, found_inf, loss_scale, norm, max_norm)
            if plant == "bitflip" and rank == 1:
                plan.opt.exp_avg.view(torch.int32)[:] ^= 1  # one ulp off everywhere

        def finalize(self, exch_all, n_ranks, n_slots, out):
            super().finalize(exch_all, n_ranks, n_slots, out)
            if plant == "norm":
                out[1] = out[1] * 1.001

    try:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        params = [torch.nn.Parameter(torch.zeros(s, dtype=torch.bfloat16)) for s in SHAPES]
        groups = [{"params": [p for p in params if p.dim() >= 2], "weight_decay": 0.1},
                  {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}]
        opt = ZeroAdamW(groups, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, _kernels=Planted(),
                        defer_param_gather=True)
        gen = torch.Generator().manual_seed(1 + 101 * rank)
        opt.master.normal_(0, 0.02, generator=gen)
        opt.exp_avg.normal_(0, 1e-3, generator=gen)
        opt.exp_avg_sq.normal_(0, 1, generator=gen).abs_().mul_(1e-6)
        opt.steps.fill_(999.0)
        with torch.no_grad():
            opt.owned_param_shard().copy_(opt.master)
        opt.gather_params()
        g = torch.Generator().manual_seed(7)  # the same gradients on every rank
        opt.flat_grad.copy_((torch.randn(opt.flat_grad.numel(), generator=g) * 1e-3 * 2.0 ** 12)
                            .to(torch.bfloat16))
        opt.make_flat_grads_()
        scaler = GradScaler("cpu", init_scale=2.0 ** 12)
        scaler.scale(torch.ones(()))
        res = bench.parity_check(opt, scaler, opt.managed_params(), world, rank)
        if rank == 0:
            with open(os.path.join(out_dir, "res.json"), "w") as f:
                json.dump(res, f)
        dist.barrier()
    except Exception:
        traceback.print_exc()
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(tmp_path, plant):
    mp.spawn(_worker, args=(2, str(tmp_path / "rdzv"), str(tmp_path), plant), nprocs=2,
             join=True)
    return json.loads((tmp_path / "res.json").read_text())


@pytest.mark.slow
def test_parity_leg_reports_ok_on_correct_steps(tmp_path):
    res = _run(tmp_path, "none")
    assert res["ok"], res
    assert res["state_words_mismatched"] == 0 and res["max_ulp_diff"] == 0
    assert res["gathered_bf16_checked"] > 0 and res["gathered_bf16_mismatched"] == 0
    assert res["own_shard_bf16_vs_master_mismatched"] == 0
    assert res["samples_checked"] == sum(int(np.prod(s)) for s in SHAPES)
    assert res["norm"]["ulp_diff"] <= 2
    assert res["skip"]["found_inf_on_every_rank"]
    assert res["skip"]["state_and_steps_unchanged_on_every_rank"]
    assert res["skip"]["scale"] == [2.0 ** 12, 2.0 ** 11]


@pytest.mark.slow
@pytest.mark.parametrize("plant", ["bitflip", "noskip", "norm"])
def test_parity_leg_catches_planted_mistakes(tmp_path, plant):
    res = _run(tmp_path, plant)
    assert not res["ok"]
    if plant == "bitflip":
        assert res["state_words_mismatched"] > 0 and res["max_ulp_diff"] == 1
    if plant == "noskip":
        assert not res["skip"]["state_and_steps_unchanged_on_every_rank"]
    if plant == "norm":
        assert res["norm"]["ulp_diff"] > 2

"""The optimizers refuse a step whose gradients changed after this package's statistics pass.

``train.py:485-486`` calls ``scaler.unscale_(optimizer)`` and then
``torch.nn.utils.clip_grad_norm_`` by its full path.  With this package's ``GradScaler`` the
gradients stay scaled (the update kernel applies ``1/S``); torch's clip would rescale them in
place by ``max_norm / (S * norm)`` and the step would apply ``1/S`` a second time, clipping to
``max_norm / S`` with no error.  The version counters of the gradients expose that.  These cases
run the ZeRO-1 host logic on CPU with the oracle standing in for the kernels (one process, no
process group); the same guard in ``FusedAdamW`` is exercised on a GPU in
``test_gpu_dropin.py``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from minigpt_train_infra_b200 import GradScaler, clip_grad_norm_
from minigpt_train_infra_b200.optim import GradStats, check_stats_current
from minigpt_train_infra_b200.zero1 import ZeroAdamW
from zero_oracle_backend import OracleKernels

SHAPES = [(24, 16), (16,), (5,)]


def _setup():
    gen = torch.Generator().manual_seed(3)
    params = [torch.nn.Parameter(torch.randn(s, generator=gen) * 0.02) for s in SHAPES]
    opt = ZeroAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1,
                    _kernels=OracleKernels())
    scaler = GradScaler("cpu", init_scale=2.0 ** 8)
    scaler.scale(torch.ones(()))
    return params, opt, scaler


def _set_grads(params, step):
    gen = torch.Generator().manual_seed(50 + step)
    for p in params:
        p.grad = torch.randn(p.shape, generator=gen) * 0.1 * 2.0 ** 8


def test_supported_pairing_steps():
    params, opt, scaler = _setup()
    for step in range(3):
        _set_grads(params, step)
        scaler.unscale_(opt)
        clip_grad_norm_(opt.managed_params(), 1.0)
        scaler.step(opt)
        scaler.update()
    assert np.all(opt.steps.numpy() == 3.0)


@pytest.mark.parametrize("how", ["torch_clip", "mul_", "replace"])
def test_modified_gradients_make_the_step_raise(how):
    params, opt, scaler = _setup()
    _set_grads(params, 0)
    scaler.unscale_(opt)
    if how == "torch_clip":
        torch.nn.utils.clip_grad_norm_(opt.managed_params(), 1.0)
    else:
        clip_grad_norm_(opt.managed_params(), 1.0)
        if how == "mul_":
            params[1].grad.mul_(0.5)
        else:
            params[2].grad = params[2].grad.clone() * 2.0
    master = opt.master.clone()
    with pytest.raises(RuntimeError, match="modified after"):
        scaler.step(opt)
    assert torch.equal(opt.master, master)
    assert not bool(opt.steps.any())


def test_check_compares_versions_only_when_stats_are_pending():
    check_stats_current(None, (1, 2))
    pend = GradStats(found_inf=torch.zeros(()), norm=torch.zeros(()), loss_scale=None,
                     versions=(3,))
    check_stats_current(pend, (3,))
    with pytest.raises(RuntimeError, match="minigpt_train_infra_b200.clip_grad_norm_"):
        check_stats_current(pend, (4,))

"""``clip_grad_norm_`` with torch's signature, deferred into the fused update.

Drop-in site: ``train.py:486`` calls ``torch.nn.utils.clip_grad_norm_(model.parameters(),
grad_clip)`` and keeps the returned norm as a device tensor (``:487-489``).

When the parameters are exactly the (gradient-carrying) parameters of one
:class:`~minigpt_train_infra_b200.optim.FusedAdamW` (or of one ``ZeroAdamW``, where the norm is
the global one over all ranks), this returns the total norm the statistics
pass computed (running that pass now if ``GradScaler.unscale_`` did not) and records
``max_norm``; the update kernel then multiplies by ``clamp(max_norm / (norm + 1e-6), max=1)``
(``torch/nn/utils/clip_grad.py:165-174``) while it updates the state.  Gradients are not
rewritten.  Other parameter sets go to ``torch.nn.utils.clip_grad_norm_`` unchanged.
"""

from __future__ import annotations

from typing import Iterable

import torch

from .optim import fused_optimizers


def clip_grad_norm_(parameters: torch.Tensor | Iterable[torch.Tensor], max_norm: float,
                    norm_type: float = 2.0, error_if_nonfinite: bool = False,
                    foreach: bool | None = None) -> torch.Tensor:
    if isinstance(parameters, torch.Tensor):
        parameters = [parameters]
    params = list(parameters)
    owner = None
    for opt in fused_optimizers():
        if opt._owns_exactly(params):
            owner = opt
            break
    if owner is None:
        ids = {id(p) for p in params}
        for opt in fused_optimizers():
            if opt._pending is not None and any(
                    id(p) in ids for g in opt.param_groups for p in g["params"]):
                raise RuntimeError(
                    "clip_grad_norm_ got a parameter set that differs from its FusedAdamW's "
                    "after unscale_; pass exactly the optimizer's parameters")
        return torch.nn.utils.clip_grad_norm_(params, max_norm, norm_type, error_if_nonfinite,
                                              foreach)
    if float(norm_type) != 2.0:
        raise NotImplementedError("FusedAdamW clips by the L2 norm only")
    stats = owner._pending if owner._pending is not None else owner._grad_stats(None)
    if stats.max_norm is not None:
        raise RuntimeError("clip_grad_norm_ was already applied to these gradients in this step")
    stats.max_norm = float(max_norm)
    if error_if_nonfinite and bool(torch.logical_or(stats.norm.isnan(), stats.norm.isinf())):
        raise RuntimeError(
            f"The total norm of order {float(norm_type)} for gradients from `parameters` is "
            "non-finite, so it cannot be clipped. To disable this error and scale the gradients "
            "by the non-finite norm anyway, set `error_if_nonfinite=False`")
    return stats.norm

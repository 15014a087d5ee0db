"""``GradScaler``: ``torch.amp.GradScaler`` with the fused, sync-free path for ``FusedAdamW``.

Drop-in site: ``train.py:366-370`` (construction), ``:479`` (``scale``), ``:485`` (``unscale_``),
``:490`` (``step``), ``:491`` (``update``), ``:504`` (``get_scale``), ``checkpoint.py:42``
(``state_dict``) and ``src/minigpt/optim.py:254-273`` (``load_state_dict``).  Everything except
the three methods below is inherited unchanged, so ``state_dict`` keeps torch's five keys
(``scale, growth_factor, backoff_factor, growth_interval, _growth_tracker``).

For a :class:`~minigpt_train_infra_b200.optim.FusedAdamW` or
:class:`~minigpt_train_infra_b200.zero1.ZeroAdamW`:

* ``unscale_`` runs the read-only statistics pass (``b2o_grad_stats``): the non-finite flag and
  the L2 norm of the unscaled gradients, in one read of the gradients.  It does not rewrite
  ``param.grad``; the update kernel applies ``1/scale`` itself (torch/amp/grad_scaler.py:302-361
  rewrites the gradients in place instead).
* ``step`` passes the device ``found_inf`` straight to the optimizer (the
  ``_step_supports_amp_scaling`` contract of grad_scaler.py:418-470) without torch's extra sum.
* ``update`` runs ``b2o_scaler_update`` (one thread) instead of ``torch._amp_update_scale_``.

Other optimizers get torch's behaviour unchanged.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Any

import torch
from torch.amp.grad_scaler import OptState, _refresh_per_optimizer_state

from . import _lib
from .optim import is_fused
from .plan import stream_ptr


class GradScaler(torch.amp.GradScaler):
    def unscale_(self, optimizer: torch.optim.Optimizer) -> None:
        if not is_fused(optimizer):
            return super().unscale_(optimizer)
        if not self._enabled:
            return
        self._check_scale_growth_tracker("unscale_")
        optimizer_state = self._per_optimizer_states[id(optimizer)]
        if optimizer_state["stage"] is OptState.UNSCALED:
            raise RuntimeError(
                "unscale_() has already been called on this optimizer since the last update().")
        if optimizer_state["stage"] is OptState.STEPPED:
            raise RuntimeError("unscale_() is being called after step().")
        stats = optimizer._grad_stats(self._scale)
        optimizer_state["found_inf_per_device"] = {stats.found_inf.device: stats.found_inf}
        optimizer_state["stage"] = OptState.UNSCALED

    def step(self, optimizer: torch.optim.Optimizer, *args: Any, **kwargs: Any):
        if not is_fused(optimizer):
            return super().step(optimizer, *args, **kwargs)
        if not self._enabled:
            return optimizer.step(*args, **kwargs)
        if "closure" in kwargs:
            raise RuntimeError("Closure use is not currently supported if GradScaler is enabled.")
        self._check_scale_growth_tracker("step")
        optimizer_state = self._per_optimizer_states[id(optimizer)]
        if optimizer_state["stage"] is OptState.STEPPED:
            raise RuntimeError("step() has already been called since the last update().")
        if optimizer_state["stage"] is OptState.READY:
            self.unscale_(optimizer)
        found = list(optimizer_state["found_inf_per_device"].values())
        found_inf = found[0] if len(found) == 1 else torch.stack(
            [f.to(found[0].device) for f in found]).sum()
        optimizer.found_inf = found_inf
        try:
            retval = optimizer.step(*args, **kwargs)
        finally:
            del optimizer.found_inf
        optimizer_state["stage"] = OptState.STEPPED
        return retval

    def update(self, new_scale: float | torch.Tensor | None = None) -> None:
        if not self._enabled:
            return
        if new_scale is not None:
            return super().update(new_scale)
        _scale, _growth_tracker = self._check_scale_growth_tracker("update")
        dev = _scale.device
        found_infs = [f if f.device == dev else f.to(device=dev, non_blocking=True)
                      for state in self._per_optimizer_states.values()
                      for f in state["found_inf_per_device"].values()]
        if len(found_infs) == 0:
            raise AssertionError("No inf checks were recorded prior to update.")
        found = found_infs[0]
        for f in found_infs[1:]:
            found = found + f
        if dev.type == "cuda":
            if found.dtype != torch.float32:
                found = found.to(torch.float32)
            _lib.call("b2o_scaler_update", _scale.data_ptr(), _growth_tracker.data_ptr(),
                      found.data_ptr(), float(self._growth_factor), float(self._backoff_factor),
                      int(self._growth_interval), stream_ptr(_scale.device))
        else:
            torch._amp_update_scale_(_scale, _growth_tracker, found, self._growth_factor,
                                     self._backoff_factor, self._growth_interval)
        self._per_optimizer_states = defaultdict(_refresh_per_optimizer_state)

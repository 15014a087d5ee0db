"""``FusedAdamW``: a drop-in ``torch.optim.AdamW`` whose step runs as two sm_100a kernels.

Drop-in site: the reference builds ``torch.optim.AdamW(build_adamw_param_groups(model, wd), lr,
betas, eps, fused=...)`` at ``train.py:359-365`` and drives it through ``zero_grad`` (``:465``),
``scaler.step`` (``:490``), ``state_dict`` (``checkpoint.py:41``) and ``load_state_dict``
(``src/minigpt/optim.py:136-251``).  This class keeps that surface:

* constructor arguments and defaults of ``torch.optim.AdamW`` (``torch/optim/adamw.py``), the same
  ``param_groups`` keys (``lr, betas, eps, weight_decay, amsgrad, maximize, foreach, capturable,
  differentiable, fused, decoupled_weight_decay``) and any extra keys the caller adds
  (``param_names``, ``group_name``);
* per-parameter state ``{"step", "exp_avg", "exp_avg_sq"}`` laid out as torch lays it out, plus
  ``"master_param"`` (fp32) for bf16 parameters;
* ``_step_supports_amp_scaling = True``: ``GradScaler.step`` hands over ``found_inf`` (and, if
  the caller skipped ``unscale_``, ``grad_scale``) as device tensors, so no step synchronises the
  host (``torch/amp/grad_scaler.py:418-470``).

What is different underneath:

* master weights, moments and step counters live in flat fp32 device buffers (one allocation
  each, 256-byte aligned segments per parameter); the state entries are views into them.  Update
  an entry's tensors in place (``copy_``) or assign a whole new dict to ``optimizer.state[p]``
  (copied into the buffers at the next step, which is how the reference's loaders write state);
  rebinding a single key of an existing entry to another tensor is not seen by the kernels;
* ``GradScaler.unscale_`` and ``clip_grad_norm_`` of this package do not rewrite gradients; they
  run one read-only statistics pass (``b2o_grad_stats``) and record the loss scale and clip
  threshold, which the update kernel (``b2o_adamw_step``) applies while it updates the state --
  so ``param.grad`` still holds the scaled gradients after ``unscale_``;
* bf16 parameters are refreshed from the fp32 masters by the same kernel.

``capturable=True`` makes the step capturable in a CUDA graph: the update kernel then reads the
group hyper-parameters from a device array instead of launch arguments, and ``prepare_replay()``
stages the current lr and gradient pointers before each replay.

CUDA tensors only; there is no CPU path.  Not supported (raise): ``amsgrad``, ``maximize``,
``differentiable``, sparse gradients, fp16 parameters.
"""

from __future__ import annotations

import functools
import operator
import warnings
import weakref
from collections import defaultdict
from dataclasses import dataclass
from itertools import chain
from typing import Any

import numpy as np
import torch
from torch.optim import optimizer as _torch_optimizer

from . import _lib
from .plan import DEFAULT_CHUNK_ELEMS, ChunkPlan, Entry, dtype_code, stream_ptr

_ALIGN = 64  # elements per segment alignment: 256 bytes of fp32

_REGISTRY: weakref.WeakSet = weakref.WeakSet()


@dataclass
class GradStats:
    """Result of the statistics pass of one iteration (device tensors, no host sync)."""
    found_inf: torch.Tensor      # 0-dim fp32, 1.0 when a gradient held inf/NaN
    norm: torch.Tensor           # 0-dim fp32, total L2 norm of the unscaled gradients
    loss_scale: torch.Tensor | None
    max_norm: float | None = None
    versions: tuple = ()         # gradient signature (addresses and version counters) after it
    plans: Any = None            # the plans the pass ran on, reused by the update


_version_of = torch.Tensor._version.__get__
_data_ptr = torch.Tensor.data_ptr
_dtype_of = operator.attrgetter("dtype")


def grad_signature(grads: list) -> tuple:
    """The gradient tensors' addresses and autograd version counters, built with C-level maps
    (this runs twice per step).  A missing gradient is recorded by its position."""
    try:
        return (tuple(map(_data_ptr, grads)), tuple(map(_version_of, grads)))
    except TypeError:  # a parameter without a gradient
        act = [g for g in grads if g is not None]
        return (tuple(map(_data_ptr, act)), tuple(map(_version_of, act)),
                tuple(i for i, g in enumerate(grads) if g is None))


STALE_STATS_MESSAGE = (
    "gradients were modified after this package's GradScaler.unscale_() / clip_grad_norm_() "
    "took their statistics, so the recorded loss scale, non-finite flag and norm no longer "
    "describe them (torch.nn.utils.clip_grad_norm_, for one, rescales gradients in place: "
    "with this package's GradScaler, clip with minigpt_train_infra_b200.clip_grad_norm_ "
    "instead, or use torch.amp.GradScaler together with torch's clip)")


def check_stats_current(pend: GradStats | None, versions: tuple) -> None:
    """Raise when the gradients changed since the statistics pass of ``pend`` was launched.

    This package's ``unscale_`` leaves the gradients scaled and hands the scale to the update
    kernel; a torch ``clip_grad_norm_`` run in between multiplies them in place by
    ``max_norm / (S * norm)`` and the kernel would then apply ``1/S`` a second time -- a step
    clipped to ``max_norm / S`` with no error.  Every in-place write bumps a tensor's version
    counter, so comparing the counters catches this and any other modification.
    """
    if pend is not None and pend.versions != versions:
        raise RuntimeError(STALE_STATS_MESSAGE)


def hooked_step(func):
    """The wrapper torch.optim.Optimizer puts around every subclass's ``step``
    (``Optimizer.profile_hook_step``: step pre/post hooks and a profiler range), used only when
    a hook is registered or the profiler runs; otherwise the step is called directly, which
    saves that wrapper's fixed cost on every step of a small model."""
    slow = torch.optim.Optimizer.profile_hook_step(func)

    @functools.wraps(func)
    def wrapper(self, *args, **kwargs):
        if (self._optimizer_step_pre_hooks or self._optimizer_step_post_hooks
                or _torch_optimizer._global_optimizer_pre_hooks
                or _torch_optimizer._global_optimizer_post_hooks
                or torch._C._autograd._profiler_enabled()):
            return slow(self, *args, **kwargs)
        return func(self, *args, **kwargs)

    wrapper.hooked = True  # torch.optim.Optimizer then leaves it as it is
    return wrapper


def validate_adamw_args(lr, betas, eps, weight_decay, amsgrad, maximize, differentiable,
                        chunk_elems) -> None:
    """torch.optim.Adam's argument checks (torch/optim/adam.py:51-86) plus this package's limits."""
    if isinstance(lr, torch.Tensor):
        raise TypeError("the fused optimizers take lr as a Python float")
    if not 0.0 <= lr:
        raise ValueError(f"Invalid learning rate: {lr}")
    if not 0.0 <= eps:
        raise ValueError(f"Invalid epsilon value: {eps}")
    if not 0.0 <= betas[0] < 1.0:
        raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
    if not 0.0 <= betas[1] < 1.0:
        raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
    if not 0.0 <= weight_decay:
        raise ValueError(f"Invalid weight_decay value: {weight_decay}")
    if amsgrad or maximize or differentiable:
        raise NotImplementedError("the fused optimizers support amsgrad=False, maximize=False, "
                                  "differentiable=False only")
    if chunk_elems is not None and (chunk_elems <= 0 or chunk_elems % _lib.VEC):
        raise ValueError("chunk_elems must be a positive multiple of 8")


class FusedAdamW(torch.optim.Optimizer):
    """AdamW with decoupled weight decay, fused unscale/clip/update and bf16 param refresh."""

    _b2o_fused = True

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2, amsgrad: bool = False, *,
                 maximize: bool = False, foreach: bool | None = None, capturable: bool = False,
                 differentiable: bool = False, fused: bool | None = None,
                 chunk_elems: int | None = DEFAULT_CHUNK_ELEMS):
        validate_adamw_args(lr, betas, eps, weight_decay, amsgrad, maximize, differentiable,
                            chunk_elems)
        defaults = dict(lr=lr, betas=(float(betas[0]), float(betas[1])), eps=eps,
                        weight_decay=weight_decay, amsgrad=False, maximize=False,
                        foreach=foreach, capturable=capturable, differentiable=False,
                        fused=fused, decoupled_weight_decay=True)
        super().__init__(params, defaults)
        self._step_supports_amp_scaling = True
        self._chunk_elems = None if chunk_elems is None else int(chunk_elems)
        self._store: _FlatStore | None = None
        self._plans: list[ChunkPlan] | None = None
        self._plan_key: tuple | None = None
        self._grad_key: tuple | None = None
        self._hp_dev: torch.Tensor | None = None
        self._pending: GradStats | None = None
        self._active_ids: frozenset | None = None
        self._owns_cache: tuple | None = None
        self._group_cache: tuple | None = None
        self._last_grads: list = []
        self.state = _TrackedState(self.state)
        _REGISTRY.add(self)

    # ------------------------------------------------------------------------------------
    # torch.optim.Optimizer surface
    # ------------------------------------------------------------------------------------

    def __setstate__(self, state: dict[str, Any]) -> None:
        super().__setstate__(state)
        self.state = _TrackedState(self.state)
        for group in self.param_groups:
            group.setdefault("amsgrad", False)
            group.setdefault("maximize", False)
            group.setdefault("foreach", None)
            group.setdefault("capturable", False)
            group.setdefault("differentiable", False)
            group.setdefault("fused", None)
            group.setdefault("decoupled_weight_decay", True)

    @hooked_step
    def step(self, closure=None):
        """One AdamW update of every parameter that has a gradient.

        Applies the pending unscale factor and clip coefficient recorded by this package's
        ``GradScaler.unscale_`` / ``clip_grad_norm_`` and skips the whole update (step counters
        included) when ``self.found_inf`` -- set by ``GradScaler.step`` -- is non-zero.  No
        autograd-recorded operation runs here (the kernels write through raw pointers, state
        loads copy under no_grad), so the step needs no ``torch.no_grad`` context of its own.
        """
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        pend = self._pending
        self._pending = None
        if pend is not None:
            # the statistics pass of this iteration planned these gradients; reuse its plans
            # unless the gradients (or the plans) changed since, which makes its results stale
            self._sync_state()
            check_stats_current(pend, grad_signature([p.grad for p in self._store.params]))
            plans = pend.plans
            if plans and plans is not self._plans:
                raise RuntimeError(STALE_STATS_MESSAGE)
        else:
            plans = self._prepare()
            self._last_grads = []
        if not plans:
            return loss
        store = self._store
        device = store.device
        found_inf = getattr(self, "found_inf", None)
        if found_inf is not None and (found_inf.dtype != torch.float32 or
                                      found_inf.device != device):
            found_inf = found_inf.to(device=device, dtype=torch.float32, non_blocking=True)
        loss_scale = pend.loss_scale if pend is not None else None
        grad_scale = getattr(self, "grad_scale", None)
        if loss_scale is None and grad_scale is not None:
            loss_scale = grad_scale.to(device=device, dtype=torch.float32, non_blocking=True)
        norm = pend.norm if (pend is not None and pend.max_norm is not None) else None
        max_norm = pend.max_norm if norm is not None else 0.0
        stream = stream_ptr(device)
        fi = None if found_inf is None else found_inf.data_ptr()
        ls = None if loss_scale is None else loss_scale.data_ptr()
        nm = None if norm is None else norm.data_ptr()
        if self._capturable():
            # hyper-parameters from device memory, so a CUDA graph of this step follows lr
            # schedules; outside a capture they are staged here, before a replay by
            # prepare_replay()
            if not torch.cuda.is_current_stream_capturing():
                self.stage_hyperparams()
            hp = self._hp_dev
            for plan in plans:
                _lib.call("b2o_adamw_step_dev", plan.tensors_ptr, plan.n_tensors,
                          plan.update_chunks_ptr, plan.n_update_chunks, hp.data_ptr(),
                          len(self.param_groups), plan.grad_dtype, plan.param_dtype,
                          store.steps.data_ptr(), fi, ls, nm, float(max_norm),
                          plan.workspace.data_ptr(), stream)
            return loss
        groups = self._group_array()
        for plan in plans:
            _lib.call("b2o_adamw_step", plan.tensors_ptr, plan.n_tensors,
                      plan.update_chunks_ptr, plan.n_update_chunks, _lib.ptr(groups),
                      len(groups), plan.grad_dtype, plan.param_dtype, store.steps.data_ptr(),
                      fi, ls, nm, float(max_norm), None, plan.workspace.data_ptr(), stream)
        return loss

    # ------------------------------------------------------------------------------------
    # CUDA graphs (capturable=True)
    # ------------------------------------------------------------------------------------

    def _capturable(self) -> bool:
        return any(g.get("capturable", False) for g in self.param_groups)

    def stage_hyperparams(self) -> None:
        """Copy every group's lr/betas/eps/weight_decay to the device array the update kernel
        reads when ``capturable=True`` (ordered on the current stream; no host wait except when
        a ring buffer from three calls ago has not been consumed yet)."""
        arr = self._group_array()
        n = arr.nbytes
        if self._hp_dev is None or self._hp_dev.numel() != n:
            dev = self._ensure_store().device
            self._hp_dev = torch.empty(n, dtype=torch.uint8, device=dev)
            self._hp_ring = [torch.empty(n, dtype=torch.uint8).pin_memory() for _ in range(3)]
            self._hp_events = [None, None, None]
            self._hp_i = 0
        i = self._hp_i
        self._hp_i = (i + 1) % 3
        if self._hp_events[i] is not None:
            self._hp_events[i].synchronize()
        self._hp_ring[i].numpy()[:] = arr.view(np.uint8)
        self._hp_dev.copy_(self._hp_ring[i], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._hp_events[i] = ev

    def prepare_replay(self) -> None:
        """Before replaying a CUDA graph that captured this optimizer's step: point the device
        tables at the current gradient tensors and stage the current hyper-parameters."""
        if not self._capturable():
            raise RuntimeError("construct the optimizer with capturable=True to replay it")
        self._prepare()
        self._last_grads = []
        self.stage_hyperparams()

    def state_dict(self) -> dict[str, Any]:
        self._sync_state()
        return super().state_dict()

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Load a ``state_dict`` of this class or of ``torch.optim.AdamW``.

        Unlike ``torch.optim.Optimizer.load_state_dict`` (``torch/optim/optimizer.py``), state
        tensors are not cast to the parameter dtype: moments and masters stay fp32 under bf16
        parameters.  A state without ``master_param`` (a reference checkpoint of fp32
        parameters) initialises the master from the parameter.
        """
        state_dict = state_dict.copy()
        for pre_hook in self._optimizer_load_state_dict_pre_hooks.values():
            res = pre_hook(self, state_dict)
            if res is not None:
                state_dict = res
        groups = self.param_groups
        saved_groups = [dict(g) for g in state_dict["param_groups"]]
        if len(groups) != len(saved_groups):
            raise ValueError("loaded state dict has a different number of parameter groups")
        if any(len(g["params"]) != len(s["params"]) for g, s in zip(groups, saved_groups)):
            raise ValueError("loaded state dict contains a parameter group that doesn't match "
                             "the size of optimizer's group")
        id_map = dict(zip(chain.from_iterable(g["params"] for g in saved_groups),
                          chain.from_iterable(g["params"] for g in groups)))
        new_groups = []
        for g, s in zip(groups, saved_groups):
            s["params"] = g["params"]
            if "param_names" in g and "param_names" not in s:
                s["param_names"] = g["param_names"]
            new_groups.append(s)
        foreign = {}
        state: defaultdict = defaultdict(dict)
        for k, v in state_dict["state"].items():
            if k in id_map:
                state[id_map[k]] = dict(v)
            else:
                foreign[k] = v
        self.__setstate__({"state": state, "param_groups": new_groups})
        self.state.update(foreign)
        self._plans = None
        self._plan_key = None
        self._sync_state(force=True)
        for post_hook in self._optimizer_load_state_dict_post_hooks.values():
            post_hook(self)

    # ------------------------------------------------------------------------------------
    # Hooks used by GradScaler / clip_grad_norm_ of this package
    # ------------------------------------------------------------------------------------

    def _grad_stats(self, loss_scale: torch.Tensor | None) -> GradStats:
        """Run the read-only statistics pass over the current gradients (no host sync; no
        autograd-recorded operation)."""
        plans = self._prepare()
        store = self._store
        device = store.device if store is not None else torch.device("cuda",
                                                                     torch.cuda.current_device())
        # [found_inf, norm]; the statistics kernels write both, so no fill is needed
        out = torch.empty(2, dtype=torch.float32, device=device) if plans else \
            torch.zeros(2, dtype=torch.float32, device=device)
        if plans:
            stream = stream_ptr(device)
            ls = None
            if loss_scale is not None:
                loss_scale = loss_scale.to(device=device, dtype=torch.float32)
                ls = loss_scale.data_ptr()
            single = len(plans) == 1
            for k, plan in enumerate(plans):
                flags = (_lib.STATS_CLEAR if k == 0 else 0) | \
                    (_lib.STATS_FINALIZE if single else 0)
                _lib.call("b2o_grad_stats", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr,
                          plan.n_chunks, store.n_slots, plan.grad_dtype, ls,
                          plan.workspace.data_ptr(), store.exch.data_ptr(), flags,
                          out.data_ptr(), out.data_ptr() + 4, stream)
            if not single:
                _lib.call("b2o_finalize_norm", store.exch.data_ptr(), 1, store.n_slots,
                          out.data_ptr(), out.data_ptr() + 4, stream)
        self._pending = GradStats(found_inf=out[0], norm=out[1], loss_scale=loss_scale,
                                  versions=grad_signature(self._last_grads) if plans else
                                  (grad_signature([p.grad for p in self._store.params])
                                   if self._store is not None else ()),
                                  plans=plans)
        self._last_grads = []  # hold no gradient past this call (zero_grad may free them)
        return self._pending

    def _owns_exactly(self, params: list[torch.Tensor]) -> bool:
        key = tuple(map(id, params))
        pending = self._pending is not None and self._active_ids is not None
        cached = self._owns_cache
        if pending and cached is not None and cached[0] is self._active_ids and cached[1] == key:
            return True  # the same parameter list as last time, against the same plan
        theirs = {id(p) for p in params if p.grad is not None}
        if pending:
            # the statistics pass of this iteration just matched the plan to these gradients
            mine = self._active_ids
        else:
            mine = {id(p) for g in self.param_groups for p in g["params"] if p.grad is not None}
        owned = mine == theirs
        if owned and pending and len(theirs) == len(key):
            self._owns_cache = (self._active_ids, key)
        return owned

    def set_master_(self, param: torch.Tensor, master: torch.Tensor) -> None:
        """Overwrite the fp32 master (and the bf16 copy) of one parameter, e.g. from fp32
        weights that a bf16 model cannot hold."""
        self._sync_state()
        store = self._store
        slot = next((i for i, q in enumerate(store.params) if q is param), None)
        if slot is None:
            raise KeyError("parameter is not managed by this optimizer")
        own = store.views[slot]
        with torch.no_grad():
            if "master_param" in own:
                own["master_param"].copy_(master.reshape(param.shape))
                param.copy_(own["master_param"])
            else:
                param.copy_(master.reshape(param.shape))

    # ------------------------------------------------------------------------------------
    # internals
    # ------------------------------------------------------------------------------------

    def _group_array(self) -> np.ndarray:
        """Every group's (lr, beta1, beta2, eps, weight_decay) as the kernel's group records;
        rebuilt only when a value changed (lr usually changes every step)."""
        key = tuple((float(g["lr"]), *map(float, g["betas"]), float(g["eps"]),
                     float(g["weight_decay"])) for g in self.param_groups)
        cached = self._group_cache
        if cached is not None and cached[0] == key:
            return cached[1]
        if len(key) > _lib.MAX_GROUPS:
            raise ValueError(f"at most {_lib.MAX_GROUPS} param groups are supported")
        arr = np.array(list(key), dtype=_lib.GROUP_DTYPE)
        self._group_cache = (key, arr)
        return arr

    def _all_params(self) -> list[torch.Tensor]:
        return [p for g in self.param_groups for p in g["params"]]

    def add_param_group(self, param_group: dict[str, Any]) -> None:
        super().add_param_group(param_group)
        if getattr(self, "_store", None) is not None:
            # re-home every parameter's state in new flat buffers that include the new group
            old = self._store
            self._sync_state()
            new = _FlatStore(self._all_params())
            index = {id(p): i for i, p in enumerate(new.params)}
            for slot, p in enumerate(old.params):
                if p in self.state:
                    new.ingest(index[id(p)], old.views[slot])
                    self.state[p] = new.views[index[id(p)]]
            self._store = new
            self._plans = None
            self._plan_key = None

    def _ensure_store(self) -> "_FlatStore":
        if self._store is None:
            self._store = _FlatStore(self._all_params())
        return self._store

    def _tracked_state(self) -> "_TrackedState":
        st = self.state
        if not isinstance(st, _TrackedState):
            st = _TrackedState(st)
            self.state = st
        return st

    def _sync_state(self, force: bool = False) -> None:
        """Make every ``self.state[p]`` entry a view into the flat buffers.

        Entries written from outside (``load_state_dict`` above, or a loader that assigns
        ``optimizer.state[p] = {...}`` such as the reference's ``optim.py:242-251``) are copied
        into the flat buffers with their values cast to fp32.  The state mapping records its own
        mutations, so an unchanged mapping costs nothing here.
        """
        st = self._tracked_state()
        if not st.dirty and not force:
            return
        if not self._all_params():
            return
        store = self._ensure_store()
        for slot, p in enumerate(store.params):
            cur = st.get(p)
            own = store.views[slot]
            if cur is own:
                continue
            if cur:
                store.ingest(slot, cur)
                st[p] = own
            elif force:
                st.pop(p, None)
        st.dirty = False

    def _prepare(self) -> list[ChunkPlan] | None:
        """Refresh state views and the device plans; returns None when no grads exist.

        The plans are keyed by structure (which parameters have gradients, their addresses and
        gradient dtypes).  New gradient tensors for the same structure -- every step of a loop
        that calls zero_grad(set_to_none=True) -- only patch the gradient pointers of the
        device tensor table; the chunk tables are kept.
        """
        if self._store is None and not self._all_params():
            return None
        store = self._ensure_store()
        self._sync_state()
        params = store.params
        grads = [p.grad for p in params]
        self._last_grads = grads  # for the caller's gradient signature; it clears the list
        try:
            gptr = tuple(map(_data_ptr, grads))
        except TypeError:  # some parameters have no gradient
            gptr = None
        if gptr is not None:
            active = None
            pptr = tuple(map(_data_ptr, params))
            key = self._plan_key
            if key is not None and key[2] is None and key[0] == pptr:
                # the planned parameters, every one with a gradient: the common case
                if gptr == self._grad_key:
                    return self._plans
                if tuple(map(_dtype_of, grads)) == key[1]:
                    if torch.cuda.is_current_stream_capturing():
                        raise RuntimeError("gradient tensors changed since the last step; call "
                                           "prepare_replay() (or one eager step) before "
                                           "capturing")
                    self._refresh_grads(grads, gptr)
                    return self._plans
            skey = (pptr, tuple(map(_dtype_of, grads)), None)
            act_grads = grads
        else:
            active = [(slot, p, g) for slot, (p, g) in enumerate(zip(params, grads))
                      if g is not None]
            if not active:
                return None
            skey = (tuple(p.data_ptr() for _, p, _ in active),
                    tuple(g.dtype for _, _, g in active), tuple(s for s, _, _ in active))
            gptr = tuple(g.data_ptr() for _, _, g in active)
            act_grads = [g for _, _, g in active]
        if skey == self._plan_key:
            if gptr != self._grad_key:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("gradient tensors changed since the last step; call "
                                       "prepare_replay() (or one eager step) before capturing")
                self._refresh_grads(act_grads, gptr)
            return self._plans
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("run one eager step before capturing the optimizer in a graph")
        if active is None:
            active = [(slot, p, g) for slot, (p, g) in enumerate(zip(params, grads))]
        for _, _, g in active:
            if g.is_sparse:
                raise RuntimeError("FusedAdamW does not support sparse gradients")
        self._plans = self._build_plans(active)
        self._plan_key = skey
        self._grad_key = gptr
        self._active_ids = frozenset(id(p) for _, p, _ in active)
        st = self._tracked_state()
        for slot, p, _ in active:
            if st.get(p) is not store.views[slot]:
                st[p] = store.views[slot]
        st.dirty = False
        return self._plans

    def _refresh_grads(self, grads: list[torch.Tensor], gptr: tuple) -> None:
        for g in grads:
            if not g.is_contiguous():
                raise RuntimeError("FusedAdamW needs contiguous gradients")
        ptrs = np.asarray(gptr, dtype=np.uint64)
        for plan in self._plans:
            plan.update_grads(ptrs[plan._src])
        self._grad_refreshes = getattr(self, "_grad_refreshes", 0) + 1
        self._grad_key = gptr

    def _build_plans(self, active) -> list[ChunkPlan]:
        self._plan_builds = getattr(self, "_plan_builds", 0) + 1
        store = self._store
        gid = {}
        for gi, g in enumerate(self.param_groups):
            for p in g["params"]:
                gid[id(p)] = gi
        buckets: dict[tuple[int, int], list[Entry]] = {}
        srcs: dict[tuple[int, int], list[int]] = {}
        for k, (slot, p, g) in enumerate(active):
            if g.device != store.device or p.device != store.device:
                raise RuntimeError("FusedAdamW needs every parameter and gradient on one CUDA "
                                   "device")
            if g.shape != p.shape:
                raise RuntimeError("gradient shape does not match its parameter")
            if not g.is_contiguous() or not p.is_contiguous():
                raise RuntimeError("FusedAdamW needs contiguous parameters and gradients")
            gd, pd = dtype_code(g.dtype), dtype_code(p.dtype)
            off, n = store.offsets[slot], p.numel()
            master = store.master_ptr(slot)
            entry = Entry(grad=g.data_ptr(), param=p.data_ptr() if pd == _lib.BF16 else 0,
                          master=master, exp_avg=store.exp_avg.data_ptr() + 4 * off,
                          exp_avg_sq=store.exp_avg_sq.data_ptr() + 4 * off, numel=n,
                          group=gid[id(p)], slot=slot)
            buckets.setdefault((gd, pd), []).append(entry)
            srcs.setdefault((gd, pd), []).append(k)
        plans = []
        for key, entries in buckets.items():
            plan = ChunkPlan(store.device, entries, len(self.param_groups), store.n_slots,
                             key[0], key[1], self._chunk_elems)
            plan._src = np.asarray(srcs[key], dtype=np.int64)  # positions in the active list
            plans.append(plan)
        return plans


class _FlatStore:
    """Flat fp32 device buffers holding every parameter's optimizer state."""

    def __init__(self, params: list[torch.Tensor]):
        devs = {p.device for p in params}
        if len(devs) != 1 or next(iter(devs)).type != "cuda":
            raise RuntimeError("FusedAdamW needs every parameter on one CUDA device "
                               f"(got {sorted(map(str, devs))}); there is no CPU path")
        self.device = next(iter(devs))
        for p in params:
            if p.dtype not in (torch.bfloat16, torch.float32):
                raise TypeError(f"unsupported parameter dtype {p.dtype} (bf16 or fp32 only)")
        self.params = params
        self.n_slots = len(params)
        self.offsets = []
        self.master_offsets = []
        total = 0
        mtotal = 0
        for p in params:
            self.offsets.append(total)
            total += _round_up(p.numel(), _ALIGN)
            if p.dtype == torch.bfloat16:
                self.master_offsets.append(mtotal)
                mtotal += _round_up(p.numel(), _ALIGN)
            else:
                self.master_offsets.append(-1)
        with torch.no_grad():
            self.exp_avg = torch.zeros(max(total, 1), dtype=torch.float32, device=self.device)
            self.exp_avg_sq = torch.zeros(max(total, 1), dtype=torch.float32, device=self.device)
            self.master = torch.zeros(max(mtotal, 1), dtype=torch.float32, device=self.device)
            self.steps = torch.zeros(max(self.n_slots, 1), dtype=torch.float32, device=self.device)
            self.exch = torch.zeros(self.n_slots + 1, dtype=torch.float64, device=self.device)
            self.views = []
            for slot, p in enumerate(params):
                off, n = self.offsets[slot], p.numel()
                v = {"step": self.steps[slot],
                     "exp_avg": self.exp_avg[off:off + n].view(p.shape),
                     "exp_avg_sq": self.exp_avg_sq[off:off + n].view(p.shape)}
                if self.master_offsets[slot] >= 0:
                    mo = self.master_offsets[slot]
                    mv = self.master[mo:mo + n].view(p.shape)
                    mv.copy_(p.detach())
                    v["master_param"] = mv
                self.views.append(v)

    def master_ptr(self, slot: int) -> int:
        mo = self.master_offsets[slot]
        if mo < 0:
            return self.params[slot].data_ptr()
        return self.master.data_ptr() + 4 * mo

    @torch.no_grad()
    def ingest(self, slot: int, st: dict) -> None:
        own = self.views[slot]
        p = self.params[slot]
        if "step" in st:
            val = st["step"]
            own["step"].fill_(float(val.item() if isinstance(val, torch.Tensor) else val))
        for k in ("exp_avg", "exp_avg_sq", "master_param"):
            src = st.get(k)
            if isinstance(src, torch.Tensor) and src.dtype in (torch.bfloat16, torch.float16):
                warnings.warn(
                    f"optimizer state '{k}' arrived as {src.dtype} for a {p.dtype} parameter: it "
                    "was rounded to that dtype before it reached the optimizer (a loader that "
                    "casts state to the parameter dtype, such as the reference's "
                    "_move_optimizer_state, does this), so its fp32 value lost its low bits.  "
                    "Load through optimizer.load_state_dict() to keep optimizer state in fp32.",
                    RuntimeWarning, stacklevel=3)
        for k in ("exp_avg", "exp_avg_sq"):
            if k in st:
                own[k].copy_(st[k].reshape(p.shape))
        if "master_param" in own:
            if "master_param" in st:
                own["master_param"].copy_(st["master_param"].reshape(p.shape))
                p.copy_(own["master_param"])
            else:
                own["master_param"].copy_(p)


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class _TrackedState(defaultdict):
    """``optimizer.state`` that remembers whether anyone changed it since the optimizer last
    reconciled it with its flat buffers (torch keeps a plain ``defaultdict(dict)`` here)."""

    def __init__(self, *args):
        super().__init__(dict, *args)
        self.dirty = True

    def __reduce__(self):
        return (dict, (dict(self),))

    def __missing__(self, key):
        self.dirty = True
        return super().__missing__(key)

    def __setitem__(self, key, value):
        self.dirty = True
        super().__setitem__(key, value)

    def __delitem__(self, key):
        self.dirty = True
        super().__delitem__(key)

    def clear(self):
        self.dirty = True
        super().clear()

    def pop(self, *args):
        self.dirty = True
        return super().pop(*args)

    def popitem(self):
        self.dirty = True
        return super().popitem()

    def update(self, *args, **kwargs):
        self.dirty = True
        super().update(*args, **kwargs)

    def setdefault(self, key, default=None):
        self.dirty = True
        return super().setdefault(key, default)


def fused_optimizers() -> list:
    """Live optimizers of this package (FusedAdamW and ZeroAdamW instances)."""
    return list(_REGISTRY)


def is_fused(optimizer) -> bool:
    return bool(getattr(optimizer, "_b2o_fused", False))

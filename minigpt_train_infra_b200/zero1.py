"""``ZeroAdamW``: the fused AdamW step with ZeRO-1 sharding over the GPUs of one node.

No counterpart in the reference: its training loop is single-device (``train.py``) and its only
process-group code serves tensor-parallel inference (``src/minigpt/distributed.py:46-148``).  This
optimizer reuses that boundary's choice -- ``torch.distributed`` with NCCL, one process per GPU --
and the step kernels of this package:

* Layout.  Every parameter becomes a view into one flat buffer (``flat_param``), its gradient a
  view into a second one (``flat_grad``); each parameter's segment starts on a 64-element
  boundary and the total is padded to a multiple of ``64 * world_size``.  Rank ``r`` owns the
  contiguous range ``[r*S, (r+1)*S)`` with ``S = padded_total / world_size`` and keeps fp32
  master, ``exp_avg`` and ``exp_avg_sq`` for that range only (12 bytes per owned element).
* Step.  (1) the statistics pass over the owned gradient range writes one fp64 sum of squares
  per parameter slot plus a non-finite flag; (2) an NCCL all-gather of those ``n_slots + 1``
  doubles from every rank; (3) a one-CTA kernel sums them in rank order (the same total on
  every rank, independent of NCCL's reduction order) into the norm and ``found_inf``; (4) the
  AdamW kernel updates the owned range and writes its bf16 parameters; (5) an in-place NCCL
  all-gather of the bf16 shards refreshes ``flat_param`` on every rank.
* Skips.  ``found_inf`` is global after (3), so every rank skips or steps together; the bf16
  all-gather still runs so all ranks issue the same collectives in the same order.

``defer_param_gather=True`` leaves step (5) to an explicit :meth:`gather_params` call (for a
trainer that overlaps it with the next forward pass, or a benchmark that times it separately).

Fused collectives over peer memory (``peer_memory=True``, bf16 parameters): the flat buffers are
allocated so every rank maps every other rank's (``peer.py``, legacy CUDA IPC), and

* ``reduce_grads=True`` -- each rank's ``flat_grad`` holds its own (unreduced) gradients; the
  statistics pass becomes one kernel that reads this rank's shard range from every rank's buffer
  over NVLink, sums in fp32 in rank order, applies ``1/world_size`` (``grad_average``), writes the
  bf16 result in place and takes the statistics on it (``b2o_reduce_scatter_stats``): the
  gradient reduce-scatter of a data-parallel trainer fused with the norm partials.  Without
  ``peer_memory`` the same reduction is an NCCL ``reduce_scatter_tensor`` before the pass.
* the update kernel stores every updated bf16 value into every rank's ``flat_param``
  (``b2o_adamw_step_bcast``): step (5) fused into step (4), followed by a one-element all-reduce
  that orders the ranks.

Gradients: ``zero_grad`` zeroes ``flat_grad`` in place and keeps the views (``set_to_none`` has
no effect: the flat buffer is the gradient storage).  A gradient that autograd allocated
elsewhere is copied into the flat buffer at the next statistics pass or step.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .optim import (GradStats, _REGISTRY, _round_up, _version_of, check_stats_current,
                    validate_adamw_args)
from .plan import DEFAULT_CHUNK_ELEMS, ChunkPlan, Entry, dtype_code, stream_ptr

_ALIGN = 64
_INSTANCES = 0  # ZeroAdamW objects built in this process (names a group in the membership store)


class ShardGeometry:
    """Flat offsets of every parameter and the owned range of one rank (pure arithmetic)."""

    def __init__(self, numels: list[int], world_size: int, rank: int, align: int = _ALIGN):
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError("bad world_size / rank")
        self.numels = list(numels)
        self.offsets = []
        total = 0
        for n in numels:
            self.offsets.append(total)
            total += _round_up(n, align)
        self.total = total
        self.padded = _round_up(max(total, 1), align * world_size)
        self.shard = self.padded // world_size
        self.world_size = world_size
        self.rank = rank
        self.lo = rank * self.shard
        self.hi = self.lo + self.shard

    def local_ranges(self) -> list[tuple[int, int, int]]:
        """(slot, flat_lo, flat_hi) of every parameter clipped to the owned range; empty
        ranges are kept (lo == hi) so every rank's table lists every slot."""
        out = []
        for slot, (off, n) in enumerate(zip(self.offsets, self.numels)):
            lo, hi = max(off, self.lo), min(off + n, self.hi)
            out.append((slot, lo, hi) if lo < hi else (slot, self.lo, self.lo))
        return out

    def owned_numel(self) -> int:
        return sum(hi - lo for _, lo, hi in self.local_ranges())


class CudaKernels:
    """The product backend: the sm_100a kernels of ``lib/libb200_optim.so``."""

    def make_plan(self, opt: "ZeroAdamW", ranges) -> ChunkPlan:
        esz = opt.flat_param.element_size()
        gd = dtype_code(opt.flat_grad.dtype)
        pd = dtype_code(opt.flat_param.dtype)
        entries = []
        for slot, lo, hi in ranges:
            n = hi - lo
            loc = lo - opt.geom.lo
            if n == 0:
                entries.append(Entry(0, 0, 0, 0, 0, 0, opt._slot_group[slot], slot))
                continue
            master = (opt.master.data_ptr() + 4 * loc) if pd == _lib.BF16 else \
                opt.flat_param.data_ptr() + esz * lo
            entries.append(Entry(
                grad=opt.flat_grad.data_ptr() + opt.flat_grad.element_size() * lo,
                param=opt.flat_param.data_ptr() + esz * lo if pd == _lib.BF16 else 0,
                master=master, exp_avg=opt.exp_avg.data_ptr() + 4 * loc,
                exp_avg_sq=opt.exp_avg_sq.data_ptr() + 4 * loc, numel=n,
                group=opt._slot_group[slot], slot=slot))
        return ChunkPlan(opt.device, entries, len(opt.param_groups), opt.n_slots, gd, pd,
                         opt._chunk_elems)

    def grad_stats(self, plan: ChunkPlan, loss_scale, exch_local: torch.Tensor) -> None:
        _lib.call("b2o_grad_stats", plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr,
                  plan.n_chunks, plan.n_slots, plan.grad_dtype,
                  None if loss_scale is None else loss_scale.data_ptr(),
                  plan.workspace.data_ptr(), exch_local.data_ptr(), _lib.STATS_CLEAR, None, None,
                  stream_ptr(plan.device))

    def finalize(self, exch_all: torch.Tensor, n_ranks: int, n_slots: int,
                 out: torch.Tensor) -> None:
        _lib.call("b2o_finalize_norm", exch_all.data_ptr(), n_ranks, n_slots, out.data_ptr(),
                  out.data_ptr() + 4, stream_ptr(out.device))

    def adamw(self, plan: ChunkPlan, groups: np.ndarray, steps: torch.Tensor, found_inf,
              loss_scale, norm, max_norm: float) -> None:
        _lib.call("b2o_adamw_step", plan.tensors_ptr, plan.n_tensors, plan.update_chunks_ptr,
                  plan.n_update_chunks, _lib.ptr(groups), len(groups), plan.grad_dtype,
                  plan.param_dtype, steps.data_ptr(),
                  None if found_inf is None else found_inf.data_ptr(),
                  None if loss_scale is None else loss_scale.data_ptr(),
                  None if norm is None else norm.data_ptr(), float(max_norm), None,
                  plan.workspace.data_ptr(), stream_ptr(plan.device))

    def reduce_scatter_stats(self, plan: ChunkPlan, peer_grads, n_ranks: int, my_base: int,
                             scale_factor: float, loss_scale, exch_local: torch.Tensor) -> None:
        _lib.call("b2o_reduce_scatter_stats", peer_grads, n_ranks, my_base, float(scale_factor),
                  plan.tensors_ptr, plan.n_tensors, plan.chunks_ptr, plan.n_chunks, plan.n_slots,
                  None if loss_scale is None else loss_scale.data_ptr(),
                  plan.workspace.data_ptr(), exch_local.data_ptr(), stream_ptr(plan.device))

    def adamw_bcast(self, plan: ChunkPlan, groups: np.ndarray, steps: torch.Tensor, found_inf,
                    loss_scale, norm, max_norm: float, peer_params, n_ranks: int, my_rank: int,
                    my_base: int) -> None:
        _lib.call("b2o_adamw_step_bcast", plan.tensors_ptr, plan.n_tensors,
                  plan.update_chunks_ptr, plan.n_update_chunks, _lib.ptr(groups), len(groups),
                  plan.grad_dtype, steps.data_ptr(),
                  None if found_inf is None else found_inf.data_ptr(),
                  None if loss_scale is None else loss_scale.data_ptr(),
                  None if norm is None else norm.data_ptr(), float(max_norm), peer_params,
                  n_ranks, my_rank, my_base, plan.workspace.data_ptr(), stream_ptr(plan.device))


class ZeroAdamW(torch.optim.Optimizer):
    """ZeRO-1 sharded :class:`FusedAdamW` (same constructor arguments plus the group)."""

    _b2o_fused = True

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2, amsgrad: bool = False, *,
                 maximize: bool = False, foreach: bool | None = None, capturable: bool = False,
                 differentiable: bool = False, fused: bool | None = None,
                 process_group=None, chunk_elems: int | None = DEFAULT_CHUNK_ELEMS,
                 defer_param_gather: bool = False, peer_memory: bool = False,
                 reduce_grads: bool = False, grad_average: bool = True, membership_store=None,
                 _kernels=None):
        validate_adamw_args(lr, betas, eps, weight_decay, amsgrad, maximize, differentiable,
                            chunk_elems)
        defaults = dict(lr=lr, betas=(float(betas[0]), float(betas[1])), eps=eps,
                        weight_decay=weight_decay, amsgrad=False, maximize=False,
                        foreach=foreach, capturable=capturable, differentiable=False,
                        fused=fused, decoupled_weight_decay=True)
        super().__init__(params, defaults)
        self._step_supports_amp_scaling = True
        self._chunk_elems = None if chunk_elems is None else int(chunk_elems)
        self.defer_param_gather = defer_param_gather
        if process_group is None and dist.is_available() and dist.is_initialized():
            process_group = dist.group.WORLD
        self.pg = process_group
        self.world_size = dist.get_world_size(process_group) if process_group is not None else 1
        self.rank = dist.get_rank(process_group) if process_group is not None else 0
        plist = [p for g in self.param_groups for p in g["params"]]
        if not plist:
            raise ValueError("ZeroAdamW got no parameters")
        devs = {p.device for p in plist}
        dts = {p.dtype for p in plist}
        if len(devs) != 1 or len(dts) != 1:
            raise RuntimeError("ZeroAdamW needs every parameter on one device with one dtype")
        self.device = next(iter(devs))
        dtype = next(iter(dts))
        dtype_code(dtype)
        self._kernels = _kernels if _kernels is not None else CudaKernels()
        if _kernels is None and self.device.type != "cuda":
            raise RuntimeError("ZeroAdamW runs on CUDA devices only; there is no CPU path")
        # Host-side membership check (opt-in): a rank that leaves between steps announces it in
        # this torch.distributed Store, and every rank looks before its step's first collective,
        # so the others end their next step with an error instead of waiting in a collective.
        # All ranks build their ZeroAdamW objects in the same order, so the count of objects
        # built in this process names the same group on every rank.
        global _INSTANCES
        _INSTANCES += 1
        self._members = membership_store
        self._members_key = f"b2o_zero1/{_INSTANCES}/left"
        self.peer_memory = bool(peer_memory) and self.world_size > 1
        self.reduce_grads = bool(reduce_grads)
        self.grad_scale_factor = 1.0 / self.world_size if grad_average else 1.0
        if self.peer_memory and _kernels is not None:
            raise ValueError("peer_memory needs the CUDA kernels")
        if self.reduce_grads and self.peer_memory and dtype != torch.bfloat16:
            raise NotImplementedError("the fused reduce-scatter takes bf16 gradients")
        self.params = plist
        self.n_slots = len(plist)
        self._slot_group = [gi for gi, g in enumerate(self.param_groups) for _ in g["params"]]
        self.geom = ShardGeometry([p.numel() for p in plist], self.world_size, self.rank)
        S = self.geom.shard
        with torch.no_grad():
            self._peer_bufs = []
            if self.peer_memory:
                from .peer import PeerBuffer
                pb = PeerBuffer(self.geom.padded, dtype, self.device, process_group)
                gb = PeerBuffer(self.geom.padded, dtype, self.device, process_group)
                self._peer_bufs = [pb, gb]
                self.flat_param, self.flat_grad = pb.local, gb.local
                self.flat_param.zero_()
                self.flat_grad.zero_()
            else:
                self.flat_param = torch.zeros(self.geom.padded, dtype=dtype, device=self.device)
                self.flat_grad = torch.zeros(self.geom.padded, dtype=dtype, device=self.device)
            self._bar = torch.zeros(1, dtype=torch.float32, device=self.device)
            self._grad_views = []
            for p, off in zip(plist, self.geom.offsets):
                view = self.flat_param[off:off + p.numel()].view(p.shape)
                view.copy_(p.detach())
                p.data = view
                self._grad_views.append(self.flat_grad[off:off + p.numel()].view(p.shape))
            own = self.flat_param[self.geom.lo:self.geom.hi]
            if dtype == torch.bfloat16:
                self.master = own.float()
            else:
                self.master = own  # fp32 parameters are their own masters
            self.exp_avg = torch.zeros(S, dtype=torch.float32, device=self.device)
            self.exp_avg_sq = torch.zeros(S, dtype=torch.float32, device=self.device)
            self.steps = torch.zeros(self.n_slots, dtype=torch.float32, device=self.device)
            self.exch_local = torch.zeros(self.n_slots + 1, dtype=torch.float64,
                                          device=self.device)
            self.exch_all = torch.zeros(self.world_size * (self.n_slots + 1), dtype=torch.float64,
                                        device=self.device)
        for p, v in zip(plist, self._grad_views):
            p.grad = v
        self._plan = self._kernels.make_plan(self, self.geom.local_ranges())
        self._plans = [self._plan]
        self._pending: GradStats | None = None
        _REGISTRY.add(self)

    # ------------------------------------------------------------------------------------
    # helpers used by the benchmark and by trainers
    # ------------------------------------------------------------------------------------

    def managed_params(self) -> list[torch.Tensor]:
        return list(self.params)

    def make_flat_grads_(self) -> list[torch.Tensor]:
        for p, v in zip(self.params, self._grad_views):
            p.grad = v
        return list(self._grad_views)

    def local_numel(self) -> int:
        return self.geom.owned_numel()

    def owned_param_shard(self) -> torch.Tensor:
        return self.flat_param[self.geom.lo:self.geom.hi]

    def gather_params(self) -> None:
        """Refresh every rank's ``flat_param`` with the other ranks' updated shards (with
        ``peer_memory`` the update kernel already stored them; this only orders the ranks)."""
        if self.world_size > 1:
            if self.peer_memory:
                self._barrier()
            else:
                dist.all_gather_into_tensor(self.flat_param, self.owned_param_shard(),
                                            group=self.pg)

    def announce_leave(self) -> None:
        """Called by a rank that is about to leave the group between steps (needs
        ``membership_store``).  Call it after its last step and before a last barrier with the
        other ranks, then exit: the barrier orders the announcement before their next step,
        whose membership check then raises before any collective or kernel is issued."""
        if self._members is None:
            raise RuntimeError("announce_leave needs ZeroAdamW(membership_store=...)")
        self._members.add(self._members_key, 1)

    def _check_members(self) -> None:
        if self._members is not None:
            left = self._members.add(self._members_key, 0)
            if left:
                raise RuntimeError(
                    f"{left} rank(s) of this ZeroAdamW group announced that they left; the step "
                    "was not started (no collective or kernel issued).  Rebuild the process "
                    "group and the optimizer, e.g. from consolidated_state_dict()")

    def _barrier(self) -> None:
        """Stream-ordered rendezvous: returns (on the stream) once every rank's earlier work
        on its stream has completed.  A one-element all-reduce, no host blocking."""
        dist.all_reduce(self._bar, group=self.pg)

    def close(self) -> None:
        """Release the peer mappings (with ``peer_memory``); call on every rank.  A step after
        this raises instead of launching kernels on the released mappings."""
        if self._peer_bufs:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.pg)
            for b in self._peer_bufs:
                b.close()
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.pg)

    # ------------------------------------------------------------------------------------
    # torch.optim.Optimizer surface
    # ------------------------------------------------------------------------------------

    def zero_grad(self, set_to_none: bool = True) -> None:
        with torch.no_grad():
            self.flat_grad.zero_()
        for p, v in zip(self.params, self._grad_views):
            p.grad = v

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._pending is None:
            self._check_members()
        self._adopt_grads()
        pend = self._pending
        self._pending = None
        if pend is not None:
            # every gradient is a view of flat_grad and shares its version counter; a gradient
            # tensor replaced since the statistics pass was copied in just now, which bumps it
            check_stats_current(pend, (_version_of(self.flat_grad),))
        found_inf = getattr(self, "found_inf", None)
        if found_inf is not None:
            found_inf = found_inf.to(device=self.device, dtype=torch.float32)
        loss_scale = pend.loss_scale if pend is not None else None
        grad_scale = getattr(self, "grad_scale", None)
        if loss_scale is None and grad_scale is not None:
            loss_scale = grad_scale.to(device=self.device, dtype=torch.float32)
        norm = pend.norm if (pend is not None and pend.max_norm is not None) else None
        max_norm = pend.max_norm if norm is not None else 0.0
        if self.peer_memory:
            # the update stores every new bf16 value into every rank's parameter buffer; the
            # norm exchange before it already ordered all ranks past their backward passes
            pb = self._peer_bufs[0]
            self._kernels.adamw_bcast(self._plan, self._group_array(), self.steps, found_inf,
                                      loss_scale, norm, max_norm, pb.ptr_array, self.world_size,
                                      self.rank, pb.local.data_ptr())
        else:
            self._kernels.adamw(self._plan, self._group_array(), self.steps, found_inf,
                                loss_scale, norm, max_norm)
        if not self.defer_param_gather:
            self.gather_params()
        return loss

    def state_dict(self) -> dict[str, Any]:
        """This rank's shard: the reference's param_groups plus the owned fp32 state."""
        groups = []
        idx = 0
        for g in self.param_groups:
            packed = {k: v for k, v in g.items() if k != "params"}
            packed["params"] = list(range(idx, idx + len(g["params"])))
            idx += len(g["params"])
            groups.append(packed)
        return {"state": {}, "param_groups": groups,
                "zero1": {"world_size": self.world_size, "rank": self.rank,
                          "shard": [self.geom.lo, self.geom.hi],
                          "numels": self.geom.numels,
                          "master": self.master.detach().clone(),
                          "exp_avg": self.exp_avg.detach().clone(),
                          "exp_avg_sq": self.exp_avg_sq.detach().clone(),
                          "steps": self.steps.detach().clone()}}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        z = state_dict.get("zero1")
        if z is None:
            raise ValueError("not a ZeroAdamW shard state_dict")
        if z["world_size"] != self.world_size or list(z["shard"]) != [self.geom.lo, self.geom.hi] \
                or list(z["numels"]) != self.geom.numels:
            raise ValueError("shard layout differs (world size or parameter list changed)")
        for g, s in zip(self.param_groups, state_dict["param_groups"]):
            for k, v in s.items():
                if k != "params":
                    g[k] = v
        with torch.no_grad():
            self.master.copy_(z["master"])
            self.exp_avg.copy_(z["exp_avg"])
            self.exp_avg_sq.copy_(z["exp_avg_sq"])
            self.steps.copy_(z["steps"])
            if self.flat_param.dtype == torch.bfloat16:
                self.owned_param_shard().copy_(self.master)
        self.gather_params()

    def consolidated_state_dict(self, to_rank: int = 0,
                                piece_elems: int = 1 << 26) -> dict[str, Any] | None:
        """The whole optimizer state in FusedAdamW's (torch AdamW's) per-parameter layout, on
        rank ``to_rank`` (CPU tensors); None on the other ranks.  Call on every rank.

        The owned fp32 ranges are gathered in pieces of ``piece_elems`` elements per rank, so
        the device holds at most ``world_size * piece_elems`` extra floats at a time.  The
        result is what the reference's single-file checkpoint stores (``checkpoint.py:41``) and
        loads into :class:`FusedAdamW` on one GPU or into a ZeroAdamW of any world size
        (:meth:`load_consolidated_state_dict`).
        """
        g = self.geom
        me = self.rank == to_rank
        names = ["master", "exp_avg", "exp_avg_sq"]
        full = {k: torch.empty(g.padded, dtype=torch.float32) for k in names} if me else None
        for k in names:
            local = getattr(self, k).detach()
            if local.dtype != torch.float32:
                local = local.float()
            for a in range(0, g.shard, piece_elems):
                b = min(a + piece_elems, g.shard)
                piece = local[a:b].contiguous()
                if self.world_size == 1:
                    parts = [piece]
                else:
                    parts = [torch.empty_like(piece) for _ in range(self.world_size)] if me \
                        else None
                    dist.gather(piece, parts, dst=to_rank, group=self.pg)
                if me:
                    for r, part in enumerate(parts):
                        full[k][r * g.shard + a:r * g.shard + b].copy_(part.cpu())
        steps = self.steps.detach().cpu()
        if not me:
            return None
        state = {}
        groups = []
        slot = 0
        for gi, grp in enumerate(self.param_groups):
            packed = {k: v for k, v in grp.items() if k != "params"}
            packed["params"] = list(range(slot, slot + len(grp["params"])))
            groups.append(packed)
            for p in grp["params"]:
                off, n = g.offsets[slot], g.numels[slot]
                st = {"step": steps[slot].clone(),
                      "exp_avg": full["exp_avg"][off:off + n].view(p.shape),
                      "exp_avg_sq": full["exp_avg_sq"][off:off + n].view(p.shape)}
                if self.flat_param.dtype == torch.bfloat16:
                    st["master_param"] = full["master"][off:off + n].view(p.shape)
                state[slot] = st
                slot += 1
        return {"state": state, "param_groups": groups}

    def load_consolidated_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Take this rank's range from a per-parameter state dict (from
        :meth:`consolidated_state_dict` at any world size, from ``FusedAdamW.state_dict()`` or
        from ``torch.optim.AdamW.state_dict()``).  Call on every rank with the same dict."""
        g = self.geom
        saved_groups = state_dict["param_groups"]
        if len(saved_groups) != len(self.param_groups) or any(
                len(a["params"]) != len(b["params"])
                for a, b in zip(saved_groups, self.param_groups)):
            raise ValueError("state dict groups do not match this optimizer's parameter groups")
        for grp, saved in zip(self.param_groups, saved_groups):
            for k, v in saved.items():
                if k != "params":
                    grp[k] = v
        ids = [i for grp in saved_groups for i in grp["params"]]
        bf16 = self.flat_param.dtype == torch.bfloat16
        with torch.no_grad():
            for slot, sid in enumerate(ids):
                st = state_dict["state"].get(sid)
                off, n = g.offsets[slot], g.numels[slot]
                lo, hi = max(off, g.lo), min(off + n, g.hi)
                if not st:
                    continue
                if "step" in st:
                    v = st["step"]
                    self.steps[slot] = float(v.item() if isinstance(v, torch.Tensor) else v)
                if lo >= hi:
                    continue
                a, b = lo - off, hi - off
                la, lb = lo - g.lo, hi - g.lo
                for key, dst in (("exp_avg", self.exp_avg), ("exp_avg_sq", self.exp_avg_sq)):
                    if key in st:
                        dst[la:lb].copy_(st[key].reshape(-1)[a:b])
                if "master_param" in st:
                    self.master[la:lb].copy_(st["master_param"].reshape(-1)[a:b])
                elif bf16:
                    self.master[la:lb].copy_(self.flat_param[lo:hi])
            if bf16:
                self.owned_param_shard().copy_(self.master)
        self.gather_params()

    # ------------------------------------------------------------------------------------
    # GradScaler / clip_grad_norm_ hooks
    # ------------------------------------------------------------------------------------

    @torch.no_grad()
    def _grad_stats(self, loss_scale: torch.Tensor | None) -> GradStats:
        self._check_members()
        self._adopt_grads()
        if loss_scale is not None:
            loss_scale = loss_scale.to(device=self.device, dtype=torch.float32)
        out = torch.empty(2, dtype=torch.float32, device=self.device)  # finalize writes both
        if self.reduce_grads and self.world_size > 1:
            if self.peer_memory:
                gb = self._peer_bufs[1]
                peers = gb.ptr_array  # raises after close(), before any collective is issued
                self._barrier()  # every rank's gradients are complete
                self._kernels.reduce_scatter_stats(self._plan, peers, self.world_size,
                                                   gb.local.data_ptr(), self.grad_scale_factor,
                                                   loss_scale, self.exch_local)
            else:
                shard = self.flat_grad[self.geom.lo:self.geom.hi]
                dist.reduce_scatter_tensor(shard, self.flat_grad, group=self.pg)
                if self.grad_scale_factor != 1.0:
                    shard.mul_(self.grad_scale_factor)
                self._kernels.grad_stats(self._plan, loss_scale, self.exch_local)
        else:
            self._kernels.grad_stats(self._plan, loss_scale, self.exch_local)
        if self.world_size > 1:
            dist.all_gather_into_tensor(self.exch_all, self.exch_local, group=self.pg)
            exch = self.exch_all
        else:
            exch = self.exch_local
        self._kernels.finalize(exch, self.world_size, self.n_slots, out)
        self._pending = GradStats(found_inf=out[0], norm=out[1], loss_scale=loss_scale,
                                  versions=(_version_of(self.flat_grad),))
        return self._pending

    def _owns_exactly(self, params) -> bool:
        mine = {id(p) for p in self.params}
        theirs = {id(p) for p in params if p.grad is not None}
        return mine == theirs

    def _adopt_grads(self) -> None:
        for i, (p, v) in enumerate(zip(self.params, self._grad_views)):
            g = p.grad
            if g is v:
                continue
            if g is None:
                raise RuntimeError("ZeroAdamW needs a gradient for every parameter")
            with torch.no_grad():
                v.copy_(g)
            p.grad = v

    def _group_array(self) -> np.ndarray:
        arr = np.zeros(len(self.param_groups), dtype=_lib.GROUP_DTYPE)
        if len(arr) > _lib.MAX_GROUPS:
            raise ValueError(f"at most {_lib.MAX_GROUPS} param groups are supported")
        for i, g in enumerate(self.param_groups):
            b1, b2 = g["betas"]
            arr[i] = (float(g["lr"]), float(b1), float(b2), float(g["eps"]),
                      float(g["weight_decay"]))
        return arr

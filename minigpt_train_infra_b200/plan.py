"""Multi-tensor-apply launcher: device-side tensor and chunk tables for the step kernels.

The reference hands PyTorch lists of tensors every step (``torch/amp/grad_scaler.py:294``,
``torch/optim/adam.py:880``) and ATen re-chunks them into kernel-argument structs on every call.
Here a :class:`ChunkPlan` packs each tensor's pointers (grad, bf16 param, fp32 master, exp_avg,
exp_avg_sq), its element count, param-group and step slot, plus two chunk tables, into one
device buffer (``b2o_plan_chunks`` in ``csrc/b2o_plan.cu`` does the packing and validation):

* the statistics pass reads 128 Ki-element chunks (64 Ki in plans of at most 2**29 elements),
  also handed out in order, and writes one fp64 partial per chunk;
* the update pass hands out 2 Ki-element chunks in order from a counter, which keeps every
  CTA inside one compact window of each array (measured: coarser or statically assigned chunks
  lose 5-10% of DRAM bandwidth to row misses).

The plan is built once per parameter set and reused while the pointers are unchanged, so a step
costs only the kernel launches.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

STATS_CHUNK_ELEMS = 1 << 17   # statistics pass: one fp64 partial per 128 Ki elements ...
STATS_CHUNK_ELEMS_SMALL = 1 << 16  # ... or per 64 Ki for plans of at most 2**29 elements
STATS_SMALL_PLAN_ELEMS = 1 << 29
UPDATE_CHUNK_ELEMS = 1 << 11  # update pass: 2 Ki elements = one loop iteration of a CTA
DEFAULT_CHUNK_ELEMS = None    # None = the two defaults above

_DTYPE_CODE = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; gradients/params must be bf16 or fp32") from None


@dataclass
class Entry:
    """One tensor slice as the kernels see it (all device addresses)."""
    grad: int
    param: int           # 0 when parameters are fp32 (the master is the parameter)
    master: int
    exp_avg: int
    exp_avg_sq: int
    numel: int
    group: int
    slot: int


def _plan_chunks(lib, host_t: np.ndarray, n_groups: int, n_slots: int, chunk_elems: int,
                 grad_dtype: int) -> np.ndarray:
    n = len(host_t)
    n_chunks = np.zeros(1, dtype=np.int64)
    _lib.check("b2o_plan_chunks", lib.b2o_plan_chunks(
        _lib.ptr(host_t), n, n_groups, n_slots, chunk_elems, grad_dtype, None, 0,
        _lib.ptr(n_chunks)))
    host_c = np.zeros(int(n_chunks[0]), dtype=_lib.CHUNK_DTYPE)
    _lib.check("b2o_plan_chunks", lib.b2o_plan_chunks(
        _lib.ptr(host_t), n, n_groups, n_slots, chunk_elems, grad_dtype,
        _lib.ptr(host_c) if host_c.size else None, host_c.size, _lib.ptr(n_chunks)))
    return host_c


class ChunkPlan:
    """Device tables (tensor entries + stats chunks + update chunks) and the stats workspace
    for one dtype bucket.

    ``chunk_elems`` overrides both chunk sizes (tests use tiny chunks to cross many chunk
    boundaries); by default the statistics pass uses 128 Ki elements (64 Ki for plans of at most
    2**29 elements) and the update pass 2 Ki.
    """

    def __init__(self, device: torch.device, entries: list[Entry], n_groups: int, n_slots: int,
                 grad_dtype: int, param_dtype: int, chunk_elems: int | None = None,
                 workspace: torch.Tensor | None = None):
        lib = _lib.load()
        self.device = device
        self.grad_dtype = grad_dtype
        self.param_dtype = param_dtype
        self.n_groups = n_groups
        self.n_slots = n_slots
        # Smaller plans take smaller statistics chunks, so that several chunks per CTA even out
        # the ragged tensor ends (measured on B200: GPT-2 124M's pass 74 -> 68 us).
        total = sum(e.numel for e in entries)
        self.stats_chunk_elems = chunk_elems or (
            STATS_CHUNK_ELEMS_SMALL if total <= STATS_SMALL_PLAN_ELEMS else STATS_CHUNK_ELEMS)
        self.update_chunk_elems = chunk_elems or UPDATE_CHUNK_ELEMS
        self.chunk_elems = self.stats_chunk_elems
        n = len(entries)
        host_t = np.zeros(n, dtype=_lib.TENSOR_DTYPE)
        for i, e in enumerate(entries):
            host_t[i] = (e.grad, e.param, e.master, e.exp_avg, e.exp_avg_sq, e.numel, e.group,
                         e.slot, 0, 0, 0, 0)
        # The update table first; the stats table second, so the per-tensor chunk ranges left in
        # the tensor entries are the stats pass's (only its final fold reads them).
        host_u = _plan_chunks(lib, host_t, n_groups, n_slots, self.update_chunk_elems, grad_dtype)
        host_s = _plan_chunks(lib, host_t, n_groups, n_slots, self.stats_chunk_elems, grad_dtype)
        self.n_tensors = n
        self.n_chunks = len(host_s)
        self.n_update_chunks = len(host_u)
        self.host_tensors = host_t
        # One device buffer: [tensor table | stats chunks | update chunks], 256-byte aligned.
        t_bytes = _round_up(host_t.nbytes, 256)
        s_bytes = _round_up(host_s.nbytes, 256)
        u_bytes = _round_up(host_u.nbytes, 256)
        blob = np.zeros(t_bytes + s_bytes + u_bytes, dtype=np.uint8)
        blob[:host_t.nbytes] = host_t.view(np.uint8)
        blob[t_bytes:t_bytes + host_s.nbytes] = host_s.view(np.uint8)
        blob[t_bytes + s_bytes:t_bytes + s_bytes + host_u.nbytes] = host_u.view(np.uint8)
        staging = torch.from_numpy(blob).pin_memory()
        self.table = torch.empty(blob.size, dtype=torch.uint8, device=device)
        self.table.copy_(staging, non_blocking=True)
        self._staging = staging  # kept alive with the plan, so the async copy never races
        # Gradient pointers change every step in a loop that frees its gradients
        # (zero_grad(set_to_none=True)); the chunk tables do not depend on them, so only the
        # tensor entries are patched and re-uploaded (update_grads), through a small ring of
        # pinned buffers so a pending upload is never overwritten.
        other = np.ones(n, dtype=bool)
        for f in ("param", "master", "exp_avg", "exp_avg_sq"):
            other &= (host_t[f] & np.uint64(15)) == 0
        self._others_aligned = other
        self._t_nbytes = host_t.nbytes
        self._ring = [torch.empty(host_t.nbytes, dtype=torch.uint8).pin_memory()
                      for _ in range(3)]
        self._ring_events: list = [None, None, None]
        self._ring_i = 0
        self.tensors_ptr = self.table.data_ptr()
        self.chunks_ptr = self.table.data_ptr() + t_bytes
        self.update_chunks_ptr = self.table.data_ptr() + t_bytes + s_bytes
        ws_bytes = int(lib.b2o_workspace_bytes(self.n_chunks, n_slots))
        if workspace is not None and workspace.numel() >= ws_bytes:
            self.workspace = workspace
        else:
            self.workspace = torch.empty(_round_up(ws_bytes, 256), dtype=torch.uint8,
                                         device=device)
            _lib.call("b2o_workspace_init", self.workspace.data_ptr(), self.workspace.numel(),
                      torch.cuda.current_stream(device).cuda_stream)

    def update_grads(self, grad_ptrs: np.ndarray) -> None:
        """Point the tensor entries at new gradient tensors (same sizes and dtypes, in entry
        order) and upload the entries on the current stream, after the kernels already queued."""
        t = self.host_tensors
        grad_ptrs = np.asarray(grad_ptrs, dtype=np.uint64)
        if np.any((grad_ptrs == 0) & (t["numel"] > 0)):
            raise RuntimeError("null gradient pointer for a non-empty tensor")
        t["grad"] = grad_ptrs
        ok = ((grad_ptrs & np.uint64(15)) == 0) & self._others_aligned
        t["flags"] = np.where(ok, _lib.FLAG_VECTOR, 0).astype(np.int32)
        i = self._ring_i
        self._ring_i = (i + 1) % len(self._ring)
        if self._ring_events[i] is not None:
            self._ring_events[i].synchronize()
        buf = self._ring[i]
        buf.numpy()[:] = t.view(np.uint8)
        self.table[:self._t_nbytes].copy_(buf, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._ring_events[i] = ev

    def vector_fraction(self) -> float:
        """Fraction of elements whose tensor qualifies for the 128-bit path."""
        tot = int(self.host_tensors["numel"].sum())
        if tot == 0:
            return 1.0
        vec = int(self.host_tensors["numel"][(self.host_tensors["flags"] & _lib.FLAG_VECTOR)
                                             != 0].sum())
        return vec / tot


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device | None = None) -> int:
    """The current CUDA stream of ``device`` as a raw ``cudaStream_t`` value."""
    if _raw_stream is not None and device is not None and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream

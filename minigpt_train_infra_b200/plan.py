"""Multi-tensor-apply launcher: device-side tensor and chunk tables for the step kernels.

The reference hands PyTorch lists of tensors every step (``torch/amp/grad_scaler.py:294``,
``torch/optim/adam.py:880``) and ATen re-chunks them into kernel-argument structs on every call.
Here a :class:`ChunkPlan` packs each tensor's pointers (grad, bf16 param, fp32 master, exp_avg,
exp_avg_sq), its element count, param-group and step slot, plus a chunk table, into one device
buffer (``b2o_plan_chunks`` in ``csrc/b2o_plan.cu`` does the packing and validation).  The plan is
built once per parameter set and reused while the pointers are unchanged, so a step costs only
the kernel launches.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

DEFAULT_CHUNK_ELEMS = 1 << 16  # 64 Ki elements: 1.75 MiB of optimizer traffic per chunk

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


class ChunkPlan:
    """Device tables (tensor entries + chunks) and the stats workspace for one dtype bucket."""

    def __init__(self, device: torch.device, entries: list[Entry], n_groups: int, n_slots: int,
                 grad_dtype: int, param_dtype: int, chunk_elems: int = DEFAULT_CHUNK_ELEMS,
                 workspace: torch.Tensor | None = None):
        lib = _lib.load()
        self.device = device
        self.grad_dtype = grad_dtype
        self.param_dtype = param_dtype
        self.n_groups = n_groups
        self.n_slots = n_slots
        self.chunk_elems = chunk_elems
        n = len(entries)
        host_t = np.zeros(n, dtype=_lib.TENSOR_DTYPE)
        for i, e in enumerate(entries):
            host_t[i] = (e.grad, e.param, e.master, e.exp_avg, e.exp_avg_sq, e.numel, e.group,
                         e.slot, 0, 0, 0, 0)
        n_chunks = np.zeros(1, dtype=np.int64)
        _lib.check("b2o_plan_chunks", lib.b2o_plan_chunks(
            _lib.ptr(host_t), n, n_groups, n_slots, chunk_elems, grad_dtype, None, 0,
            _lib.ptr(n_chunks)))
        host_c = np.zeros(int(n_chunks[0]), dtype=_lib.CHUNK_DTYPE)
        _lib.check("b2o_plan_chunks", lib.b2o_plan_chunks(
            _lib.ptr(host_t), n, n_groups, n_slots, chunk_elems, grad_dtype,
            _lib.ptr(host_c) if host_c.size else None, host_c.size, _lib.ptr(n_chunks)))
        self.n_tensors = n
        self.n_chunks = int(n_chunks[0])
        self.host_tensors = host_t
        self.host_chunks = host_c
        # One device buffer: [tensor table | chunk table], each 256-byte aligned.
        t_bytes = _round_up(host_t.nbytes, 256)
        c_bytes = _round_up(host_c.nbytes, 256)
        blob = np.zeros(t_bytes + c_bytes, dtype=np.uint8)
        blob[:host_t.nbytes] = host_t.view(np.uint8)
        blob[t_bytes:t_bytes + host_c.nbytes] = host_c.view(np.uint8)
        staging = torch.from_numpy(blob).pin_memory()
        self.table = torch.empty(blob.size, dtype=torch.uint8, device=device)
        self.table.copy_(staging, non_blocking=True)
        self._staging = staging  # kept alive until the copy has run
        self._staging_done = torch.cuda.Event()
        self._staging_done.record()
        self.tensors_ptr = self.table.data_ptr()
        self.chunks_ptr = self.table.data_ptr() + t_bytes
        ws_bytes = int(lib.b2o_workspace_bytes(self.n_chunks, n_slots))
        if workspace is not None and workspace.numel() >= ws_bytes:
            self.workspace = workspace
        else:
            self.workspace = torch.empty(_round_up(ws_bytes, 256), dtype=torch.uint8,
                                         device=device)
            _lib.call("b2o_workspace_init", self.workspace.data_ptr(), self.workspace.numel(),
                      torch.cuda.current_stream(device).cuda_stream)
        # Per-slot exchange vector (n_slots + 1 doubles) inside the workspace.
        exch_off = 64 + 8 * self.n_chunks
        self.exch = self.workspace[exch_off:exch_off + 8 * (n_slots + 1)].view(torch.float64)

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


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream

"""Device buffers shared between the processes of one node (legacy CUDA IPC).

Each rank allocates its flat buffer with ``b2o_peer_alloc`` (``cudaMalloc``), publishes the
64-byte IPC handle through ``torch.distributed.all_gather_object``, and maps every other rank's
buffer with ``b2o_peer_import``.  The fused collective kernels then read and write the other
ranks' buffers with plain loads and stores over NVLink; no multicast object is involved.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib


class _CudaArray:
    """Exposes a raw device allocation through ``__cuda_array_interface__`` so a torch tensor
    can alias it; frees it (or unmaps it) when the last tensor referring to it is gone."""

    def __init__(self, ptr: int, nbytes: int, release):
        self.ptr = ptr
        self.nbytes = nbytes
        self._release = release
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None,
                                         "stream": None}

    def __del__(self):
        rel, self._release = self._release, None
        if rel is not None and self.ptr:
            try:
                rel(self.ptr)
            except Exception:
                pass


class PeerBuffer:
    """One flat buffer of ``numel`` elements of ``dtype`` on every rank of ``group``.

    ``local`` is this rank's buffer as a torch tensor; ``peer_ptrs[r]`` is rank r's buffer as
    mapped in this process (``peer_ptrs[rank] == local.data_ptr()``).
    """

    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device, group=None):
        lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        nbytes = int(numel) * torch.empty((), dtype=dtype).element_size()
        with torch.cuda.device(device):
            out = ctypes.c_void_p()
            _lib.check("b2o_peer_alloc", lib.b2o_peer_alloc(nbytes, ctypes.byref(out)))
            base = int(out.value)
            self._own = _CudaArray(base, nbytes, lambda p: lib.b2o_peer_free(p))
            raw = torch.as_tensor(self._own, device=device)
            self.local = raw.view(dtype)
            handle = np.zeros(_lib.IPC_HANDLE_BYTES, dtype=np.uint8)
            _lib.check("b2o_peer_export", lib.b2o_peer_export(base, _lib.ptr(handle)))
            handles: list = [None] * self.world
            dist.all_gather_object(handles, handle.tobytes(), group=group)
            self.peer_ptrs = []
            self._imports = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.peer_ptrs.append(base)
                    continue
                hb = np.frombuffer(h, dtype=np.uint8).copy()
                mapped = ctypes.c_void_p()
                _lib.check("b2o_peer_import", lib.b2o_peer_import(_lib.ptr(hb),
                                                                  ctypes.byref(mapped)))
                self.peer_ptrs.append(int(mapped.value))
                self._imports.append(int(mapped.value))
        self._ptr_array = _lib.ptr_array(self.peer_ptrs)

    @property
    def ptr_array(self):
        if self._ptr_array is None:
            raise RuntimeError("peer buffer is closed: its peer mappings were released")
        return self._ptr_array

    def close(self) -> None:
        """Unmap the other ranks' buffers (this rank's own buffer is freed with ``local``).
        Call on every rank, with every kernel that touches peer memory finished, then
        synchronise the ranks before any of them frees its buffer."""
        lib = _lib.load()
        self._ptr_array = None  # no kernel may be handed the released mappings
        for p in self._imports:
            lib.b2o_peer_close(p)
        self._imports = []
        self.peer_ptrs = [self.local.data_ptr()]

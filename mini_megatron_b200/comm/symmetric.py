"""Symmetric device buffers: one equally sized allocation per rank, mapped into every peer.

Each rank allocates ``nbytes`` with cudaMalloc (through the extension), exports
a CUDA IPC handle, and the handles are exchanged with ``all_gather_object``
over the given process group.  ``peer_ptr(r)`` is then a device address, valid
in this process, of rank ``r``'s buffer (its GPU memory, reached over
NVLink/NVSwitch); the kernels load from and store to it directly.  All ranks
of the group must be on one node.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import native


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None, device=None):
        C = native()
        self.group = group
        self.world = 1 if group is None else dist.get_world_size(group)
        self.rank = 0 if group is None else dist.get_rank(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.nbytes = (int(nbytes) + 4095) // 4096 * 4096
        self.local = C.symm_alloc(self.nbytes)
        handles = [None] * self.world
        mine = C.symm_export(self.local)
        if self.world > 1:
            dist.all_gather_object(handles, mine, group=group)
        else:
            handles = [mine]
        self.ptrs = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.local)
            else:
                p = C.symm_open(h)
                self._opened.append(p)
                self.ptrs.append(p)
        self._closed = False

    def poison(self, offset_bytes: int = 0, nbytes: int | None = None):
        """Fill [offset, offset + nbytes) of THIS rank's buffer with 0xFF bytes (NaN as fp32 and bf16).

        Debug aid: a kernel that reads a symmetric region before its producer
        wrote it then propagates NaNs instead of silently reusing stale data.
        The caller must make sure no peer is reading the region meanwhile.
        """
        n = self.nbytes - offset_bytes if nbytes is None else nbytes
        self.tensor(offset_bytes, n, torch.uint8).fill_(0xFF)

    def peer_ptr(self, rank: int, offset_bytes: int = 0) -> int:
        return self.ptrs[rank] + offset_bytes

    def tensor(self, offset_bytes: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A view of this rank's buffer (``offset_bytes`` must respect ``dtype``'s alignment)."""
        return native().tensor_from_ptr(self.local + offset_bytes, numel, dtype, self.device.index)

    def close(self):
        if self._closed:
            return
        C = native()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            C.symm_close(p)
        C.symm_free(self.local)
        self._closed = True

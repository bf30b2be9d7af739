"""Symmetric device buffers shared over CUDA IPC, with copy-engine puts to peers.

``SymmetricBuffer(nbytes, group)`` allocates the same number of bytes on every rank of
``group``, maps every peer's buffer, and offers ``put(tensor, peer, offset)`` (one
``cudaMemcpyAsync`` over NVLink) plus ``local`` (a uint8 view of this rank's buffer).
Collective construction; ``barrier()`` orders puts between ranks on the host.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import load


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._b = load().SymmBuffer(self.world, self.rank, int(nbytes), dev.index or 0)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self._b.ipc_handle(), group=group)
            self._b.open_peers(handles)
            dist.barrier(group=group)
        self.local = self._b.local()

    def put(self, tensor: torch.Tensor, peer: int, byte_offset: int = 0):
        self._b.put(tensor.contiguous(), peer, int(byte_offset))

    def view(self, dtype, shape, byte_offset: int = 0) -> torch.Tensor:
        n = int(torch.tensor([], dtype=dtype).element_size())
        count = 1
        for s in shape:
            count *= s
        return self.local[byte_offset:byte_offset + n * count].view(dtype).view(*shape)

    def barrier(self):
        """Make every rank's outstanding puts visible to every other rank (host ordered)."""
        torch.cuda.current_stream().synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)

    def close(self):
        self._b.close()

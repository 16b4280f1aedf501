"""Peer-addressable device buffers for the fused collective kernels (one process per GPU).

``PeerBuffers`` allocates one zeroed device region per rank with a plain
``cudaMalloc``, exports it through CUDA IPC, exchanges the handles over the
process group and maps every peer's region.  Kernels then read and write peer
memory with ordinary loads and stores over NVLink / NVSwitch.  No multicast
object is created and no library kernel is ever handed a peer address.

A region is carved into named, 256-byte aligned sub-buffers::

    bufs = PeerBuffers({"grad": (n, torch.bfloat16), "out": (n, torch.float32)}, group)
    bufs.local("grad")        # this rank's tensor view
    bufs.addresses("grad")    # [address on rank 0, ..., address on rank W-1]
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext

_ALIGN = 256


class PeerBuffers:
    def __init__(self, layout: dict[str, tuple[int, torch.dtype]], group=None, device=None):
        ext = _ext.require()
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        offsets, cursor = {}, 0
        for name, (numel, dtype) in layout.items():
            offsets[name] = cursor
            nbytes = int(numel) * torch.empty((), dtype=dtype).element_size()
            cursor += (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        self.layout = dict(layout)
        self.offsets = offsets
        self.nbytes = max(cursor, _ALIGN)
        self.region, handle = ext.ipc_alloc(self.nbytes, self.device.index)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        for peer, h in enumerate(handles):
            if peer == self.rank:
                self.bases.append(self.region.data_ptr())
            else:
                address = ext.ipc_open(h, self.device.index)
                self._opened.append(address)
                self.bases.append(address)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def local(self, name: str) -> torch.Tensor:
        numel, dtype = self.layout[name]
        start = self.offsets[name]
        size = int(numel) * torch.empty((), dtype=dtype).element_size()
        return self.region[start: start + size].view(dtype)

    def addresses(self, name: str) -> list[int]:
        return [base + self.offsets[name] for base in self.bases]

    def close(self) -> None:
        """Unmap the peers' regions (call on every rank before the process group goes away)."""
        ext = _ext.require()
        torch.cuda.synchronize(self.device)
        for address in self._opened:
            ext.ipc_close(address, self.device.index)
        self._opened = []

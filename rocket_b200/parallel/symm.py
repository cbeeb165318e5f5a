"""Symmetric heap: one device buffer per rank, mapped into every other rank.

Each rank cudaMallocs the same number of bytes, exports a CUDA IPC handle,
all-gathers the handles over the process group and opens every peer's buffer,
so a kernel can address any rank's copy as ``base[r] + offset``.  The first
4 KiB hold the epoch flag block (comm.cuh); ``alloc`` hands out aligned
offsets that are identical on every rank because every rank allocates the same
sequence.  The mapping is registered with the extension under a slot id that
kernels look up at launch.

Reference counterpart: the registered RDMA regions of the 2-node fabric
(engines/glm5-moe-nvfp4-2b/src/fabric/fabric.h:66, register_region) -- on one
NVSwitch node, peer memory replaces RDMA.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

FLAG_BYTES = 4096
N_SITES = 16


class SymmetricHeap:
    def __init__(self, par, nbytes: int, slot: int = 0):
        from .. import _C
        self.C = _C
        self.par = par
        self.slot = slot
        dev = par.device
        self.dev_index = dev.index if dev.index is not None else torch.cuda.current_device()
        self.size = FLAG_BYTES + ((nbytes + 4095) // 4096) * 4096
        self.local = _C.symm_alloc(self.size, self.dev_index)
        h = _C.ipc_handle(self.local)
        if par.world > 1:
            hs = [torch.zeros(64, dtype=torch.uint8, device=dev) for _ in range(par.world)]
            dist.all_gather(hs, h.to(dev), group=par.group)
            hs = [x.cpu() for x in hs]
        else:
            hs = [h]
        self.bases = []
        self.opened = []
        for r in range(par.world):
            if r == par.rank:
                self.bases.append(self.local.data_ptr())
            else:
                p = _C.ipc_open(hs[r], self.dev_index)
                self.bases.append(p)
                self.opened.append(p)
        # producer epochs, consumer epochs, last-CTA arrival counters
        self.counters = torch.zeros(3 * N_SITES, dtype=torch.int32, device=dev)
        _C.peer_register(slot, self.bases, par.rank, par.world, 0, self.counters)
        self.next = FLAG_BYTES
        par.barrier()

    def alloc(self, nbytes: int, align: int = 1024) -> int:
        off = (self.next + align - 1) // align * align
        if off + nbytes > self.size:
            raise MemoryError(f"symmetric heap exhausted ({off + nbytes} > {self.size})")
        self.next = off + nbytes
        return off

    def view(self, off: int, shape, dtype) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        return self.local[off:off + nbytes].view(dtype).view(*shape)

    def close(self):
        for p in self.opened:
            self.C.ipc_close(p)
        self.opened = []

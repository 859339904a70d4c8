"""Symmetric peer memory and the fused tensor-parallel all-reduce.

Each rank of a TP group allocates one device buffer, exports it with a CUDA
IPC handle and opens every peer's buffer, so a kernel on this GPU can store
straight into the other GPUs' memory over NVLink / NVSwitch.  The buffer
holds the per-source arrival flags and two parities of per-source fp32
receive slots.  The native producers (row-parallel GEMV epilogue, expert
combine) push their partial sums into every peer's slot and publish an
epoch; the native consumer (the next RMSNorm) waits on the flags with a
bounded spin, sums the slots in rank order plus the residual, and normalises
-- one all-reduce per sublayer with no extra kernel launch.

The descriptor handed to the kernels is a CPU int64 tensor (layout in
``csrc/kernels/symm.cuh``); it is fixed for the life of the buffer, which is
what CUDA-graph replay needs.
"""
from __future__ import annotations

import torch

MAX_TP = 8
FLAG_BYTES = 256
DESC_LEN = 8 + 2 * MAX_TP


class SymmAllReduce:
    def __init__(self, group, max_elems: int, device, status: torch.Tensor, spin_limit: int = 1 << 22):
        import torch.distributed as dist
        from ..ops import native
        self.C = native()
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if self.world > MAX_TP:
            raise ValueError(f"fused all-reduce supports up to {MAX_TP} ranks")
        self.device = torch.device(device)
        self.cap = int(max_elems)
        nbytes = FLAG_BYTES + 2 * self.world * self.cap * 4
        self.ptr, handle = self.C.symm_alloc(nbytes)
        self.nbytes = nbytes
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
            self.peers = [self.ptr if r == self.rank else self.C.symm_open(handles[r]) for r in range(self.world)]
            dist.barrier(group=group)
        else:
            self.peers = [self.ptr]
        # local protocol state: ncall (u64), arrive (u32), done (u32)
        self.state = torch.zeros(2, dtype=torch.int64, device=self.device)
        sp = self.state.data_ptr()
        d = torch.zeros(DESC_LEN, dtype=torch.int64)
        d[0], d[1], d[2], d[3] = self.world, self.rank, self.cap, spin_limit
        d[4], d[5], d[6], d[7] = sp, sp + 8, sp + 12, status.data_ptr()
        for r, p in enumerate(self.peers):
            d[8 + r] = p + FLAG_BYTES
            d[8 + MAX_TP + r] = p
        self.desc = d
        self._status = status

    def fits(self, rows: int, cols: int) -> bool:
        return rows * cols <= self.cap

    def close(self):
        if getattr(self, "ptr", None) is None:
            return
        torch.cuda.synchronize(self.device)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                self.C.symm_close(p)
        self.C.symm_free(self.ptr)
        self.ptr = None

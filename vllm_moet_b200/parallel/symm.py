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


class EpSymm:
    """Symmetric peer buffer of the expert-parallel all-to-all (decode-sized MoE layers under
    data-parallel attention; kernels and layout in ``csrc/kernels/ep_a2a.cuh``).

    Each rank of the EP group allocates one buffer -- dispatch slabs for every source
    (e4m3 rows, scales, expert ids), the return rows of its own routings, arrival flags --
    exports it by CUDA IPC and opens every peer's.  ``cap`` is the most routed rows
    (tokens x top-k) one rank sends in one layer.  ``group`` None gives a one-rank
    loopback (every expert local), which exercises the same kernels on one GPU.
    """

    def __init__(self, group, cap: int, hidden: int, experts_local: int, top_k: int, device, status: torch.Tensor,
                 spin_limit: int = 1 << 22):
        import torch.distributed as dist
        from ..ops import native
        self.C = native()
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if self.world > MAX_TP:
            raise ValueError(f"EP all-to-all supports up to {MAX_TP} ranks")
        if hidden % 64:
            raise ValueError("EP all-to-all: hidden % 64")
        self.cap, self.H, self.E_loc, self.k = int(cap), int(hidden), int(experts_local), int(top_k)
        self.device = torch.device(device)
        nbytes = int(self.C.ep_buffer_bytes(self.world, self.cap, self.H))
        self.ptr, handle = self.C.symm_alloc(nbytes)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
            self.peers = [self.ptr if r == self.rank else self.C.symm_open(handles[r]) for r in range(self.world)]
            dist.barrier(group=group)
        else:
            self.peers = [self.ptr]
        self.state = torch.zeros(2, dtype=torch.int64, device=self.device)     # ncall, arrive | done
        sp = self.state.data_ptr()
        d = torch.zeros(11 + MAX_TP, dtype=torch.int64)
        d[0], d[1], d[2], d[3], d[4], d[5], d[6] = self.world, self.rank, self.cap, self.H, self.E_loc, self.k, spin_limit
        d[7], d[8], d[9], d[10] = sp, sp + 8, sp + 12, status.data_ptr()
        for r, p in enumerate(self.peers):
            d[11 + r] = p
        self.desc = d
        al = lambda x: (x + 255) // 256 * 256   # noqa: E731
        W, cap, H = self.world, self.cap, self.H
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        off_rs = 256 + al(W * cap * H)
        off_meta = off_rs + al(W * cap * (H // 64))
        off_ret = off_meta + al(W * cap * 4)
        self.rx = self.C.symm_view(self.ptr + 256, W * cap * H, dev).view(W * cap, H)
        self.rs = self.C.symm_view(self.ptr + off_rs, W * cap * (H // 64), dev).view(W * cap, H // 64)
        self.ret = self.C.symm_view(self.ptr + off_ret, cap * H * 4, dev).view(torch.float32).view(cap, H)
        self.nbytes = nbytes

    def close(self):
        if getattr(self, "ptr", None) is None:
            return
        torch.cuda.synchronize(self.device)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                self.C.symm_close(p)
        self.C.symm_free(self.ptr)
        self.ptr = None

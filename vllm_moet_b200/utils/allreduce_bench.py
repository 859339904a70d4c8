"""Latency of one decode-sized tensor-parallel reduction: the fused peer-memory protocol
(push kernel + reduce kernel, ``csrc/kernels/symm.cuh``) against NCCL all-reduce, eager and
inside a CUDA graph.  One process per GPU:

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m vllm_moet_b200.utils.allreduce_bench

Prints microseconds per reduction of a [3, 4096] activation (the 1-stream MTP verify rows of
the DS4 shape), max over ranks, CUDA-event timed.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    from ..ops import native
    from ..parallel.symm import SymmAllReduce
    C = native()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ar = SymmAllReduce(dist.group.WORLD, 128 * 4096, "cuda", status)
    x = torch.randn(3, 4096, device="cuda")
    resid = torch.randn(3, 4096, device="cuda")
    out = torch.empty_like(x)
    xb = torch.randn(3, 4096, device="cuda", dtype=torch.bfloat16)

    def timeit(fn, n=2000):
        for _ in range(50):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / n * 1000], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    fused = lambda: C.ar_test(ar.desc, x, resid, out, 0)        # noqa: E731
    nccl = lambda: dist.all_reduce(xb)                          # noqa: E731
    res = {"fused push+reduce (2 kernels)": timeit(fused), "nccl all_reduce bf16 [3,4096]": timeit(nccl),
           "nccl all_reduce f32 [3,4096]": timeit(lambda: dist.all_reduce(x))}
    for name, fn in (("fused", fused), ("nccl", nccl)):
        g = torch.cuda.CUDAGraph()
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for _ in range(100):
                fn()
        res[f"{name}, 100 per CUDA graph"] = timeit(g.replay, 50) / 100
    if int(status) != 0:
        raise RuntimeError(f"fused all-reduce status {int(status)}")
    if rank == 0:
        for k, v in res.items():
            print(f"{k}: {v:.2f} us")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

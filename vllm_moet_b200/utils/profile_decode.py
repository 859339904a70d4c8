"""Profiling driver: one captured DS4-Flash-shaped decode step, replayed inside
``torch.cuda.profiler.start/stop`` so an external profiler can capture exactly
the decode kernels (``ncu --profile-from-start off``).

    python -m vllm_moet_b200.utils.profile_decode --layers 2 --batch 1 --reps 1

Prints the device-timed ms per step (CUDA events, outside the profiler range).
"""
from __future__ import annotations

import argparse

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--reps", type=int, default=1)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--tp", type=int, default=1,
                    help="run rank 0's shards of a TP-N model on this GPU without a group (kernel shapes and "
                         "costs of TP-N; partial sums are not reduced, no collectives)")
    ap.add_argument("--mode", choices=["decode", "prefill"], default="decode",
                    help="profile the captured decode step, or one prefill of --prompt-len tokens")
    a = ap.parse_args(argv)
    from ..engine.llm import LLM
    B = a.batch
    llm = LLM("ds4-flash-shape", device="cuda", num_speculative_tokens=2, max_model_len=a.prompt_len + 256,
              max_num_seqs=B, num_layers=a.layers, tensor_parallel_size=a.tp, tp_rank=0)
    r = llm.runner
    st = llm._state(B)
    g = torch.Generator().manual_seed(0)
    bt = torch.zeros(B, llm.max_blocks, dtype=torch.int32)
    prompts = []
    for i in range(B):
        blocks = llm.blocks.allocate(f"s{i}", a.prompt_len + 200)
        bt[i, :len(blocks)] = torch.tensor(blocks)
        prompts.append(torch.randint(3, llm.cfg.vocab, (a.prompt_len,), generator=g).tolist())
    st.block_table.copy_(bt)
    r.prefill(prompts, [bt[i].tolist() for i in range(B)], list(range(B)), st)
    if a.mode == "prefill":
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        r.prefill(prompts, [bt[i].tolist() for i in range(B)], list(range(B)), st)
        e.record()
        torch.cuda.synchronize()
        print("ms/prefill", s.elapsed_time(e))
        torch.cuda.profiler.start()
        r.prefill(prompts, [bt[i].tolist() for i in range(B)], list(range(B)), st)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        return
    st.set_active(torch.ones(B, dtype=torch.int32, device="cuda"))
    gr = r.capture(st)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(10):
        gr.replay()
    e.record()
    torch.cuda.synchronize()
    print("ms/step", s.elapsed_time(e) / 10)
    torch.cuda.profiler.start()
    for _ in range(a.reps):
        gr.replay()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()

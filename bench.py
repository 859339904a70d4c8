"""Headline benchmark: DeepSeek-V4-Flash-shaped MoE,
random-init weights, synthetic prompts.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

Metric: decode tok/s at 1 stream (MTP k=2, greedy) -- the
JSON `value` -- with 32-stream aggregate decode and 8192-token prefill
tok/s reported alongside.  `value` is device-timed: K decode steps replayed
back to back from the captured graph (each step is a full MTP verify +
draft step that advances the sequence on the device), between a barrier +
synchronize on both sides, max over ranks.  `e2e` is the same metric
through the public `LLM.generate` API, timed on the host from the first emitted
token to completion: per step it copies the row-activity vector H2D from pinned
memory, replays the graph, reads the emitted tokens D2H and runs the host loop.  Each decode
step streams ~7 GB of weights (>> 126 MB L2), so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

BASELINE = {1: 161.0, 2: 210.0, 4: 214.0, 8: 214.0}   # published decode tok/s at 1 / 2 / 4 GPUs (8 GPUs: the 4-GPU bar)
METRIC = "decode tok/s @1/32 streams + 8k prefill tok/s, DS4-Flash shape, 1/2/4/8 B200"


def _reference_arm(args):
    print(json.dumps({"impl": "reference", "unavailable":
                      "the reference is a patch over vLLM v0.24.0 plus SM120-only SASS cubins; it has no "
                      "setup.py/pyproject (pip refused: not installable) and its kernels refuse any GPU but sm_120",
                      "metric": METRIC, "n_gpus": args.gpus}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer layers (invalid for reporting)")
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--prefill-len", type=int, default=8192)
    ap.add_argument("--streams", type=int, default=32)
    ap.add_argument("--skip-extra", action="store_true", help="skip the 32-stream and prefill measurements")
    ap.add_argument("--ep", action="store_true",
                    help="data-parallel attention + expert-parallel MoE (BASELINE config 3): every rank serves its "
                         "own streams, routed experts are partitioned over the ranks and exchanged all-to-all")
    ap.add_argument("--ep-streams", default="1,4,8,16,32", help="--ep: total concurrent streams to measure")
    ap.add_argument("--sp", type=int, default=0,
                    help="sequence-parallel prefill of one prompt of this many tokens over the N ranks "
                         "(replicated weights); reports prefill tok/s, device-timed, max over ranks")
    ap.add_argument("--sp-chunk", type=int, default=0,
                    help="--sp on one GPU: prefill the prompt in chunks of this many tokens (block-aligned)")
    ap.add_argument("--expert-cache-gb", type=float, default=0.0,
                    help="residency: serve routed experts from a GPU cache of this many GiB over a host store "
                         "(reports 1-stream decode through LLM.generate, host fetches included)")
    ap.add_argument("--expert-store", default="pinned", choices=["pinned", "pack", "tiered"])
    ap.add_argument("--delta-slots", type=int, default=0, help="residency: FP4 delta-tier slots")
    ap.add_argument("--gate", action="store_true", help="residency: confidence gate on the delta tier")
    args = ap.parse_args()
    if args.impl == "reference":
        return _reference_arm(args)
    if args.warmup < 3:
        print("warning: --warmup < 3 is below the timing rules; using 3", file=sys.stderr)
        args.warmup = 3

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    from vllm_moet_b200 import LLM, SamplingParams
    from vllm_moet_b200.utils.benchmark import ClockSampler, LaunchCounter

    t0 = time.time()
    max_len = max(args.prompt_len + args.steps * 3 + args.warmup * 3 + 64, args.prefill_len + 64)
    if args.ep:
        if world == 1:
            dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", local),
                                    store=dist.HashStore())
        per_rank = -(-max(int(x) for x in args.ep_streams.split(",")) // world)
        llm = LLM("ds4-flash-shape", device="cuda", num_speculative_tokens=2, max_model_len=max_len,
                  max_num_seqs=max(per_rank, 1), num_layers=args.layers, seed=0, ep_group=dist.group.WORLD)
    elif args.expert_cache_gb > 0 or args.delta_slots > 0:
        return _residency(args, world, rank, local)
    elif args.sp:
        return _sp_prefill(args, world, rank, local, dist)
    else:
        llm = LLM("ds4-flash-shape", device="cuda", num_speculative_tokens=2, max_model_len=max_len,
                  max_num_seqs=args.streams, num_layers=args.layers, seed=0, tensor_parallel_size=world,
                  tp_group=dist.group.WORLD if world > 1 else None, tp_rank=rank)

    def maxr(v):   # max over ranks of a time-like value
        if world == 1:
            return v
        t = torch.tensor([float(v)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    def minr(v):   # min over ranks of a rate
        return -maxr(-v) if world > 1 else v
    torch.cuda.synchronize()
    load_s = time.time() - t0
    runner = llm.runner
    g = torch.Generator().manual_seed(1234)
    vocab = llm.cfg.vocab

    def prompt(n):
        return torch.randint(3, vocab, (n,), generator=g).tolist()

    # ---- 1-stream decode: device-timed graph replays ----------------------------------------
    from vllm_moet_b200.engine.gpu_runner import DecodeState
    st = llm._state(1)
    blocks = llm.blocks.allocate("bench", args.prompt_len + (args.steps + args.warmup + 4) * 3 + 8)
    bt = torch.zeros(1, llm.max_blocks, dtype=torch.int32)
    bt[0, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
    st.block_table.copy_(bt)
    runner.prefill([prompt(args.prompt_len)], [bt[0].tolist()], [0], st)
    st.set_active(torch.ones(1, dtype=torch.int32, device="cuda"))
    # count the native launches of one step on the eager warm-up pass (the same code path the
    # graph records), then capture with the plain module
    counter = LaunchCounter(runner.C)
    real_C = runner.C
    runner.C = counter
    try:
        runner.decode_body_eager_warm(st)
    finally:
        runner.C = real_C
    launches_per_step = counter.count
    graph = runner.capture(st, warm=False)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    pos0 = int(st.seq_pos[0])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        s_ev.record()
        for _ in range(args.steps):       # nothing but graph replays between the events
            graph.replay()
        e_ev.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = s_ev.elapsed_time(e_ev) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    # every step advances the sequence by 1 + accepted drafts
    acc = (int(st.seq_pos[0]) - pos0) / args.steps - 1.0
    tok_per_step = 1.0 + acc
    # --ep: every rank decodes its own stream (data-parallel attention), so the job's aggregate
    # is world streams' worth of tokens per step
    value = tok_per_step * 1000.0 / ms * (world if args.ep else 1)
    llm.blocks.release("bench")

    # ---- e2e through LLM.generate (1 stream) -----------------------------------------------
    # host wall clock from the first emitted token to the request's completion: every decode
    # step's H2D copy of the row-activity vector from pinned memory, graph replay, D2H read of
    # the emitted tokens and all host work between steps (emit, stop checks, detokenise)
    n_tok = args.steps + 1
    llm.generate([prompt(args.prompt_len)], SamplingParams(max_tokens=4, ignore_eos=True))  # warm
    outs = llm.generate([prompt(args.prompt_len)], SamplingParams(max_tokens=n_tok, ignore_eos=True))
    m = outs[0].metrics
    e2e_tok_s = (len(outs[0].outputs[0].token_ids) - 1) / maxr(m["e2e_s"] - m["ttft_s"])

    extra, errors = {}, {}
    if world > 1 and not args.ep:
        # correctness gate across the TP ranks: every rank emits the whole sequence, and the
        # same greedy tokens on every rank are the condition for the timed steps to mean
        # anything (diverging ranks would write their KV shards for different sequences)
        ids = torch.full((n_tok,), -1, dtype=torch.int64, device="cuda")
        mine = torch.tensor(outs[0].outputs[0].token_ids[:n_tok], dtype=torch.int64)
        ids[:mine.numel()] = mine.to("cuda")
        every = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(every, ids)
        extra["tp_ranks_same_tokens"] = all(torch.equal(every[0], x) for x in every[1:])

    def secondary(name, fn):
        """A secondary measurement that fails (the same way on every rank) is reported as an
        error field; the headline number above stands."""
        try:
            fn()
        except Exception as e:  # noqa: BLE001
            errors[name] = f"{type(e).__name__}: {str(e)[:200]}"
            torch.cuda.synchronize()

    def streams():
        # ---- 32-stream aggregate decode (public API, device replays inside) ------------------
        S = args.streams
        llm.generate([prompt(args.prompt_len) for _ in range(S)], SamplingParams(max_tokens=4, ignore_eos=True))
        outs = llm.generate([prompt(args.prompt_len) for _ in range(S)],
                            SamplingParams(max_tokens=args.steps + 1, ignore_eos=True))
        stt = dict(llm.stats)
        gen = sum(len(o.outputs[0].token_ids) - 1 for o in outs)
        # wall clock from the first emitted token to the last request's completion
        first = min(o.metrics["ttft_s"] for o in outs)
        last = max(o.metrics["e2e_s"] for o in outs)
        dec_s = maxr(last - first)
        extra[f"decode_{S}_streams_tok_s"] = gen / dec_s
        extra[f"decode_{S}_streams_steps_s"] = stt["steps"] / dec_s

    def ep_streams():
        # ---- DP + EP serving: S total streams spread over the ranks, aggregate decode --------
        res = {}
        for S in [int(x) for x in args.ep_streams.split(",")]:
            n_loc = S // world + (1 if rank < S % world else 0)
            ps = [prompt(args.prompt_len) for _ in range(n_loc)]
            llm.generate([prompt(args.prompt_len) for _ in range(n_loc)], SamplingParams(max_tokens=4, ignore_eos=True))
            outs = llm.generate(ps, SamplingParams(max_tokens=args.steps + 1, ignore_eos=True))
            gen = sum(len(o.outputs[0].token_ids) - 1 for o in outs)
            t = torch.tensor([float(gen)], device="cuda")
            if world > 1:
                dist.all_reduce(t)
            dec = (max(o.metrics["e2e_s"] for o in outs) - min(o.metrics["ttft_s"] for o in outs)) if outs else 0.0
            res[str(S)] = round(float(t) / maxr(dec), 2)
        extra["ep_decode_tok_s_by_streams"] = res

    def prefill():
        # ---- 8k prefill ----------------------------------------------------------------------
        p8 = prompt(args.prefill_len)
        st1 = llm._state(1)
        blocks = llm.blocks.allocate("pf", args.prefill_len + 16)
        try:
            bt = torch.zeros(1, llm.max_blocks, dtype=torch.int32)
            bt[0, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
            runner.prefill([p8], [bt[0].tolist()], [0], st1)   # warm-up
            torch.cuda.synchronize()
            times = []
            for _ in range(3):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                runner.prefill([p8], [bt[0].tolist()], [0], st1)
                e.record()
                torch.cuda.synchronize()
                times.append(s.elapsed_time(e))
        finally:
            llm.blocks.release("pf")
        pf_ms = maxr(min(times))
        extra["prefill_8k_tok_s"] = args.prefill_len * 1000.0 / pf_ms * (world if args.ep else 1)
        extra["prefill_8k_ms"] = pf_ms

    if not args.skip_extra:
        if args.ep:
            ep_streams()     # collective on every rank: not wrapped (a failure must stop all ranks alike)
        else:
            secondary(f"decode_{args.streams}_streams", streams)
        secondary("prefill_8k", prefill)

    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong" if world > 1 and not args.ep else "weak",
            "vs_baseline": round(value / BASELINE.get(args.gpus, 214.0), 3),
            "dtype": "bf16 activations; fp8 e4m3 dense + 2-bit codebook experts (the reference's formats)",
            "data": "synthetic prompts, random-init weights (N(0,0.02)) of the DS4-Flash shape",
            "config": {"model": "ds4-flash-shape (32 layers, hidden 4096, 256 experts top-8, MLA, MTP k=2)",
                       "global_batch": world if args.ep else 1, "seq_len": args.prompt_len,
                       "parallelism": (f"dp{world} attention + ep{world} experts (peer-memory all-to-all)" if args.ep
                                       else (f"tp{world} (" + ("fused peer-memory" if llm.runner.ar is not None
                                                               else "NCCL") + " all-reduce; attention "
                                             + ("replicated" if not llm.mw.layers[0].attn_tp else "head-sharded")
                                             + ", experts / FFN / vocab sharded)") if world > 1 else "single"),
                       "l2": "inputs larger than L2 (each step streams ~7 GB of weights)",
                       "layers": args.layers or 32},
            "mtp_acceptance_per_step": round(acc, 4), "steps_per_s": round(1000.0 / ms, 2),
            "clocks": clk.summary(),
            "e2e": {"value": round(e2e_tok_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 * (llm.k + 1) + 4},
            "gpu_launches": launches_per_step * args.steps,
            "load_s": round(load_s, 1),
            **{k: (round(v, 2) if isinstance(v, float) else v) for k, v in extra.items()},
        }
        if errors:
            out["errors"] = errors
        print(json.dumps(out), flush=True)
    if world > 1:
        # NCCL teardown with communicators still referenced by captured CUDA graphs
        # can block at interpreter exit; leave the process directly once every
        # rank is done (nothing is in flight after the final synchronize).
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)
    return 0


def _sp_prefill(args, world, rank, local, dist):
    """Sequence-parallel prefill on the DS4 shape: one prompt of --sp tokens split into
    block-aligned chunks over the ranks (each holds the whole model), per-layer all-gathers
    of the cache blocks before attention.  Device-timed (CUDA events, barrier + synchronize
    on both sides), max over ranks; one GPU runs the plain prefill of the same prompt."""
    import torch
    from vllm_moet_b200 import LLM
    n = args.sp
    llm = LLM("ds4-flash-shape", device="cuda", num_speculative_tokens=2, max_model_len=n + 256, max_num_seqs=1,
              num_layers=args.layers, seed=0, sp_group=dist.group.WORLD if world > 1 else None)
    g = torch.Generator().manual_seed(99)
    prompt = torch.randint(3, llm.cfg.vocab, (n,), generator=g).tolist()
    st = llm._state(1)
    blocks = llm.blocks.allocate("sp", n + 64)
    bt = [0] * llm.max_blocks
    bt[:len(blocks)] = blocks
    st.block_table[0, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
    C = args.sp_chunk

    def chunked():      # one GPU, chunks of C tokens: every chunk after the first reads cached positions
        for lo in range(0, n - C, C):
            llm.runner.prefill_chunk(prompt, bt, lo, min(n, lo + C))
        return llm.runner.prefill([prompt], [bt], [0], st, starts=[(n - 1) // C * C])
    if world > 1:
        run = lambda: llm.runner.prefill_sp(prompt, bt, 0, st)     # noqa: E731
    elif C:
        run = chunked
    else:
        run = lambda: llm.runner.prefill([prompt], [bt], [0], st)   # noqa: E731
    for _ in range(max(1, args.warmup - 2)):
        run()
    times = []
    for _ in range(3):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        first = run()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e)], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(float(t))
    ms = min(times)
    if rank == 0:
        print(json.dumps({"metric": "prefill tok/s, one prompt, DS4-Flash shape [SP prefill]",
                          "value": round(n * 1000.0 / ms, 1), "unit": "tok/s", "n_gpus": world, "prompt_tokens": n,
                          "ms": round(ms, 2), "higher_is_better": True, "scaling": "strong",
                          "parallelism": f"sp{world} (replicated weights, per-layer cache all-gather)" if world > 1
                          else (f"single, {C}-token chunks" if C else "single"), "first_token": int(first) if not hasattr(first, "tolist") else
                          int(first.tolist()[0]), "dtype": "bf16 activations; fp8 dense; 2-bit experts",
                          "data": "synthetic prompt, random-init weights"}), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        os._exit(0)
    return 0


def _residency(args, world, rank, local):
    """Residency tiers on the DS4 shape: routed experts served from a GPU expert cache
    (misses fetched from the pinned / pack / tiered host store and the step replayed) and/or
    the FP4 delta tier (with the confidence gate).  Decode runs through LLM.generate with
    one stream; the rate is host wall clock from the first token to completion (fetches,
    replays and promotions included), the device graph replays in between."""
    import tempfile

    import torch
    from vllm_moet_b200 import LLM, SamplingParams
    from vllm_moet_b200.models.weights import ExpertLayout
    from vllm_moet_b200.config import get_preset
    if world > 1:
        raise SystemExit("residency bench: one GPU")
    cfg = get_preset("ds4-flash-shape")
    slot_b = ExpertLayout(H=cfg.hidden, I=cfg.moe_intermediate).slot_bytes
    slots = int(args.expert_cache_gb * (1 << 30) // slot_b)
    store_dir = tempfile.mkdtemp(prefix="moet-pack-") if args.expert_store != "pinned" else None
    t0 = time.time()
    llm = LLM("ds4-flash-shape", device="cuda", num_speculative_tokens=2, max_model_len=args.prompt_len + 4096,
              max_num_seqs=1, num_layers=args.layers, seed=0, expert_cache_slots=slots,
              expert_store=args.expert_store, expert_store_dir=store_dir, delta_slots=args.delta_slots,
              gate=args.gate if args.delta_slots else None)
    load_s = time.time() - t0
    g = torch.Generator().manual_seed(1234)
    prompt = lambda n: torch.randint(3, llm.cfg.vocab, (n,), generator=g).tolist()   # noqa: E731
    for _ in range(args.warmup):
        llm.generate([prompt(args.prompt_len)], SamplingParams(max_tokens=8, ignore_eos=True))
    outs = llm.generate([prompt(args.prompt_len)], SamplingParams(max_tokens=args.steps + 1, ignore_eos=True))
    m = outs[0].metrics
    n = len(outs[0].outputs[0].token_ids) - 1
    rate = n / (m["e2e_s"] - m["ttft_s"])
    n_moe = sum(1 for lw in llm.mw.layers if lw.is_moe) + (1 if llm.mw.mtp is not None else 0)
    out = {"metric": METRIC + " [residency tiers]", "value": round(rate, 2), "unit": "tok/s", "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16 activations; fp8 dense; 2-bit experts (+ FP4 delta tier)",
           "data": "synthetic prompts, random-init weights of the DS4-Flash shape",
           "config": {"model": "ds4-flash-shape (32 layers, 256 experts top-8, MTP k=2)", "global_batch": 1,
                      "seq_len": args.prompt_len, "parallelism": "single",
                      "expert_cache_gb": args.expert_cache_gb, "expert_cache_slots": slots,
                      "expert_slots_total": n_moe * cfg.num_experts, "expert_store": args.expert_store,
                      "delta_slots": args.delta_slots, "gate": bool(args.gate)},
           "stats": {k: v for k, v in llm.stats.items() if isinstance(v, (int, float))},
           "cache": dict(llm.cache.stats) if getattr(llm, "cache", None) is not None else None,
           "load_s": round(load_s, 1)}
    print(json.dumps(out, default=str), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

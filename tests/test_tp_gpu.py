"""Tensor parallelism on B200s: the fused peer-memory all-reduce protocol
(loopback on one GPU, including its bounded wait), and a TP=2 engine (one
process per GPU, NCCL + peer memory) checked against the fp32 oracle run
over the same shards, with identical tokens on both ranks."""
import os

import pytest
import torch

from mp_util import run_ranks

pytestmark = pytest.mark.gpu


def _C():
    from vllm_moet_b200.ops import native
    return native()


def test_symm_allreduce_loopback_and_timeout():
    from vllm_moet_b200.parallel.symm import SymmAllReduce
    C = _C()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ar = SymmAllReduce(None, 64 * 1024, "cuda", status, spin_limit=20000)
    x = torch.randn(8, 1024, device="cuda")
    resid = torch.randn(8, 1024, device="cuda")
    out = torch.empty_like(x)
    for _ in range(3):       # alternating parities
        C.ar_test(ar.desc, x, resid, out, 0)
        torch.cuda.synchronize()
        assert torch.equal(out, resid + x)
        assert int(status) == 0
    # a consumer whose producer never ran gives up with kTimeout (2) instead of hanging
    C.ar_test(ar.desc, x, resid, out, 2)
    torch.cuda.synchronize()
    assert int(status) == 2
    ar.close()


@pytest.mark.parametrize("T,H,N", [(3, 4096, 1600), (8, 1024, 512), (1, 2048, 4096)])
def test_gemv_stream_allreduce_push_consume_loopback(T, H, N):
    """World-1 loopback of the fused TP reduction in the streaming GEMV: a row-parallel
    GEMV pushes its fp32 partial, the next GEMV's norm prologue consumes it.  The new
    residual stream and the consumer's output equal the unfused sequence (fp32 partial,
    bf16 residual add, fused-norm GEMV) bit for bit."""
    from vllm_moet_b200.formats import fp8
    from vllm_moet_b200.models.weights import Fp8Linear
    from vllm_moet_b200.parallel.symm import SymmAllReduce
    C = _C()
    g = torch.Generator().manual_seed(T * H + N)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ar = SymmAllReduce(None, 128 * H, "cuda", status, spin_limit=1 << 20)
    Ko = 1024                                   # producer (o_proj-like) K
    lo = Fp8Linear.from_float(torch.randn(H, Ko, generator=g) * 0.05)
    lq = Fp8Linear.from_float(torch.randn(N, H, generator=g) * 0.05)
    aq, sa = fp8.quant_act_fp8(torch.randn(T, Ko, generator=g))
    aq, sa = aq.view(torch.uint8).cuda(), sa.cuda()
    resid = (torch.randn(T, H, generator=g)).to(torch.bfloat16).cuda()
    gamma = (torch.rand(H, generator=g) + 0.5).to(torch.bfloat16).cuda()
    # unfused reference
    part = torch.empty(T, H, device="cuda")
    C.gemv_stream_fp8(aq, sa, lo.w.cuda(), lo.s.cuda(), part, None, status)
    xnew = (resid.float() + part).to(torch.bfloat16)
    want = torch.empty(T, N, device="cuda")
    C.gemv_stream_fp8(None, None, lq.w.cuda(), lq.s.cuda(), want, None, status, xnew, gamma, 1e-6)
    for _ in range(3):      # alternating parities
        xout = torch.zeros(T, H, dtype=torch.bfloat16, device="cuda")
        got = torch.empty(T, N, device="cuda")
        dummy = torch.empty(T, H, device="cuda")
        C.gemv_stream_fp8(aq, sa, lo.w.cuda(), lo.s.cuda(), dummy, None, status, ar_push=ar.desc)
        C.gemv_stream_fp8(None, None, lq.w.cuda(), lq.s.cuda(), got, None, status, resid, gamma, 1e-6,
                          None, xout, None, ar.desc)
        torch.cuda.synchronize()
        assert int(status) == 0
        assert torch.equal(xout, xnew)
        assert torch.equal(got, want)
    # argmax merge over the same buffers (world 1: the local pairs)
    mv = torch.tensor([[1.5, 7.0], [-2.0, 3.0]], device="cuda")
    mv[:, 1] = torch.tensor([7, 3], dtype=torch.int32, device="cuda").view(torch.float32)
    ids = torch.zeros(2, dtype=torch.int32, device="cuda")
    C.argmax_merge_ar(mv, ids, ar.desc)
    torch.cuda.synchronize()
    assert ids.tolist() == [7, 3] and int(status) == 0
    # a consumer whose producer never ran times out (kTimeout = 2) and leaves the GPU usable
    C.gemv_stream_fp8(None, None, lq.w.cuda(), lq.s.cuda(), got, None, status, resid, gamma, 1e-6,
                      None, xout, None, ar.desc)
    torch.cuda.synchronize()
    assert int(status) == 2
    ar.close()


def _small_cfg():
    from vllm_moet_b200.config import ds4_flash_config
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


def _tp_engine(rank, world, fused, ep=False, attn="shard"):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    os.environ["MOET_TP_FUSED"] = "1" if fused else "0"     # read by set_tp_group
    os.environ["MOET_TP_ATTN"] = attn                         # read by LLM (random-init weights)
    cfg = _small_cfg()
    llm = LLM(cfg, device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              tensor_parallel_size=world, tp_group=dist.group.WORLD, tp_rank=rank, expert_parallel=ep)
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(3, 2048, (n,), generator=g).tolist() for n in (37, 64)]
    outs = [o.outputs[0].token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True))]
    # teacher-forced oracle check of the first prompt (TP oracle over the same shards)
    cs = reference.rope_cos_sin(cfg, 256, "cuda")
    toks, worst = list(prompts[0]), 0.0
    with reference.tp_context(dist.group.WORLD):
        for tok in outs[0]:
            lg, _ = reference.forward(llm.mw, torch.tensor(toks, device="cuda"),
                                      torch.arange(len(toks), device="cuda"), cs)
            row = lg[-1]
            worst = max(worst, float(row.max() - row[tok]) / (float(row.std()) + 1e-6))
            toks.append(tok)
    return outs, worst


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [True, False])
def test_tp2_engine_tracks_oracle(fused):
    res = run_ranks(_tp_engine, 2, fused, backend="nccl", env={"NCCL_NVLS_ENABLE": "0"})
    (o0, w0), (o1, w1) = res
    assert o0 == o1                      # both ranks emit the same tokens
    assert all(len(o) == 10 for o in o0)
    assert max(w0, w1) < 0.5, (w0, w1)   # each token is the oracle argmax or a near-tie


def _pp_engine(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    cfg = _small_cfg()
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(3, 2048, (n,), generator=g).tolist() for n in (33, 70)]
    sp = SamplingParams(max_tokens=10, ignore_eos=True)
    llm = LLM(cfg, device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              pipeline_parallel_size=world, pp_group=dist.group.WORLD, pp_rank=rank)
    outs = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    ref = None
    if rank == 0:     # the same model on one GPU (per-layer weight streams make it identical)
        one = LLM(cfg, device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2, cuda_graphs=False)
        ref = [o.outputs[0].token_ids for o in one.generate(prompts, sp)]
    return outs, ref


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pp2_matches_single_gpu():
    (o0, ref), (o1, _) = run_ranks(_pp_engine, 2, backend="nccl", env={"NCCL_NVLS_ENABLE": "0"})
    assert o0 == o1 == ref


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep2_engine_tracks_oracle():
    """Expert parallelism inside the TP group (each rank owns half of the experts whole)."""
    res = run_ranks(_tp_engine, 2, False, True, backend="nccl", env={"NCCL_NVLS_ENABLE": "0"})
    (o0, w0), (o1, w1) = res
    assert o0 == o1 and all(len(o) == 10 for o in o0)
    assert max(w0, w1) < 0.5, (w0, w1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_replicated_attention_engine_tracks_oracle():
    """TP2 with replicated attention (whole attention per rank, no o_proj reduction; experts
    and dense FFN sharded and reduced): identical tokens on both ranks, each the oracle's argmax
    or a near-tie under the same replication."""
    res = run_ranks(_tp_engine, 2, False, False, "replicate", backend="nccl", env={"NCCL_NVLS_ENABLE": "0"})
    (o0, w0), (o1, w1) = res
    assert o0 == o1 and all(len(o) == 10 for o in o0)
    assert max(w0, w1) < 0.5, (w0, w1)

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


def _small_cfg():
    from vllm_moet_b200.config import ds4_flash_config
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


def _tp_engine(rank, world, fused, ep=False):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    os.environ["MOET_TP_FUSED"] = "1" if fused else "0"     # read by set_tp_group
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

"""Trellis base tier kernels (csrc/kernels/trellis.cu) against the fp32 CPU path of the
same packs: the input / output rotations, the decode GEMV over expert groups (1, 3 and
9 tokens: one row, several rows, and experts split over two groups), both codebooks,
2 / 3 / 4 bits, widths whose Hadamard block is below 128 and n-tile counts that do not
fill the last CTA."""
import pytest
import torch

from vllm_moet_b200.formats import trellis as tf
from vllm_moet_b200.residency import trellis_tier as tt

pytestmark = pytest.mark.gpu


def _random_pack(d, E, H, I, K13, K2, L, codebook, seed):
    """A pack of random words and scale vectors: the kernels' arithmetic does not depend
    on the words being a good encoding."""
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    out = {}
    for e in range(E):
        for name, (n, k, K) in {"w1": (I, H, K13), "w3": (I, H, K13), "w2": (H, I, K2)}.items():
            out[f"e{e}.{name}.k{K}.trellis"] = torch.randint(-32768, 32768, (k // 16, n // 16, 16 * K), generator=g,
                                                             dtype=torch.int64).to(torch.int16)
            out[f"e{e}.{name}.k{K}.suh"] = ((torch.rand(k, generator=g) + 0.5) *
                                           (torch.randint(0, 2, (k,), generator=g) * 2 - 1)).half() * 0.1
            out[f"e{e}.{name}.k{K}.svh"] = ((torch.rand(n, generator=g) + 0.5) *
                                           (torch.randint(0, 2, (n,), generator=g) * 2 - 1)).half() * 0.1
    save_file(out, tt.pack_path(str(d), 0), metadata={
        "format": tf.FORMAT, "L": str(L), "codebook": codebook, "num_experts": str(E),
        "w13_k": str(K13), "w2_k": str(K2)})


def _rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().norm().clamp_min(1e-30))


def test_trellis_rotations_match_fwht():
    from vllm_moet_b200.ops import native
    C = native()
    torch.manual_seed(0)
    for n in (96, 384, 4096):
        x = torch.randn(3, n, device="cuda")
        su = (torch.randn(5, n, device="cuda")).half()
        src = torch.tensor([2, 0, -1, 1], dtype=torch.int32, device="cuda")
        eid = torch.tensor([4, 0, 1, 3], dtype=torch.int32, device="cuda")
        out = torch.empty(4, n, device="cuda")
        C.trellis_rot_in(x, src, eid, su, out)
        for p in range(4):
            if int(src[p]) < 0:
                assert (out[p] == 0).all()
                continue
            want = tf.fwht((x[int(src[p])] * su[int(eid[p])].float()).double().cpu())
            assert _rel(out[p], want) < 1e-5
        sc = torch.rand(4, device="cuda")
        y = torch.empty_like(out)
        C.trellis_rot_out(out, eid, su, sc, y)
        for p in range(4):
            want = tf.fwht(out[p].double().cpu()) * su[int(eid[p])].double().cpu() * float(sc[p])
            assert _rel(y[p], want) < 1e-5


@pytest.mark.parametrize("K13,K2,L,codebook", [(2, 2, 16, "3inst"), (3, 4, 12, "1mad"), (2, 3, 16, "1mad")])
def test_trellis_tier_gpu_matches_cpu(tmp_path, K13, K2, L, codebook):
    E, H, I = 8, 384, 96
    _random_pack(tmp_path, E, H, I, K13, K2, L, codebook, seed=K13 * 10 + K2)
    cpu = tt.TrellisBaseTier(str(tmp_path), [0], act_limit=7.0)
    gpu = tt.TrellisBaseTier(str(tmp_path), [0], device="cuda", act_limit=7.0)
    g = torch.Generator().manual_seed(3)
    for T in (1, 3, 9):
        x = torch.randn(T, H, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:4] for _ in range(T)])
        w = torch.rand(T, 4, generator=g)
        mask = torch.zeros(T, 4, dtype=torch.bool)
        mask[0, 1] = True
        for m in (None, mask):
            want = cpu.forward_topk(0, x, ids, w, fp4_mask=m)
            got = gpu.forward_topk(0, x.cuda(), ids.cuda(), w.cuda(),
                                   fp4_mask=None if m is None else m.cuda())
            torch.cuda.synchronize()
            assert got.shape == (T, H) and got.is_cuda
            assert _rel(got, want) < 1e-4, (T, m is not None)
        # deterministic: fixed-order sums everywhere
        again = gpu.forward_topk(0, x.cuda(), ids.cuda(), w.cuda())
        assert torch.equal(again, gpu.forward_topk(0, x.cuda(), ids.cuda(), w.cuda()))


def test_trellis_delta_pool_gpu_matches_cpu(tmp_path):
    E, H, I = 8, 256, 128
    _random_pack(tmp_path, E, H, I, 2, 2, 12, "3inst", seed=11)
    g = torch.Generator().manual_seed(4)
    true = [(torch.randn(2 * I, H, generator=g) * 0.01, torch.randn(H, I, generator=g) * 0.01) for _ in range(3)]
    tiers = {}
    for dev in ("cpu", "cuda"):
        t = tt.TrellisBaseTier(str(tmp_path), [0], device=dev, act_limit=7.0)
        pool = tt.TrellisDeltaPool(t, slots=2, dk13=2, dk2=3, L=8)
        for e in (2, 5, 7):                       # the third promotion evicts expert 2
            pool.promote(0, e, *true[(2, 5, 7).index(e)])
        tiers[dev] = (t, pool)
    assert torch.equal(tiers["cuda"][1].slot_of[0], tiers["cpu"][1].slot_of[0])
    for T in (1, 4):
        x = torch.randn(T, H, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:4] for _ in range(T)])
        ids[0] = torch.tensor([5, 7, 0, 2])        # both pooled experts, one evicted, one never pooled
        w = torch.rand(T, 4, generator=g)
        want = tiers["cpu"][0].forward_topk(0, x, ids, w, delta=tiers["cpu"][1])
        got = tiers["cuda"][0].forward_topk(0, x.cuda(), ids.cuda(), w.cuda(), delta=tiers["cuda"][1])
        torch.cuda.synchronize()
        assert _rel(got, want) < 1e-4, T


def test_gpu_engine_serves_the_trellis_tier(tmp_path):
    """The GPU engine with trellis packs: its prefill logits track the fp32 oracle whose MoE
    blocks run through the same tier (routing, per-pair outputs, weighted combine with the
    residual and the shared expert), and graph-replayed decode is deterministic."""
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.config import ds4_flash_config
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    cfg = ds4_flash_config(num_layers=2, hidden=1024, vocab=2048, num_experts=8, moe_intermediate=128,
                           dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=2)
    base = LLM(cfg, device="cuda", num_speculative_tokens=0, max_model_len=512, max_num_seqs=2, seed=0)
    layers = tt.write_model_packs(base.mw, str(tmp_path), L=8, device=torch.device("cuda"))
    del base
    torch.cuda.empty_cache()
    llm = LLM(cfg, device="cuda", num_speculative_tokens=0, max_model_len=512, max_num_seqs=2, seed=0,
              trellis_pack=str(tmp_path))
    assert llm.trellis is not None and sorted(llm.trellis.layers) == layers and llm.runner.trellis is llm.trellis
    g = torch.Generator().manual_seed(21)
    p = torch.randint(3, 2048, (40,), generator=g).tolist()
    st = llm._state(1)
    blocks = llm.blocks.allocate("tr", 128)
    bt = torch.zeros(1, llm.max_blocks, dtype=torch.int32)
    bt[0, :len(blocks)] = torch.tensor(blocks)
    st.block_table.copy_(bt)
    llm.runner.prefill([p], [bt[0].tolist()], [0], st)
    lg = llm.runner.ws_prefill.bufs[("main.logits", torch.float32)].reshape(-1, cfg.vocab)[-1].clone()
    llm.blocks.release("tr")
    cs = reference.rope_cos_sin(llm.cfg, 256, "cuda")
    with reference.moe_context(llm.trellis.moe_fn(llm.mw)):
        want, _ = reference.forward(llm.mw, torch.tensor(p, device="cuda"), torch.arange(len(p), device="cuda"), cs)
    assert _rel(lg, want[-1]) < 0.1
    sp = SamplingParams(max_tokens=8, ignore_eos=True)
    a = [o.outputs[0].token_ids for o in llm.generate([p, p[:17]], sp)]
    b = [o.outputs[0].token_ids for o in llm.generate([p, p[:17]], sp)]
    assert a == b and all(len(x) == 8 for x in a)

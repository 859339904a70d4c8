"""GPU engine end to end on a reduced DS4-Flash-shaped model (same attention
dims, fewer/smaller layers): native logits vs the fp32 reference, CUDA graph
vs eager, determinism."""
import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import ds4_flash_config
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.models import reference

pytestmark = pytest.mark.gpu


def small_cfg():
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


@pytest.fixture(scope="module")
def llm():
    return LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)


def _prompt(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, 2048, (n,), generator=g).tolist()


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def _oracle_last_logits(llm, prompt):
    cs = reference.rope_cos_sin(llm.cfg, len(prompt) + 64, "cuda")
    t = torch.tensor(prompt, device="cuda")
    lg, _ = reference.forward(llm.mw, t, torch.arange(len(prompt), device="cuda"), cs)
    return lg[-1]


def test_prefill_logits_match_reference(llm):
    p = _prompt(70, 0)
    runner = llm.runner
    st = llm._state(1)
    blocks = llm.blocks.allocate("t", 200)
    bt = torch.zeros(1, llm.max_blocks, dtype=torch.int32)
    bt[0, :len(blocks)] = torch.tensor(blocks)
    st.block_table.copy_(bt)
    first = runner.prefill([p], [bt[0].tolist()], [0], st)
    native_logits = runner.ws_prefill.bufs[("main.logits", torch.float32)][: llm.cfg.vocab].clone()
    llm.blocks.release("t")
    cs = reference.rope_cos_sin(llm.cfg, 256, "cuda")
    t = torch.tensor(p, device="cuda")
    ref_logits, _ = reference.forward(llm.mw, t, torch.arange(len(p), device="cuda"), cs)
    r = ref_logits[-1]
    rel = float((native_logits - r).norm() / r.norm())
    assert rel < 0.08, rel
    # the native top-1 is the reference top-1 or within FP8-activation noise of it
    assert float(r[int(first[0])]) >= float(r.max()) - 0.3


def test_graph_equals_eager_and_is_deterministic(llm):
    prompts = [_prompt(40, 1), _prompt(90, 2)]
    sp = SamplingParams(max_tokens=20, ignore_eos=True)
    a = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    b = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert a == b
    assert all(len(x) == 20 for x in a)
    llm.ecfg.cuda_graphs = False
    try:
        c = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    finally:
        llm.ecfg.cuda_graphs = True
    assert a == c


def test_nodraft_step_keeps_greedy_output(llm):
    """The spec guard's no-draft step (main model over one row per sequence, no MTP pass;
    its own captured graph) emits exactly the drafting engine's greedy tokens, and drafting
    resumes on the stale drafts without changing them either."""
    prompts = [_prompt(40, 61), _prompt(77, 62)]
    sp = SamplingParams(max_tokens=12, ignore_eos=True)
    want = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    llm._spec_draft = False
    try:
        got = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    finally:
        llm._spec_draft = True
    assert got == want
    assert llm.runner.nodraft_graphs
    again = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert again == want


def test_decode_tracks_reference_greedy(llm):
    """Teacher-forced check: every emitted token is the reference argmax given
    the emitted prefix, or a near-tie in the reference logits."""
    p = _prompt(33, 3)
    out = llm.generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0].outputs[0].token_ids
    cs = reference.rope_cos_sin(llm.cfg, 256, "cuda")
    toks = list(p)
    for tok in out:
        t = torch.tensor(toks, device="cuda")
        lg, _ = reference.forward(llm.mw, t, torch.arange(len(toks), device="cuda"), cs)
        row = lg[-1]
        top = float(row.max())
        assert float(row[tok]) >= top - 0.05 * (float(row.std()) + 1e-6) * 10, (tok, int(row.argmax()))
        toks.append(tok)


def test_nvfp4_kv_engine_tracks_bf16_engine(llm):
    """The same model with a 352 B/token NVFP4 latent cache: prefill logits equal (the cache
    is not read in prefill); every decode step reads the NVFP4 cache, and its verify-row
    logits, teacher-forced on the bf16-cache engine's own tokens, stay close to the bf16
    engine's (NVFP4 KV error only); the decode is deterministic."""
    nv = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4,
             kv_cache_dtype="nvfp4")
    p = [_prompt(40, 11)]
    sp = SamplingParams(max_tokens=10, ignore_eos=True)
    a = nv.generate(p, sp)[0].outputs[0].token_ids
    b = nv.generate(p, sp)[0].outputs[0].token_ids
    ref = llm.generate(p, sp)[0].outputs[0].token_ids
    assert a == b and len(a) == 10
    assert a[0] == ref[0]
    # teacher-forced decode logits: both engines prefill the same prompt + ref prefix, then one
    # decode step reads the whole latent cache (bf16 rows vs 352-byte NVFP4 rows)
    one = SamplingParams(max_tokens=2, ignore_eos=True)
    errs = []
    for n in (0, 4, 8):
        q = [p[0] + ref[:n]]
        nv.generate(q, one)
        llm.generate(q, one)
        lg_nv, lg_bf = nv.runner.main_logits(1)[0].clone(), llm.runner.main_logits(1)[0].clone()
        errs.append(_rel(lg_nv, lg_bf))
    assert max(errs) < 0.1, errs


def test_indexer_engine(llm):
    """DSA indexer + sparse MLA: with top-k >= the context the selection is every position,
    so tokens equal the dense engine's.  With a small top-k the prompt is prefilled in
    top-k-sized chunks (sparse attention over the paged cache after the first chunk) and
    decoded sparsely; the emitted tokens track the fp32 oracle with the same DSA selection
    (teacher-forced), and the run is deterministic."""
    p = [_prompt(45, 21)]
    sp = SamplingParams(max_tokens=8, ignore_eos=True)
    ref = llm.generate(p, sp)[0].outputs[0].token_ids
    full = LLM(small_cfg().replace(index_heads=8, index_topk=2048), device="cuda", num_speculative_tokens=2,
               max_model_len=1024, max_num_seqs=4)
    assert full.generate(p, sp)[0].outputs[0].token_ids == ref
    del full
    # top-k 64 over a 150-token prompt: chunks [0, 64) dense (exact), [64, 128) and [128, 150)
    # sparse over the paged cache.  The final prefill logits sit at the quantisation floor
    # from the fp32 oracle with the same DSA selection (0.124 with no sparsity on this
    # model) and far from the dense oracle; smaller top-k makes the comparison depend on
    # selection flips of the fp8-quantised indexer inputs near the boundary.
    sparse = LLM(small_cfg().replace(index_heads=8, index_topk=64), device="cuda", num_speculative_tokens=2,
                 max_model_len=1024, max_num_seqs=4)
    p = [_prompt(150, 22)]
    a = sparse.generate(p, sp)[0].outputs[0].token_ids
    assert [(s0, e) for _, s0, e, _ in sparse._chunk_log] == [(0, 64), (64, 128), (128, 150)]
    b = sparse.generate(p, SamplingParams(max_tokens=1, ignore_eos=True))[0].outputs[0].token_ids
    lg = sparse.runner.ws_prefill.bufs[("main.logits", torch.float32)][: sparse.cfg.vocab].clone()
    assert a == sparse.generate(p, sp)[0].outputs[0].token_ids and len(a) == 8 and b[0] == a[0]
    cs = reference.rope_cos_sin(sparse.cfg, 512, "cuda")
    t = torch.tensor(p[0], device="cuda")
    ref_sparse = reference.forward(sparse.mw, t, torch.arange(150, device="cuda"), cs)[0][-1]
    cfg0 = sparse.mw.cfg
    sparse.mw.cfg = cfg0.replace(index_topk=4096)
    try:
        ref_dense = reference.forward(sparse.mw, t, torch.arange(150, device="cuda"), cs)[0][-1]
    finally:
        sparse.mw.cfg = cfg0
    e_s, e_d = _rel(lg, ref_sparse), _rel(lg, ref_dense)
    assert e_s < 0.2 and e_s < 0.5 * e_d, (e_s, e_d)
    assert float(ref_sparse[a[0]]) >= float(ref_sparse.max()) - 0.5 * (float(ref_sparse.std()) + 1e-6)


@pytest.mark.parametrize("tp,ep", [(4, False), (8, False), (8, True)])
def test_tp_shard_shapes_run_on_one_gpu(tp, ep):
    """Rank 0's shards of a TP4 / TP8 DS4-dims model (4 or 8 heads, expert shards of
    384 / 192 rows, padded FFN shards, a vocab slice) run through every prefill and
    decode kernel on one GPU (no group: partial sums are not reduced, so only the
    shape paths are checked)."""
    from vllm_moet_b200.config import ds4_flash_config
    cfg = ds4_flash_config(num_layers=2, num_experts=16, vocab=4096)
    llm = LLM(cfg, device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=2,
              tensor_parallel_size=tp, tp_rank=0, expert_parallel=ep)
    out = llm.generate([_prompt(300, 5)], SamplingParams(max_tokens=6, ignore_eos=True))
    assert len(out[0].outputs[0].token_ids) == 6
    llm.runner.check_status("tp shard shapes")


def test_glm_head_dims_engine():
    """GLM-5.x attention dims (q/k nope 192, v 256, 64-wide rope) with the DSA indexer:
    non-absorbed prefill (two value chunks per head), absorbed decode with the 256-wide
    W_UV combine; prefill logits and greedy decode track the fp32 reference and the
    CUDA graph equals eager."""
    from vllm_moet_b200.config import glm52_config
    cfg = glm52_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                       dense_intermediate=512, num_dense_layers=1, num_heads=8, q_lora_rank=256, top_k=4,
                       index_heads=8, index_topk=2048)
    assert (cfg.qk_nope_dim, cfg.v_head_dim) == (192, 256)
    glm = LLM(cfg, device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)
    p = _prompt(150, 31)            # > 128 tokens: two query tiles in the prefill kernel
    sp = SamplingParams(max_tokens=8, ignore_eos=True)
    out = glm.generate([p], sp)[0].outputs[0].token_ids
    cs = reference.rope_cos_sin(glm.cfg, 512, "cuda")
    toks = list(p)
    for i, tok in enumerate(out):
        lg, _ = reference.forward(glm.mw, torch.tensor(toks, device="cuda"), torch.arange(len(toks), device="cuda"), cs)
        row = lg[-1]
        assert float(row[tok]) >= float(row.max()) - 0.5 * (float(row.std()) + 1e-6), (i, tok, int(row.argmax()))
        toks.append(tok)
    glm.ecfg.cuda_graphs = False
    try:
        assert glm.generate([p], sp)[0].outputs[0].token_ids == out
    finally:
        glm.ecfg.cuda_graphs = True
    glm.runner.check_status("glm dims")


def test_sampling_variant_of_the_decode_graph(llm):
    """temperature > 0 on one GPU: top-k 1 sampling is greedy decoding; a seeded request is
    reproducible, graph and eager alike; a greedy row batched with a sampling row is
    unchanged."""
    prompts = [_prompt(40, 11), _prompt(60, 12)]
    greedy = [o.outputs[0].token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=16, ignore_eos=True))]
    top1 = llm.generate(prompts, SamplingParams(max_tokens=16, ignore_eos=True, temperature=1.0, top_k=1))
    assert [o.outputs[0].token_ids for o in top1] == greedy
    sp = SamplingParams(max_tokens=16, ignore_eos=True, temperature=0.9, top_p=0.95, seed=5)
    a = llm.generate([prompts[1]], sp)[0].outputs[0].token_ids
    b = llm.generate([prompts[1]], sp)[0].outputs[0].token_ids
    llm.ecfg.cuda_graphs = False
    try:
        c = llm.generate([prompts[1]], sp)[0].outputs[0].token_ids
    finally:
        llm.ecfg.cuda_graphs = True
    assert a == b == c and len(a) == 16
    mixed = llm.generate(prompts, [SamplingParams(max_tokens=16, ignore_eos=True), sp])
    assert mixed[0].outputs[0].token_ids == greedy[0]
    assert llm.runner.sample_graphs


def test_logit_bias_and_penalties_on_the_gpu(llm):
    """Penalties / bias run in the sampling variant: a huge bias forces its token, with and
    without presence / frequency penalties (at most 2 + 2 x 6 against a bias of 1000)."""
    p = _prompt(30, 13)
    forced = llm.generate([p], SamplingParams(max_tokens=8, ignore_eos=True, logit_bias={42: 1e4}))
    assert forced[0].outputs[0].token_ids == [42] * 8
    once = SamplingParams(max_tokens=6, ignore_eos=True, logit_bias={42: 1e3}, presence_penalty=2.0,
                          frequency_penalty=2.0)
    assert llm.generate([p], once)[0].outputs[0].token_ids == [42] * 6


def test_prefix_cached_prefill_matches_full_prefill():
    """GPU prefix caching: the second prompt's shared 128-token prefix is read from the
    first prompt's blocks (one copied, position 127 recomputed) and only the rest runs
    through the absorbed-attention ("cached") prefill; its last logits match a full
    prefill of the same prompt."""
    pc = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4,
             enable_prefix_caching=True)
    prefix = _prompt(128, 21)
    a, b = prefix + _prompt(20, 22), prefix + _prompt(30, 23)
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    pc.generate([a], sp)
    got = pc.generate([b], sp)[0].outputs[0].token_ids
    lg_cached = pc.runner.ws_prefill.bufs[("main.logits", torch.float32)][: pc.cfg.vocab].clone()
    assert pc.blocks.stats["hit_blocks"] == 2 and len(got) == 4
    full = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)
    want = full.generate([b], sp)[0].outputs[0].token_ids
    lg_full = full.runner.ws_prefill.bufs[("main.logits", torch.float32)][: full.cfg.vocab].clone()
    # both native paths against the fp32 oracle: the cached (absorbed-attention) prefill is
    # within the full prefill's own tolerance and not materially worse than it
    r = _oracle_last_logits(pc, b)
    e_cached, e_full = _rel(lg_cached, r), _rel(lg_full, r)
    assert e_cached < 0.1 and e_cached <= e_full + 0.02, (e_cached, e_full)
    assert got[0] == want[0] or float(r[got[0]]) >= float(r.max()) - 0.3


def test_chunked_prefill_matches_full_prefill():
    """GPU chunked prefill: a 150-token prompt prefilled 48 tokens a step (first chunk
    dense, then the cached mode) ends with the same last logits as one full prefill."""
    ch = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4,
             enable_chunked_prefill=True, max_num_batched_tokens=48)
    p = _prompt(150, 31)
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    got = ch.generate([p], sp)[0].outputs[0].token_ids
    lg_chunked = ch.runner.ws_prefill.bufs[("main.logits", torch.float32)][: ch.cfg.vocab].clone()
    assert len(ch._chunk_log) == 4 and len(got) == 4
    full = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)
    full.generate([p], sp)
    lg_full = full.runner.ws_prefill.bufs[("main.logits", torch.float32)][: full.cfg.vocab].clone()
    r = _oracle_last_logits(ch, p)
    e_chunked, e_full = _rel(lg_chunked, r), _rel(lg_full, r)
    assert e_chunked < 0.08 and e_chunked <= e_full + 0.03, (e_chunked, e_full)


@pytest.mark.parametrize("flash_min", [128, 1 << 30])
def test_chunked_prefill_flash_and_absorbed_paths(flash_min):
    """Chunks of 128 rows over cached positions: with the flash path (key rows gathered from
    the cache, W_kv_b applied, flash kernel with the queries at the end of each key range)
    and with absorbed attention over the paged cache, the last logits track the fp32
    oracle as closely as one full prefill does."""
    ch = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4,
             enable_chunked_prefill=True, max_num_batched_tokens=128)
    ch.runner.cached_flash_min = flash_min
    p = _prompt(400, 41)
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    got = ch.generate([p], sp)[0].outputs[0].token_ids
    lg = ch.runner.ws_prefill.bufs[("main.logits", torch.float32)][: ch.cfg.vocab].clone()
    assert len(ch._chunk_log) == 4 and len(got) == 4
    assert (("kvbk", torch.bfloat16) in ch.runner.ws_prefill.bufs) == (flash_min == 128)
    full = LLM(small_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)
    want = full.generate([p], sp)[0].outputs[0].token_ids
    lg_full = full.runner.ws_prefill.bufs[("main.logits", torch.float32)][: full.cfg.vocab].clone()
    r = _oracle_last_logits(ch, p)
    e, e_full = _rel(lg, r), _rel(lg_full, r)
    assert e < 0.1 and e <= e_full + 0.03, (e, e_full)
    assert got[0] == want[0] or float(r[got[0]]) >= float(r.max()) - 0.3

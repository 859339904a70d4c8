"""Hyper-connections (DeepSeek-V4 mHC) on the GPU: the site kernels against the fp32
oracle's hc_pre / hc_post / hc_head, and the engine (prefill logits, MTP draft logits,
greedy decode) of a reduced DS4-shaped model with four residual streams against the
oracle model."""
import types

import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import ds4_flash_config
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.models import reference
from vllm_moet_b200.models.weights import HyperConn

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def C():
    from vllm_moet_b200.ops import native
    return native()


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def _site(g, rows, n, H):
    return HyperConn((torch.randn(rows, n * H, generator=g) * 0.02).to(DEV),
                     (torch.randn(rows, generator=g) * 0.5).to(DEV),
                     (0.5 + torch.rand(3 if rows > n else 1, generator=g)).to(DEV))


@pytest.mark.parametrize("n,T", [(4, 3), (4, 1100), (2, 5)])
def test_hc_site_kernels_match_oracle(C, n, T):
    H = 1024
    cfg = types.SimpleNamespace(rms_eps=1e-6, hc_eps=1e-6, hc_sinkhorn_iters=20)
    g = torch.Generator().manual_seed(n * 1000 + T)
    x0 = torch.randn(T, n, H, generator=g).to(DEV)
    prev, site, head = _site(g, (n + 2) * n, n, H), _site(g, (n + 2) * n, n, H), _site(g, n, n, H)
    out = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    _, post0, comb0 = reference.hc_pre(cfg, prev, x0)
    # block site with the previous block's update pending
    xs = x0.clone()
    R = (n + 2) * n
    part = torch.empty(H // 128, T, R + 1, device=DEV)
    h = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    post, comb = torch.empty(T, n, device=DEV), torch.empty(T, n, n, device=DEV)
    C.hc_mix(xs, out, post0.contiguous(), comb0.contiguous(), site.fn.contiguous(), part)
    C.hc_apply(xs, part, site.base, site.scale, cfg.hc_eps, cfg.hc_sinkhorn_iters, cfg.rms_eps, h, post, comb)
    x1 = reference.hc_post(out, x0, post0, comb0)
    h_ref, post_ref, comb_ref = reference.hc_pre(cfg, site, x1)
    assert _rel(xs, x1) < 1e-5
    assert _rel(post, post_ref) < 1e-4 and _rel(comb, comb_ref) < 1e-3
    assert _rel(h, h_ref) < 1e-2
    # head site (gated sum), no update
    part_h = torch.empty(H // 128, T, n + 1, device=DEV)
    C.hc_mix(xs, fn=head.fn.contiguous(), part=part_h)
    C.hc_apply(xs, part_h, head.base, head.scale, cfg.hc_eps, cfg.hc_sinkhorn_iters, cfg.rms_eps, h)
    assert _rel(h, reference.hc_head(cfg, head, x1)) < 1e-2
    # update only
    C.hc_mix(xs, out, post, comb)
    assert _rel(xs, reference.hc_post(out, x1, post_ref, comb_ref)) < 1e-4


def _cfg():
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4, hc_mult=4)


@pytest.fixture(scope="module")
def llm():
    return LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)


def _prompt(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, 2048, (n,), generator=g).tolist()


def _prefill_logits(llm, p):
    """-> (first token, main logits of the last row, the last MTP pass's logits -- the
    draft chain's second pass, at position len(p) from the first draft -- and the first
    draft)."""
    st = llm._state(1)
    blocks = llm.blocks.allocate("hc", 200)
    bt = torch.zeros(1, llm.max_blocks, dtype=torch.int32)
    bt[0, :len(blocks)] = torch.tensor(blocks)
    st.block_table.copy_(bt)
    first = llm.runner.prefill([p], [bt[0].tolist()], [0], st)
    bufs = llm.runner.ws_prefill.bufs
    lg = bufs[("main.logits", torch.float32)][: llm.cfg.vocab].clone()
    mlg = bufs[("mtp.logits", torch.float32)][: llm.cfg.vocab].clone()
    d1 = int(st.tokens[0, 1])           # drafts follow the first token in the decode row
    llm.blocks.release("hc")
    return first, lg, mlg, d1


def test_hc_engine_prefill_and_mtp_logits(llm):
    """Prefill and MTP draft logits against the fp32 oracle with four streams, within the
    tolerance of FP8 activations through three layers.  The MTP oracle runs both draft
    passes: the prompt rows (next tokens, the main model's streams) and then the first
    draft at the next position, fed the MTP layer's own output streams."""
    p = _prompt(70, 5)
    first, lg, mlg, d1 = _prefill_logits(llm, p)
    cs = reference.rope_cos_sin(llm.cfg, 256, DEV)
    t = torch.tensor(p, device=DEV)
    T = len(p)
    pos = torch.arange(T + 1, device=DEV)
    ref, hid = reference.forward(llm.mw, t, pos[:T], cs)
    assert hid.shape == (T, 4 * llm.cfg.hidden)       # the oracle really runs four streams
    nxt = torch.cat([t[1:], first[:1].to(t.dtype)])
    m1, mh = reference.mtp_forward(llm.mw, hid, nxt, pos[:T], cs)
    m2, _ = reference.mtp_forward(llm.mw, torch.cat([hid, mh[-1:]]), torch.cat([nxt, nxt.new_tensor([d1])]), pos, cs)
    e, em = _rel(lg, ref[-1]), _rel(mlg, m2[-1])
    print(f"hc engine vs oracle: main {e:.4f} mtp (second pass) {em:.4f}")
    assert e < 0.12 and em < 0.15, (e, em)
    assert float(ref[-1][int(first[0])]) >= float(ref[-1].max()) - 0.3
    assert float(m1[-1][d1]) >= float(m1[-1].max()) - 0.3      # the first draft is the MTP argmax


def test_hc_identity_mixes_equal_the_single_stream_engine(llm):
    """Mixing weights that route everything through stream 0 (pre = gate = one-hot,
    comb = identity, post = 1) turn the four-stream model into the single-stream model
    with the same other weights: the engines' prefill and MTP logits then agree to the
    activation rounding, which pins the plumbing (sites, update order, MTP streams)."""
    n = 4
    big = 30.0
    saved = {k: tuple(t.clone() for t in v) for k, v in llm.runner._hc.items()}
    try:
        for fn, base, scale in llm.runner._hc.values():
            fn.zero_()
            scale.fill_(1.0)
            R = fn.shape[0]
            b = torch.full((R,), -big, device=DEV)
            b[0] = big                                     # pre / gate: stream 0 only
            if R > n:
                b[n:2 * n] = 0.0                           # post = 2 sigmoid(0) = 1
                b[2 * n:] = (torch.eye(n, device=DEV) * 2 * big - big).flatten()   # comb = identity
            base.copy_(b)
        p = _prompt(70, 7)
        first, lg, mlg, _ = _prefill_logits(llm, p)
    finally:
        for k, v in saved.items():
            for dst, src in zip(llm.runner._hc[k], v):
                dst.copy_(src)
    cfg1 = ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)
    plain = LLM(cfg1, device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=4)
    first1, lg1, mlg1, _ = _prefill_logits(plain, p)
    e, em = _rel(lg, lg1), _rel(mlg, mlg1)
    print(f"hc identity vs single stream: main {e:.4f} mtp {em:.4f}")
    # the single-stream engine keeps its residual in bf16, the streams are f32; the MTP
    # module of the four-stream model also zeroes the position-0 embedding
    assert e < 0.08 and em < 0.1, (e, em)


def test_hc_engine_decode_tracks_reference_greedy(llm):
    p = _prompt(33, 6)
    sp = SamplingParams(max_tokens=8, ignore_eos=True)
    out = llm.generate([p], sp)[0].outputs[0].token_ids
    assert llm.generate([p], sp)[0].outputs[0].token_ids == out          # graphs replay deterministically
    cs = reference.rope_cos_sin(llm.cfg, 256, DEV)
    toks = list(p)
    for tok in out:
        lg, _ = reference.forward(llm.mw, torch.tensor(toks, device=DEV), torch.arange(len(toks), device=DEV), cs)
        row = lg[-1]
        assert float(row[tok]) >= float(row.max()) - 0.5 * float(row.std()), (tok, int(row.argmax()))
        toks.append(tok)

"""Numerics of every native kernel against a plain PyTorch fp32/fp64 reference."""
import math

import pytest
import torch

from vllm_moet_b200.formats import codebook, fp8, kv_nvfp4, planes

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def C():
    from vllm_moet_b200.ops import native
    return native()


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def rand_e4m3(shape, g):
    x = torch.randn(shape, generator=g) * 2
    return x.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)


# ------------------------------------------------------------------------- quantisation
@pytest.mark.parametrize("T,H", [(1, 512), (5, 4096), (33, 1024)])
def test_rmsnorm_quant(C, T, H):
    g = torch.Generator().manual_seed(T)
    x = (torch.randn(T, H, generator=g) * 3).to(torch.bfloat16)
    add = (torch.randn(T, H, generator=g)).to(torch.bfloat16)
    w = (torch.rand(H, generator=g) + 0.5).to(torch.bfloat16)
    xd, ad, wd = x.to(DEV), add.to(DEV), w.to(DEV)
    xo = torch.empty_like(xd)
    y = torch.empty_like(xd)
    q0 = torch.empty(T, H, dtype=torch.uint8, device=DEV); s0 = torch.empty(T, H // 64, dtype=torch.uint8, device=DEV)
    q1 = torch.empty_like(q0); s1 = torch.empty_like(s0)
    C.rmsnorm_quant(xd, ad, xo, wd, 1e-6, y, q0, s0, q1, s1, 0)
    xs = (x.float() + add.float()).to(torch.bfloat16)
    assert torch.equal(xo.cpu(), xs)
    ref = (xs.float() * torch.rsqrt(xs.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(torch.bfloat16)
    assert rel(y.cpu().float(), ref.float()) < 1e-2
    rq, rs = fp8.quant_act_fp8(y.cpu().float())
    assert (s0.cpu() == rs).float().mean() > 0.99
    deq = fp8.dequant_act_fp8(q0.cpu().view(torch.float8_e4m3fn), s0.cpu())
    assert rel(deq, y.cpu().float()) < 4e-2
    # w2 layout is the natural bytes permuted inside 32-blocks
    assert torch.equal(q1.cpu(), fp8.to_w2_layout(q0.cpu()))
    assert torch.equal(s1.cpu(), s0.cpu())


def test_swiglu_quant(C):
    g = torch.Generator().manual_seed(0)
    R, I = 7, 256
    x = torch.randn(R, 2 * I, generator=g) * 8
    q = torch.empty(R, I, dtype=torch.uint8, device=DEV); s = torch.empty(R, I // 64, dtype=torch.uint8, device=DEV)
    C.swiglu_quant(x.to(DEV), 10.0, None, 0, q, s)
    gt, up = x[:, :I].clamp(max=10), x[:, I:].clamp(-10, 10)
    ref = (torch.nn.functional.silu(gt) * up).to(torch.bfloat16).float()
    deq = fp8.dequant_act_fp8(q.cpu().view(torch.float8_e4m3fn), s.cpu())
    assert rel(deq, ref) < 4e-2


# ------------------------------------------------------------------------- dense FP8 GEMV
@pytest.mark.parametrize("T,N,K", [(1, 1600, 4096), (3, 96, 512), (13, 256, 1024), (40, 4096, 128), (96, 130, 192)])
def test_gemv_fp8(C, T, N, K):
    g = torch.Generator().manual_seed(N + T)
    a = rand_e4m3((T, K), g)
    sa = torch.randint(120, 134, (T, K // 64), generator=g, dtype=torch.uint8)
    w = rand_e4m3((N, K), g)
    sw = torch.randint(118, 130, ((N + 127) // 128, (K + 127) // 128), generator=g, dtype=torch.uint8)
    out = torch.empty(T, N, dtype=torch.float32, device=DEV)
    C.gemv_fp8(a.to(DEV), sa.to(DEV), w.to(DEV), sw.to(DEV), out, None)
    A = fp8.dequant_act_fp8(a.view(torch.float8_e4m3fn), sa).double()
    Wd = w.view(torch.float8_e4m3fn).double() * torch.exp2(sw.double() - 127).repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)[:, :K]
    ref = A @ Wd.t()
    assert rel(out.cpu(), ref) < 1e-4
    # bf16 output + residual
    res = torch.randn(T, N, generator=g).to(torch.bfloat16)
    outb = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    C.gemv_fp8(a.to(DEV), sa.to(DEV), w.to(DEV), sw.to(DEV), outb, res.to(DEV))
    assert rel(outb.cpu().float(), ref.float() + res.float()) < 1e-2


def test_gemv_fp8_batched(C):
    g = torch.Generator().manual_seed(7)
    B, T, N, K = 4, 3, 512, 128
    a = rand_e4m3((T, B, K), g)                   # [T, B, K] viewed as [B, T, K]
    sa = torch.randint(120, 134, (T, B, K // 64), generator=g, dtype=torch.uint8)
    w = rand_e4m3((B, N, K), g)
    sw = torch.randint(118, 130, (B, N // 128, 1), generator=g, dtype=torch.uint8)
    out = torch.zeros(T, B, N + 64, dtype=torch.bfloat16, device=DEV)
    C.gemv_fp8(a.to(DEV).permute(1, 0, 2), sa.to(DEV).permute(1, 0, 2), w.to(DEV), sw.to(DEV),
               out[:, :, :N].permute(1, 0, 2), None)
    for b in range(B):
        A = fp8.dequant_act_fp8(a[:, b].view(torch.float8_e4m3fn), sa[:, b]).double()
        Wd = w[b].view(torch.float8_e4m3fn).double() * torch.exp2(sw[b].double() - 127).repeat_interleave(128, 0).repeat_interleave(128, 1)
        assert rel(out[:, b, :N].cpu().float(), (A @ Wd.t()).float()) < 1e-2
    assert (out[:, :, N:] == 0).all()


# ------------------------------------------------------------------------- routing + 2-bit experts
def test_router_topk_matches_reference(C):
    from types import SimpleNamespace
    from vllm_moet_b200.config import ds4_flash_config
    from vllm_moet_b200.models.reference import route
    cfg = ds4_flash_config(n_group=8, topk_group=4)
    g = torch.Generator().manual_seed(0)
    T, E, H = 17, 256, 64
    x = torch.randn(T, H, generator=g)
    lw = SimpleNamespace(router_w=torch.randn(E, H, generator=g), router_bias=torch.randn(E, generator=g) * 0.1)
    ids_ref, w_ref = route(cfg, lw, x)
    logits = (x @ lw.router_w.t()).to(DEV)
    ids = torch.empty(T, 8, dtype=torch.int32, device=DEV); w = torch.empty(T, 8, device=DEV)
    C.router_topk(logits, lw.router_bias.to(DEV), 8, True, 8, 4, True, cfg.routed_scaling, ids, w)
    assert torch.equal(ids.cpu().long(), ids_ref)
    assert rel(w.cpu(), w_ref) < 1e-5
    # softmax router, no groups
    cfg2 = ds4_flash_config(router="softmax", norm_topk_prob=False, routed_scaling=1.0)
    ids_ref, w_ref = route(cfg2, lw, x)
    C.router_topk(logits, None, 8, False, 1, 1, False, 1.0, ids, w)
    assert torch.equal(ids.cpu().long(), ids_ref)
    assert rel(w.cpu(), w_ref) < 1e-5


def _expert_pool(E, N, K, g, lo=122, hi=130):
    codes = torch.randint(0, 4, (E, N, K), generator=g, dtype=torch.uint8)
    sc = torch.randint(lo, hi, (E, N, K // 32), generator=g, dtype=torch.uint8)
    pool = torch.stack([torch.cat([planes.pack_codes(codes[e]), planes.pack_scales(sc[e])]) for e in range(E)])
    return codes, sc, pool


@pytest.mark.parametrize("T,k,E,N,K,MB", [(1, 8, 16, 64, 256, 8), (3, 8, 16, 128, 512, 8), (40, 4, 8, 64, 192, 16),
                                          (96, 8, 32, 64, 128, 32)])
def test_moe_w2_gemv(C, T, k, E, N, K, MB):
    g = torch.Generator().manual_seed(T * 31 + E)
    codes, sc, pool = _expert_pool(E, N, K, g)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    R = T * k
    P = R // MB + min(E, R)
    dev = lambda t: t.to(DEV)  # noqa: E731
    rank, stok, posof = (torch.empty(R, dtype=torch.int32, device=DEV) for _ in range(3))
    pairs = torch.empty(P, 4, dtype=torch.int32, device=DEV); npairs = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs(dev(ids), E, MB, rank, stok, posof, pairs, npairs, status)
    assert int(status) == 0
    x = torch.randn(T, K, generator=g)
    q, s = fp8.quant_act_fp8(x)
    qw2 = fp8.to_w2_layout(q.view(torch.uint8))
    out = torch.full((R, N), float("nan"), device=DEV)
    slot_table = torch.arange(E, dtype=torch.int32, device=DEV)
    miss = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.moe_w2_gemv(dev(qw2), dev(s), stok, pairs, npairs, dev(pool), 0, N * K // 4, slot_table, out, N, K, MB, miss)
    A = fp8.dequant_act_fp8(q, s).double()
    posof_c = posof.cpu().long()
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            W = codebook.dequant_codes(codes[e], sc[e]).double()
            ref = A[t] @ W.t()
            assert rel(out[posof_c[t * k + j]].cpu(), ref) < 1e-4, (t, j)
    assert int(miss) == 0
    # K slices (grid.z): the slices summed in order equal the whole-K GEMV
    for ks in (2, 3, K // 64 + 1):
        part = torch.full((ks, R, N), float("nan"), device=DEV)
        C.moe_w2_gemv(dev(qw2), dev(s), stok, pairs, npairs, dev(pool), 0, N * K // 4, slot_table, part, N, K, MB,
                      miss)
        assert torch.allclose(part.sum(0), out, rtol=1e-5, atol=1e-4), ks
    assert int(miss) == 0
    # a missing expert writes zeros and counts a miss
    slot_table[int(ids[0, 0])] = -1
    C.moe_w2_gemv(dev(qw2), dev(s), stok, pairs, npairs, dev(pool), 0, N * K // 4, slot_table, out, N, K, MB, miss)
    assert int(miss) >= 1
    assert (out[posof_c[0]] == 0).all()


def test_moe_w2_scale_folding_wide_exponent_range(C):
    """Neighbouring k32 blocks whose exponents differ by up to 9 stay exact."""
    g = torch.Generator().manual_seed(5)
    E, N, K, T = 2, 32, 256, 2
    codes, sc, pool = _expert_pool(E, N, K, g, lo=110, hi=119)
    ids = torch.tensor([[0, 1], [1, 0]], dtype=torch.int32)
    R, MB = 4, 8
    rank, stok, posof = (torch.empty(R, dtype=torch.int32, device=DEV) for _ in range(3))
    pairs = torch.empty(R // MB + 2, 4, dtype=torch.int32, device=DEV); npairs = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs(ids.to(DEV), E, MB, rank, stok, posof, pairs, npairs, st)
    x = torch.randn(T, K, generator=g)
    q, s = fp8.quant_act_fp8(x)
    out = torch.empty(R, N, device=DEV)
    C.moe_w2_gemv(fp8.to_w2_layout(q.view(torch.uint8)).to(DEV), s.to(DEV), stok, pairs, npairs, pool.to(DEV), 0,
                  N * K // 4, torch.arange(E, dtype=torch.int32, device=DEV), out, N, K, MB, None)
    A = fp8.dequant_act_fp8(q, s).double()
    for t in range(T):
        for j in range(2):
            W = codebook.dequant_codes(codes[int(ids[t, j])], sc[int(ids[t, j])]).double()
            assert rel(out[int(posof[t * 2 + j])].cpu(), A[t] @ W.t()) < 1e-4


@pytest.mark.parametrize("impl", ["tcd"])
@pytest.mark.parametrize("T,k,E,N,K,MB,ks,lo,hi", [(1, 8, 16, 64, 256, 8, 2, 122, 130),
                                                   (3, 8, 16, 128, 4096, 8, 8, 100, 130),
                                                   (40, 4, 8, 64, 192, 16, 3, 122, 130),
                                                   (96, 8, 32, 64, 1536, 32, 3, 110, 119),
                                                   (2, 8, 16, 32, 512, 8, 1, 60, 131),
                                                   (20, 4, 8, 208, 384, 16, 3, 118, 132),
                                                   (3, 8, 16, 64, 1536, 8, 5, 120, 132)])
def test_moe_w2_tcd_sliced(C, impl, T, k, E, N, K, MB, ks, lo, hi):
    """The K-sliced tcgen05 decode expert GEMV (block-scaled MMA, scales in TMEM) summed over
    its slices in order equals the fp64 dequantised reference, over wide scale ranges,
    partial 128-row tiles and slices past the end of K; a missing expert gives zero rows
    and a miss count.  The split-aware consumers (swiglu_quant, moe_combine) equal their
    one-slice results on the summed tensor."""
    if impl == "tcd" and (K % 128 or MB not in (8, 16)):
        pytest.skip("tcgen05 decode kernel: K % 128 == 0, 8 or 16 rows per pair")
    g = torch.Generator().manual_seed(T * 131 + K)
    codes, sc, pool = _expert_pool(E, N, K, g, lo=lo, hi=hi)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    R = T * k
    P = R // MB + min(E, R)
    dev = lambda t: t.to(DEV)  # noqa: E731
    rank, stok, posof = (torch.empty(R, dtype=torch.int32, device=DEV) for _ in range(3))
    pairs = torch.empty(P, 4, dtype=torch.int32, device=DEV); npairs = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs(dev(ids), E, MB, rank, stok, posof, pairs, npairs, status)
    x = torch.randn(T, K, generator=g)
    q, s = fp8.quant_act_fp8(x)
    qw2 = dev(fp8.to_w2_layout(q.view(torch.uint8)))
    out = torch.full((ks, R, N), float("nan"), device=DEV)
    slot_table = torch.arange(E, dtype=torch.int32, device=DEV)
    miss = torch.zeros(1, dtype=torch.int32, device=DEV)
    def run():
        C.moe_w2_tcd(qw2, dev(s), stok, pairs, npairs, dev(pool), 0, N * K // 4, slot_table, out, N, K, MB, miss,
                     status)
    run()
    tot = out.sum(0).cpu().double()
    A = fp8.dequant_act_fp8(q, s).double()
    posof_c = posof.cpu().long()
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            W = codebook.dequant_codes(codes[e], sc[e]).double()
            ref = A[t] @ W.t()
            # levels 2^-10 below a group's block maximum flush: bounded by the largest term
            assert rel(tot[posof_c[t * k + j]], ref) < 1e-4, (t, j)
    assert int(miss) == 0 and int(status) == 0
    # split-aware consumers
    if N % 128 == 0:
        I = N // 2
        qa = torch.empty(R, I, dtype=torch.uint8, device=DEV); sa = torch.empty(R, I // 64, dtype=torch.uint8, device=DEV)
        qb = torch.empty_like(qa); sb = torch.empty_like(sa)
        C.swiglu_quant(out, 0.0, None, 1, qa, sa)
        C.swiglu_quant(out.sum(0).contiguous(), 0.0, None, 1, qb, sb)
        assert (qa.view(torch.float8_e4m3fn).float() - qb.view(torch.float8_e4m3fn).float()).abs().max() <= 0.5 * \
            qb.view(torch.float8_e4m3fn).float().abs().max() * 2 ** -3
    w = torch.rand(T, k, generator=g).to(DEV)
    o1 = torch.empty(T, N, dtype=torch.bfloat16, device=DEV); o2 = torch.empty_like(o1)
    C.moe_combine(out, posof, w, None, None, o1, None)
    C.moe_combine(out.sum(0).contiguous(), posof, w, None, None, o2, None)
    assert rel(o1.float().cpu(), o2.float().cpu()) < 1e-2
    # a missing expert writes zeros in every slice and counts a miss
    slot_table[int(ids[0, 0])] = -1
    run()
    assert int(miss) >= 1 and int(status) == 0
    assert (out[:, posof_c[0]] == 0).all()


def test_moe_combine(C):
    g = torch.Generator().manual_seed(3)
    T, k, H = 5, 4, 256
    y = torch.randn(T * k, H, generator=g)
    posof = torch.randperm(T * k, generator=g).int()
    w = torch.rand(T, k, generator=g)
    res = torch.randn(T, H, generator=g).to(torch.bfloat16)
    sh = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    C.moe_combine(y.to(DEV), posof.to(DEV), w.to(DEV), res.to(DEV), sh.to(DEV), out, None)
    ref = res.float() + sh.float() + sum(w[:, j:j + 1] * y[posof.view(T, k)[:, j].long()] for j in range(k))
    assert rel(out.cpu().float(), ref) < 1e-2


# ------------------------------------------------------------------------- attention
def _paged_cache(n_blocks, g):
    kv = torch.zeros(n_blocks, 64, 584, dtype=torch.bfloat16)
    kv[:, :, :576] = (torch.randn(n_blocks, 64, 576, generator=g)).to(torch.bfloat16)
    return kv


@pytest.mark.parametrize("Hh,ctx,nsplit", [(32, [1, 65, 300], 4), (16, [130], 1), (8, [64, 7], 8)])
def test_mla_decode(C, Hh, ctx, nsplit):
    g = torch.Generator().manual_seed(Hh + len(ctx))
    nseq = len(ctx)
    maxb = max(-(-c // 64) for c in ctx)
    nblk = nseq * maxb + 3
    kv = _paged_cache(nblk, g)
    perm = torch.randperm(nblk - 1, generator=g)[: nseq * maxb] + 1
    bt = perm.view(nseq, maxb).int()
    q = (torch.randn(nseq, Hh, 576, generator=g) * 0.3).to(torch.bfloat16)
    seq = torch.arange(nseq, dtype=torch.int32)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32)
    opart = torch.empty(nsplit, nseq, Hh, 512, device=DEV)
    ml = torch.empty(nsplit, nseq, Hh, 2, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(192)
    C.mla_decode(q.to(DEV), kv.to(DEV), bt.to(DEV), seq.to(DEV), pos.to(DEV), opart, ml, scale, status)
    out = torch.empty(nseq, Hh, 512, dtype=torch.bfloat16, device=DEV)
    oq = torch.empty(nseq, Hh, 512, dtype=torch.uint8, device=DEV); os_ = torch.empty(nseq, Hh, 8, dtype=torch.uint8, device=DEV)
    C.mla_combine(opart, ml, out, oq, os_)
    assert int(status) == 0
    for i, c in enumerate(ctx):
        rows = torch.cat([kv[bt[i, p // 64], p % 64:p % 64 + 1] for p in range(c)])[:, :576].float()
        s = (q[i].float() @ rows.t()) * scale
        ref = torch.softmax(s, -1) @ rows[:, :512]
        assert rel(out[i].cpu().float(), ref) < 2e-2, i
        deq = fp8.dequant_act_fp8(oq[i].cpu().view(torch.float8_e4m3fn).reshape(Hh, 512), os_[i].cpu())
        assert rel(deq, ref) < 5e-2


@pytest.mark.parametrize("lens,Hh", [([200], 2), ([130, 70, 1], 3)])
def test_mla_prefill(C, lens, Hh):
    g = torch.Generator().manual_seed(sum(lens))
    T = sum(lens)
    q = (torch.randn(T, Hh, 192, generator=g) * 0.5).to(torch.bfloat16)
    kvb = (torch.randn(T, Hh, 256, generator=g) * 0.5).to(torch.bfloat16)
    kr = (torch.randn(T, 64, generator=g) * 0.5).to(torch.bfloat16)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    out = torch.empty(T, Hh * 128, dtype=torch.bfloat16, device=DEV)
    oq = torch.empty(T, Hh * 128, dtype=torch.uint8, device=DEV); os_ = torch.empty(T, Hh * 2, dtype=torch.uint8, device=DEV)
    scale = 1 / math.sqrt(192)
    C.mla_prefill(q.to(DEV), kvb.to(DEV), kr.to(DEV), cu.to(DEV), max(lens), scale, oq, os_, out)
    for si, n in enumerate(lens):
        s0 = int(cu[si])
        for h in range(Hh):
            qq = q[s0:s0 + n, h].float()
            kk = torch.cat([kvb[s0:s0 + n, h, :128].float(), kr[s0:s0 + n].float()], -1)
            vv = kvb[s0:s0 + n, h, 128:].float()
            s = (qq @ kk.t()) * scale
            s = s.masked_fill(torch.ones(n, n).triu(1).bool(), float("-inf"))
            ref = torch.softmax(s, -1) @ vv
            assert rel(out[s0:s0 + n, h * 128:(h + 1) * 128].cpu().float(), ref) < 2e-2, (si, h)
    deq = fp8.dequant_act_fp8(oq.cpu().view(torch.float8_e4m3fn), os_.cpu())
    assert rel(deq, out.cpu().float()) < 5e-2


@pytest.mark.parametrize("qlens,klens,Hh", [([64], [200], 2), ([130, 1, 70], [130, 300, 200], 3)])
def test_mla_prefill_query_offset(C, qlens, klens, Hh):
    """Separate key batch: sequence i's queries are its last qlens[i] positions of klens[i]
    keys (a prompt chunk over cached positions); kr is a strided view, as when it is the
    rope tail of gathered cache rows."""
    g = torch.Generator().manual_seed(sum(qlens) + sum(klens))
    T, Nk = sum(qlens), sum(klens)
    q = (torch.randn(T, Hh, 192, generator=g) * 0.5).to(torch.bfloat16)
    kvb = (torch.randn(Nk, Hh, 256, generator=g) * 0.5).to(torch.bfloat16)
    rows = (torch.randn(Nk, 584, generator=g) * 0.5).to(torch.bfloat16)
    cu = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32)
    cuk = torch.tensor([0] + torch.tensor(klens).cumsum(0).tolist(), dtype=torch.int32)
    out = torch.empty(T, Hh * 128, dtype=torch.bfloat16, device=DEV)
    oq = torch.empty(T, Hh * 128, dtype=torch.uint8, device=DEV); os_ = torch.empty(T, Hh * 2, dtype=torch.uint8, device=DEV)
    scale = 1 / math.sqrt(192)
    rows_d = rows.to(DEV)
    C.mla_prefill(q.to(DEV), kvb.to(DEV), rows_d[:, 512:576], cu.to(DEV), max(qlens), scale, oq, os_, out,
                  cu_seqlens_k=cuk.to(DEV))
    kr = rows[:, 512:576]
    for si, (n, nk) in enumerate(zip(qlens, klens)):
        s0, k0, off = int(cu[si]), int(cuk[si]), nk - n
        for h in range(Hh):
            qq = q[s0:s0 + n, h].float()
            kk = torch.cat([kvb[k0:k0 + nk, h, :128].float(), kr[k0:k0 + nk].float()], -1)
            vv = kvb[k0:k0 + nk, h, 128:].float()
            s = (qq @ kk.t()) * scale
            mask = torch.arange(nk)[None, :] > (off + torch.arange(n))[:, None]
            ref = torch.softmax(s.masked_fill(mask, float("-inf")), -1) @ vv
            assert rel(out[s0:s0 + n, h * 128:(h + 1) * 128].cpu().float(), ref) < 2e-2, (si, h)
    deq = fp8.dequant_act_fp8(oq.cpu().view(torch.float8_e4m3fn), os_.cpu())
    assert rel(deq, out.cpu().float()) < 5e-2


def test_kv_prep_bf16_and_nvfp4(C):
    g = torch.Generator().manual_seed(11)
    T = 5
    kva = (torch.randn(T, 576 + 16, generator=g)).to(torch.bfloat16)[:, :576]
    w = (torch.rand(512, generator=g) + 0.5).to(torch.bfloat16)
    from vllm_moet_b200.config import ds4_flash_config
    from vllm_moet_b200.models.reference import rope_cos_sin, apply_rope
    cs = rope_cos_sin(ds4_flash_config(), 64)
    pos = torch.tensor([0, 3, 9, 17, 40], dtype=torch.int32)
    slots = torch.tensor([5, -1, 64, 70, 127], dtype=torch.int64)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    cache = torch.zeros(2, 64, 584, dtype=torch.bfloat16, device=DEV)
    lat = torch.empty(T, 512, dtype=torch.bfloat16, device=DEV); rp = torch.empty(T, 64, dtype=torch.bfloat16, device=DEV)
    C.kv_prep(kva.to(DEV), 512, 64, w.to(DEV), 1e-6, pos.to(DEV), cs.to(DEV), slots.to(DEV), 1, cache, lat, rp,
              None, None, st)
    assert int(st) == 0
    x = kva[:, :512].float()
    ref_lat = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float())
    assert rel(lat.cpu().float(), ref_lat) < 1e-2
    ref_rope = apply_rope(kva[:, 512:].float(), cs[pos.long()])
    assert rel(rp.cpu().float(), ref_rope) < 1e-2
    flat = cache.view(-1, 584).cpu()
    for t in range(T):
        if slots[t] >= 0:
            assert torch.equal(flat[slots[t], :512], lat[t].cpu())
            assert torch.equal(flat[slots[t], 512:576], rp[t].cpu())
    # NVFP4 rows are byte-identical to the golden encoder applied to the same latent/rope
    c4 = torch.zeros(128, 352, dtype=torch.uint8, device=DEV)
    C.kv_prep(kva.to(DEV), 512, 64, w.to(DEV), 1e-6, pos.to(DEV), cs.to(DEV), slots.to(DEV), 2, c4, lat, rp,
              None, None, st)
    enc = kv_nvfp4.encode(lat.cpu().float(), rp.cpu().float())
    for t in range(T):
        if slots[t] >= 0:
            assert torch.equal(c4[slots[t]].cpu(), enc[t]), t
    # out-of-range slot -> status, no trap
    bad = torch.tensor([1000, 0, 1, 2, 3], dtype=torch.int64, device=DEV)
    C.kv_prep(kva.to(DEV), 512, 64, w.to(DEV), 1e-6, pos.to(DEV), cs.to(DEV), bad, 2, c4, None, None, None, None, st)
    torch.cuda.synchronize()
    assert int(st) == 1


# ------------------------------------------------------------------------- load-time quantiser + sampling
def test_w2_quant_pack_matches_golden(C):
    g = torch.Generator().manual_seed(2)
    N, K = 48, 192
    w = torch.randn(N, K, generator=g) * 0.02
    ts = float(w.abs().max()) / (6 * 448)
    packed = torch.empty(N, K // 2, dtype=torch.uint8, device=DEV)
    sf = torch.empty(N, K // 16, dtype=torch.uint8, device=DEV)
    C.nvfp4_quant(w.to(DEV), ts, packed, sf)
    rp, rsf, rts = codebook.f32_to_nvfp4(w, ts)
    assert torch.equal(packed.cpu(), rp)
    assert torch.equal(sf.cpu(), rsf.view(torch.uint8))
    cp = torch.empty(N * K // 4, dtype=torch.uint8, device=DEV)
    sp = torch.empty(N * K // 32, dtype=torch.uint8, device=DEV)
    fp = torch.empty(N * K // 2, dtype=torch.uint8, device=DEV)
    cnt = torch.zeros(2, dtype=torch.int64, device=DEV)
    C.w2_quant_pack(packed, sf, ts, 0, cp, sp, fp, cnt)
    codes, sc, nib = codebook.nvfp4_to_codes_scales(rp, rsf, rts, mode="sign", want_nibbles=True)
    assert torch.equal(cp.cpu(), planes.pack_codes(codes))
    assert torch.equal(sp.cpu(), planes.pack_scales(sc))
    assert torch.equal(fp.cpu(), planes.pack_fp4(nib))


@pytest.mark.parametrize("zero_mode", ["auto", "sign", "alt"])
def test_batched_expert_quant_matches_golden(C, zero_mode):
    """The batched load-time quantiser (all experts of a chunk per launch, per-expert tensor
    scales and the zero-sign auto rule on the device) is byte-equal to the golden CPU
    pipeline, slot by slot; expert 1 has many exact zeros of one sign (auto -> alternate)."""
    from vllm_moet_b200.models.weights import ExpertLayout, quantize_experts_cpu, quantize_experts_gpu
    g = torch.Generator().manual_seed(9)
    n, H, I = 4, 256, 128
    w13 = torch.randn(n, 2 * I, H, generator=g) * 0.02
    w2 = torch.randn(n, H, I, generator=g) * 0.02
    w13[1, :, ::3] = 0.0
    w2[1, ::2, :] = 0.0
    w13[2] = 0.0                     # an all-zero matrix: tensor scale 1
    lay = ExpertLayout(H=H, I=I)
    ref = torch.zeros(n, lay.slot_bytes, dtype=torch.uint8)
    quantize_experts_cpu(w13, w2, lay, ref, zero_mode=zero_mode)
    got = torch.zeros(n, lay.slot_bytes, dtype=torch.uint8, device=DEV)
    quantize_experts_gpu(w13.to(DEV), w2.to(DEV), lay, got, zero_mode=zero_mode)
    for e in range(n):
        assert torch.equal(got[e].cpu(), ref[e]), e


def test_argmax_lse(C):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(6, 129280, generator=g)
    x[2, 77] = 50.0
    ids = torch.empty(6, dtype=torch.int32, device=DEV); lse = torch.empty(6, device=DEV)
    C.argmax_lse(x.to(DEV), ids, lse, None, None)
    assert torch.equal(ids.cpu().long(), x.argmax(-1))
    assert rel(lse.cpu(), torch.logsumexp(x, -1)) < 1e-5


def test_mtp_accept_and_finalize(C):
    tgt = torch.tensor([[5, 6, 7], [5, 6, 7], [5, 6, 7]], dtype=torch.int32)
    tok = torch.tensor([[1, 5, 6], [1, 5, 9], [1, 4, 6]], dtype=torch.int32)
    out = torch.empty(3, 3, dtype=torch.int32, device=DEV); acc = torch.empty(3, dtype=torch.int32, device=DEV)
    C.mtp_accept(tgt.to(DEV), tok.to(DEV), out, acc, None)
    assert acc.cpu().tolist() == [2, 1, 0]
    assert out.cpu().tolist() == [[5, 6, 7], [5, 6, -1], [5, -1, -1]]
    drafts = torch.tensor([[8, 9], [8, 9], [8, 9]], dtype=torch.int32, device=DEV)
    toks = tok.to(DEV).clone(); pos = torch.tensor([10, 10, 10], dtype=torch.int32, device=DEV)
    C.mtp_finalize(tgt.to(DEV), acc, drafts, toks, pos, None)
    assert toks.cpu().tolist() == [[7, 8, 9], [6, 8, 9], [5, 8, 9]]
    assert pos.cpu().tolist() == [13, 12, 11]


def test_rmsnorm_quant_output_stride(C):
    """Two norms writing the halves of one [T, 2H] FP8 operand (MTP concat)."""
    T, H = 6, 1024
    a = (torch.randn(T, H) * 0.02).to(torch.bfloat16).to(DEV)
    b = torch.randn(T, H).to(torch.bfloat16).to(DEV)
    w = torch.ones(H, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(T, 2 * H, dtype=torch.uint8, device=DEV)
    s = torch.full((T, 2 * H // 64), 255, dtype=torch.uint8, device=DEV)
    C.rmsnorm_quant(a, None, None, w, 1e-6, None, q, s, None, None, 2 * H)
    C.rmsnorm_quant(b, None, None, w, 1e-6, None, q[:, H:], s[:, H // 64:], None, None, 2 * H)
    qa = torch.empty(T, H, dtype=torch.uint8, device=DEV); sa = torch.empty(T, H // 64, dtype=torch.uint8, device=DEV)
    C.rmsnorm_quant(a, None, None, w, 1e-6, None, qa, sa, None, None, 0)
    assert torch.equal(q[:, :H], qa) and torch.equal(s[:, :H // 64], sa)
    C.rmsnorm_quant(b, None, None, w, 1e-6, None, qa, sa, None, None, 0)
    assert torch.equal(q[:, H:], qa) and torch.equal(s[:, H // 64:], sa)


@pytest.mark.parametrize("T,E", [(1, 256), (3, 256), (20, 256), (96, 256), (192, 384), (1000, 384), (300, 64)])
def test_router_logits(C, T, E):
    """Decode-sized (warp per expert) and prefill-sized (tensor-core tiles, T > 64) router
    logits against the fp32 product of the same bf16 operands."""
    g = torch.Generator().manual_seed(T)
    H = 4096
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    out = torch.empty(T, E, device=DEV)
    C.router_logits(x.to(DEV), w.to(DEV), out)
    assert rel(out.cpu(), x.float() @ w.float().t()) < 1e-5
    if 64 < T <= 512:      # K-sliced tiles with the in-kernel ordered reduction: same result, twice
        part = torch.empty(16 * T * E, device=DEV)
        cnt = torch.zeros(64, dtype=torch.int32, device=DEV)
        o2 = torch.empty(T, E, device=DEV)
        for _ in range(2):
            C.router_logits(x.to(DEV), w.to(DEV), o2, part, cnt)
            assert rel(o2.cpu(), x.float() @ w.float().t()) < 1e-5
        assert int(cnt.abs().sum()) == 0


@pytest.mark.parametrize("R,V", [(1, 129280), (7, 4096), (3, 100)])
def test_argmax_split_matches_torch_twice(C, R, V):
    g = torch.Generator().manual_seed(R)
    x = torch.randn(R, V, generator=g)
    x[0, V // 3] = 9.0
    x[-1, 5] = x[-1, 7] = 20.0   # tie -> lowest index
    part = torch.empty(R, 32, 3, device=DEV)
    cnt = torch.zeros(R, dtype=torch.int32, device=DEV)
    for _ in range(2):   # counters reset themselves
        ids = torch.empty(R, dtype=torch.int32, device=DEV)
        lse = torch.empty(R, device=DEV)
        C.argmax_split(x.to(DEV), ids, lse, None, part, cnt)
        assert torch.equal(ids.cpu().long(), x.argmax(-1))
        assert rel(lse.cpu(), torch.logsumexp(x, -1)) < 1e-5
    assert int(cnt.abs().sum()) == 0


@pytest.mark.parametrize("T,E,k,MB", [(3, 256, 8, 8), (1, 16, 4, 8), (40, 64, 6, 16)])
def test_moe_route_fused_matches_separate_kernels(C, T, E, k, MB):
    g = torch.Generator().manual_seed(T * 7 + E)
    H = 1024
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(E, generator=g) * 0.1).to(DEV)
    R = T * k
    P = R // MB + min(E, R)

    def bufs():
        return dict(lg=torch.empty(T, E, device=DEV), ids=torch.empty(T, k, dtype=torch.int32, device=DEV),
                    wts=torch.empty(T, k, device=DEV), rank=torch.empty(R, dtype=torch.int32, device=DEV),
                    stok=torch.empty(R, dtype=torch.int32, device=DEV), posof=torch.empty(R, dtype=torch.int32, device=DEV),
                    pairs=torch.empty(P, 4, dtype=torch.int32, device=DEV), np=torch.empty(1, dtype=torch.int32, device=DEV))
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    a = bufs()
    C.router_logits(x, w, a["lg"])
    C.router_topk(a["lg"], bias, k, True, 1, 1, True, 2.5, a["ids"], a["wts"])
    C.build_pairs(a["ids"], E, MB, a["rank"], a["stok"], a["posof"], a["pairs"], a["np"], st)
    b = bufs()
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):       # replayable: the arrival counter resets itself
        C.moe_route_fused(x, w, b["lg"], bias, k, True, 1, 1, True, 2.5, b["ids"], b["wts"], MB, b["rank"],
                          b["stok"], b["posof"], b["pairs"], b["np"], cnt, st)
    torch.cuda.synchronize()
    assert int(st) == 0 and int(cnt) == 0
    assert torch.allclose(a["lg"], b["lg"], rtol=1e-5, atol=1e-5)
    assert torch.equal(a["ids"], b["ids"]) and torch.allclose(a["wts"], b["wts"])
    n = int(a["np"])
    assert n == int(b["np"])
    # pair lists: same experts and row counts; every routing maps to a row of its expert with its token
    assert torch.equal(a["pairs"][:n, [0, 2]], b["pairs"][:n, [0, 2]])
    ids = b["ids"].view(-1).cpu(); posof = b["posof"].cpu(); stok = b["stok"].cpu(); pairs = b["pairs"][:n].cpu()
    for r in range(R):
        row = int(posof[r])
        assert int(stok[row]) == r // k
        pe = [p for p in pairs.tolist() if p[1] <= row < p[1] + p[2]]
        assert len(pe) == 1 and pe[0][0] == int(ids[r])


@pytest.mark.parametrize("T,Hh,S", [(3, 32, 8), (20, 4, 3)])
def test_mla_combine_uv(C, T, Hh, S):
    g = torch.Generator().manual_seed(T + Hh)
    op = torch.randn(S, T, Hh, 512, generator=g)
    ml = torch.stack([torch.randn(S, T, Hh, generator=g), torch.rand(S, T, Hh, generator=g) + 0.5], -1)
    ml[S - 1, 0, 0, 0] = float("-inf")      # an empty split
    wuv = torch.randn(Hh, 128, 512, generator=g) * 0.05
    from vllm_moet_b200.models.weights import Fp8Linear
    lins = [Fp8Linear.from_float(wuv[h]) for h in range(Hh)]
    W = torch.stack([l.w for l in lins]); SW = torch.stack([l.s for l in lins])
    q = torch.empty(T, Hh * 128, dtype=torch.uint8, device=DEV)
    qs = torch.empty(T, Hh * 2, dtype=torch.uint8, device=DEV)
    C.mla_combine_uv(op.to(DEV), ml.contiguous().to(DEV), W.to(DEV), SW.to(DEV), q, qs)
    # reference: exact split merge (base-2 exponent state), then the dequantised W_uv
    m, l = ml[..., 0], ml[..., 1]
    M = m.max(0).values
    e = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp2(m - M))
    olat = (e[..., None] * op).sum(0) / (e * l).sum(0)[..., None]              # [T, Hh, 512]
    wd = torch.stack([l.dequant() for l in lins])                             # [Hh, 128, 512]
    ref = torch.einsum("thk,hjk->thj", olat, wd).reshape(T, Hh * 128)
    got = fp8.dequant_act_fp8(q.cpu().view(torch.float8_e4m3fn), qs.cpu())
    assert rel(got, ref) < 4e-2


@pytest.mark.parametrize("Hh,ctx,nsplit", [(32, [1, 65, 300], 4), (8, [200], 2)])
def test_mla_decode_nvfp4_cache(C, Hh, ctx, nsplit):
    """Decode attention straight from 352-byte NVFP4 rows equals attention over
    the rows' golden decode."""
    g = torch.Generator().manual_seed(77 + Hh)
    nseq = len(ctx)
    maxb = max(-(-c // 64) for c in ctx)
    nblk = nseq * maxb + 2
    lat = torch.randn(nblk * 64, 512, generator=g)
    rope = torch.randn(nblk * 64, 64, generator=g)
    rows = kv_nvfp4.encode(lat, rope)                        # [nblk*64, 352]
    kv4 = rows.view(nblk, 64, 352)
    dl, dr = kv_nvfp4.decode(rows)
    full = torch.cat([dl, dr], 1).view(nblk, 64, 576)
    perm = torch.randperm(nblk - 1, generator=g)[: nseq * maxb] + 1
    bt = perm.view(nseq, maxb).int()
    q = (torch.randn(nseq, Hh, 576, generator=g) * 0.3).to(torch.bfloat16)
    seq = torch.arange(nseq, dtype=torch.int32)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32)
    opart = torch.empty(nsplit, nseq, Hh, 512, device=DEV)
    ml = torch.empty(nsplit, nseq, Hh, 2, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(192)
    C.mla_decode(q.to(DEV), kv4.contiguous().to(DEV), bt.to(DEV), seq.to(DEV), pos.to(DEV), opart, ml, scale, status)
    out = torch.empty(nseq, Hh, 512, dtype=torch.bfloat16, device=DEV)
    oq = torch.empty(nseq, Hh, 512, dtype=torch.uint8, device=DEV); os_ = torch.empty(nseq, Hh, 8, dtype=torch.uint8, device=DEV)
    C.mla_combine(opart, ml, out, oq, os_)
    assert int(status) == 0
    for i, c in enumerate(ctx):
        r = torch.cat([full[bt[i, p // 64], p % 64:p % 64 + 1] for p in range(c)]).to(torch.bfloat16).float()
        s = (q[i].float() @ r.t()) * scale
        ref = torch.softmax(s, -1) @ r[:, :512]
        assert rel(out[i].cpu().float(), ref) < 2e-2, i


# ------------------------------------------------------------------------- sparse attention (DSA indexer)
@pytest.mark.parametrize("Hi,ctx", [(32, [130, 64, 1]), (8, [300])])
def test_indexer_logits(C, Hi, ctx):
    g = torch.Generator().manual_seed(Hi)
    T = len(ctx)
    maxb = max(-(-c // 64) for c in ctx)
    nblk = T * maxb + 1
    kc = (torch.randn(nblk, 64, 128, generator=g) * 0.3).to(torch.bfloat16)
    bt = (torch.randperm(nblk - 1, generator=g)[: T * maxb] + 1).view(T, maxb).int()
    q = (torch.randn(T, Hi, 128, generator=g) * 0.3).to(torch.bfloat16)
    w = torch.randn(T, Hi, generator=g)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32)
    S = maxb * 64
    out = torch.empty(T, S, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.indexer_logits(q.to(DEV), w.to(DEV), kc.to(DEV), bt.to(DEV), torch.arange(T, dtype=torch.int32).to(DEV),
                     pos.to(DEV), out, st)
    assert int(st) == 0
    for i, c in enumerate(ctx):
        keys = torch.cat([kc[bt[i, p // 64], p % 64][None] for p in range(c)]).float()
        ref = (torch.relu(q[i].float() @ keys.t()) * w[i][:, None]).sum(0)
        got = out[i].cpu()
        assert torch.allclose(got[:c], ref, rtol=2e-3, atol=2e-3)
        assert bool(torch.isinf(got[c:]).all())


@pytest.mark.parametrize("S,k", [(5000, 2048), (100, 2048), (4096, 7), (131072, 2048)])
def test_indexer_topk(C, S, k):
    g = torch.Generator().manual_seed(S + k)
    x = torch.randn(3, S, generator=g)
    x[1, S // 2:] = float("-inf")                 # a row with a causal tail
    x[2, :: 3] = 0.5                               # many ties
    out = torch.empty(3, k, dtype=torch.int32, device=DEV)
    C.indexer_topk(x.to(DEV), k, out)
    out = out.cpu()
    for r in range(3):
        fin = torch.isfinite(x[r])
        n = min(k, int(fin.sum()))
        sel = out[r][:n]
        assert bool((out[r][n:] == -1).all())
        assert bool((sel[1:] > sel[:-1]).all())  # increasing positions
        # the selection is a valid top-n: its smallest value >= every unselected finite value
        vals = x[r][sel.long()]
        mask = torch.ones(S, dtype=torch.bool); mask[sel.long()] = False
        rest = x[r][mask & fin]
        if rest.numel():
            assert float(vals.min()) >= float(rest.max())
        # ties at the threshold are taken lowest-index first
        thr = float(vals.min())
        tied_unsel = ((x[r] == thr) & mask).nonzero().flatten()
        tied_sel = sel[vals == thr]
        if tied_unsel.numel() and tied_sel.numel():
            assert int(tied_sel.max()) < int(tied_unsel.min())


def test_sparse_mla_decode_selection(C):
    """mla_decode over a selection list equals dense attention over the selected rows."""
    g = torch.Generator().manual_seed(3)
    Hh, nblk = 16, 9
    kv = _paged_cache(nblk, g)
    bt = torch.arange(1, nblk, dtype=torch.int32).view(1, 8)
    ctx = 8 * 64
    q = (torch.randn(2, Hh, 576, generator=g) * 0.3).to(torch.bfloat16)
    sel = torch.full((2, 128), -1, dtype=torch.int32)
    picks = [torch.randperm(ctx, generator=g)[:100].sort().values, torch.arange(0, 70)]
    for i, pk in enumerate(picks):
        sel[i, :len(pk)] = pk.int()
    seq = torch.zeros(2, dtype=torch.int32)
    pos = torch.full((2,), ctx - 1, dtype=torch.int32)
    opart = torch.empty(4, 2, Hh, 512, device=DEV)
    ml = torch.empty(4, 2, Hh, 2, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(192)
    C.mla_decode(q.to(DEV), kv.to(DEV), bt.to(DEV), seq.to(DEV), pos.to(DEV), opart, ml, scale, st, sel.to(DEV))
    out = torch.empty(2, Hh, 512, dtype=torch.bfloat16, device=DEV)
    C.mla_combine(opart, ml, out, None, None)
    assert int(st) == 0
    for i, pk in enumerate(picks):
        rows = torch.cat([kv[bt[0, p // 64], p % 64][None] for p in pk.tolist()])[:, :576].float()
        ref = torch.softmax((q[i].float() @ rows.t()) * scale, -1) @ rows[:, :512]
        assert rel(out[i].cpu().float(), ref) < 2e-2, i


@pytest.mark.parametrize("T,N,K", [(1, 1600, 4096), (3, 4096, 4096), (8, 1000, 1024), (3, 130, 1536), (5, 16160, 2048)])
def test_gemv_stream_matches_gemv(C, T, N, K):
    g = torch.Generator().manual_seed(N + K + T)
    from vllm_moet_b200.models.weights import Fp8Linear
    lin = Fp8Linear.from_float(torch.randn(N, K, generator=g) * 0.05)
    x = torch.randn(T, K, generator=g)
    aq, sa = fp8.quant_act_fp8(x)
    aq = aq.view(torch.uint8).to(DEV); sa = sa.to(DEV)
    w, sw = lin.w.to(DEV), lin.s.to(DEV)
    ref = torch.empty(T, N, device=DEV)
    C.gemv_fp8(aq, sa, w, sw, ref, None)
    out = torch.empty(T, N, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.gemv_stream_fp8(aq, sa, w, sw, out, None, st)
    assert int(st) == 0
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3), float((out - ref).abs().max())
    resid = torch.randn(T, N, generator=g).to(torch.bfloat16).to(DEV)
    ob = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    C.gemv_stream_fp8(aq, sa, w, sw, ob, resid, st)
    assert torch.allclose(ob.float(), (ref + resid.float()), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("T,N,K", [(3, 1600, 4096), (1, 6144, 1024), (8, 512, 2048)])
def test_gemv_stream_fused_norm(C, T, N, K):
    """RMSNorm + e4m3 quantisation in the GEMV prologue equals rmsnorm_quant followed by the GEMV."""
    g = torch.Generator().manual_seed(T * N)
    from vllm_moet_b200.models.weights import Fp8Linear
    lin = Fp8Linear.from_float(torch.randn(N, K, generator=g) * 0.05)
    w, sw = lin.w.to(DEV), lin.s.to(DEV)
    x = (torch.randn(T, K + 64, generator=g) * 2).to(torch.bfloat16).to(DEV)[:, :K]   # strided rows
    gamma = (torch.rand(K, generator=g) + 0.5).to(torch.bfloat16).to(DEV)
    q = torch.empty(T, K, dtype=torch.uint8, device=DEV); s = torch.empty(T, K // 64, dtype=torch.uint8, device=DEV)
    C.rmsnorm_quant(x, None, None, gamma, 1e-6, None, q, s, None, None, 0)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = torch.empty(T, N, device=DEV)
    C.gemv_stream_fp8(q, s, w, sw, ref, None, st)
    out = torch.empty(T, N, device=DEV)
    C.gemv_stream_fp8(None, None, w, sw, out, None, st, x, gamma, 1e-6)
    assert int(st) == 0
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3), float((out - ref).abs().max())


def test_moe_gemv_delta_tier(C):
    """Experts with a delta slot are read from the direct-8 FP4 plane (MXFP4 values),
    the rest from the 2-bit base; both match their dequantised references."""
    from vllm_moet_b200.residency.delta import delta_layout, pack_delta_slot, dequant_delta_slot
    g = torch.Generator().manual_seed(5)
    E, H, I, T, k, MB = 6, 256, 128, 3, 2, 8
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.05
    w2 = torch.randn(E, H, I, generator=g) * 0.05
    from vllm_moet_b200.models.weights import ExpertLayout, quantize_experts_cpu
    lay = ExpertLayout(H=H, I=I)
    pool = torch.empty(E, lay.slot_bytes, dtype=torch.uint8)
    quantize_experts_cpu(w13, w2, lay, pool)
    sb8 = delta_layout(H, I)[0]
    rows8 = torch.stack([pack_delta_slot(w13[e], w2[e]) for e in range(E)])
    pool8 = torch.zeros(2, sb8, dtype=torch.uint8)
    table8 = torch.full((E,), -1, dtype=torch.int32)
    pool8[0], table8[1] = rows8[1], 0
    pool8[1], table8[4] = rows8[4], 1
    ids = torch.tensor([[1, 2], [4, 1], [0, 5]], dtype=torch.int32)
    R = T * k
    P = R // MB + min(E, R)
    rank = torch.empty(R, dtype=torch.int32, device=DEV); stok = torch.empty(R, dtype=torch.int32, device=DEV)
    posof = torch.empty(R, dtype=torch.int32, device=DEV); pairs = torch.empty(P, 4, dtype=torch.int32, device=DEV)
    npairs = torch.empty(1, dtype=torch.int32, device=DEV); st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs(ids.to(DEV), E, MB, rank, stok, posof, pairs, npairs, st)
    x = torch.randn(T, H, generator=g)
    q, s = fp8.quant_act_fp8(x)
    qw = fp8.to_w2_layout(q.view(torch.uint8)).to(DEV)
    out = torch.empty(R, 2 * I, device=DEV)
    o13 = delta_layout(H, I)
    C.moe_w2_gemv(qw, s.to(DEV), stok, pairs, npairs, pool.to(DEV), lay.off_codes13, lay.off_sc13,
                  torch.arange(E, dtype=torch.int32, device=DEV), out, 2 * I, H, MB, None,
                  pool8=pool8.to(DEV), codes_off8=o13[1], scale_off8=o13[2], slot_table8=table8.to(DEV))
    A = fp8.dequant_act_fp8(q, s).double()
    po = posof.cpu().long()
    from vllm_moet_b200.formats import planes as pl
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            if int(table8[e]) >= 0:
                W = dequant_delta_slot(rows8[e], H, I)[0].double()
            else:
                c13, s13, _, _ = lay.split(pool[e])
                W = pl.dequant_plane(c13, s13, 2 * I, H).double()
            assert rel(out[po[t * k + j]].cpu(), A[t] @ W.t()) < 1e-4, (t, j, e)


def test_moe_gemv_split_fp4_delta(C):
    """Split FP4 (quintal) delta slots: the GEMV rebuilds the exact MXFP4 values from the
    2-bit base codes + refinement digits (base scales); other experts read the 2-bit base;
    an expert whose base slot is missing is a miss (zero rows), never a refinement alone."""
    from vllm_moet_b200.residency.delta import split_layout, pack_split_slot, dequant_split_slot
    from vllm_moet_b200.models.weights import ExpertLayout, quantize_experts_cpu
    from vllm_moet_b200.formats import planes as pl
    g = torch.Generator().manual_seed(7)
    E, H, I, T, k, MB = 6, 256, 128, 3, 2, 8
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.05
    w2 = torch.randn(E, H, I, generator=g) * 0.05
    lay = ExpertLayout(H=H, I=I)
    pool = torch.empty(E, lay.slot_bytes, dtype=torch.uint8)
    rows = []
    for e in range(E):
        n13, n2 = quantize_experts_cpu(w13[e:e + 1], w2[e:e + 1], lay, pool[e:e + 1], want_nibbles=True)
        rows.append(pack_split_slot(n13, n2))
    sbq, o13, _, o2, _ = split_layout(H, I)
    pool8 = torch.zeros(3, sbq, dtype=torch.uint8)
    table8 = torch.full((E,), -1, dtype=torch.int32)
    for slot, e in enumerate((1, 4, 5)):
        pool8[slot], table8[e] = rows[e], slot
    base_table = torch.arange(E, dtype=torch.int32)
    base_table[5] = -1                 # refinement present, base absent -> miss
    ids = torch.tensor([[1, 2], [4, 1], [0, 5]], dtype=torch.int32)
    R = T * k
    P = R // MB + min(E, R)
    rank = torch.empty(R, dtype=torch.int32, device=DEV); stok = torch.empty(R, dtype=torch.int32, device=DEV)
    posof = torch.empty(R, dtype=torch.int32, device=DEV); pairs = torch.empty(P, 4, dtype=torch.int32, device=DEV)
    npairs = torch.empty(1, dtype=torch.int32, device=DEV); st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs(ids.to(DEV), E, MB, rank, stok, posof, pairs, npairs, st)
    A = {}
    outs = {}
    for name, (N, K, oc, osc, oq) in {"w13": (2 * I, H, lay.off_codes13, lay.off_sc13, o13),
                                      "w2": (H, I, lay.off_codes2, lay.off_sc2, o2)}.items():
        x = torch.randn(T if name == "w13" else R, K, generator=g)
        q, s = fp8.quant_act_fp8(x)
        qw = fp8.to_w2_layout(q.view(torch.uint8)).to(DEV)
        out = torch.full((R, N), float("nan"), device=DEV)
        miss = torch.zeros(1, dtype=torch.int32, device=DEV)
        C.moe_w2_gemv(qw, s.to(DEV), stok if name == "w13" else None, pairs, npairs, pool.to(DEV), oc, osc,
                      base_table.to(DEV), out, N, K, MB, miss, pool8=pool8.to(DEV), codes_off8=oq, scale_off8=0,
                      slot_table8=table8.to(DEV), quintal=True)
        torch.cuda.synchronize()
        A[name] = fp8.dequant_act_fp8(q, s).double()
        outs[name] = (out.cpu(), int(miss))
    po = posof.cpu().long()
    for name in ("w13", "w2"):
        out, miss = outs[name]
        assert miss >= 1
        for t in range(T):
            for j in range(k):
                e, r = int(ids[t, j]), int(po[t * k + j])
                arow = A[name][t] if name == "w13" else A[name][r]
                if e == 5:
                    assert (out[r] == 0).all(), "a refinement without its base must not be served"
                    continue
                c13, s13, c2, s2 = lay.split(pool[e])
                if int(table8[e]) >= 0:
                    W = dequant_split_slot(rows[e], pl.unpack_codes(c13, 2 * I, H), pl.unpack_scales(s13, 2 * I, H),
                                           pl.unpack_codes(c2, H, I), pl.unpack_scales(s2, H, I), H, I)
                    W = (W[0] if name == "w13" else W[1]).double()
                else:
                    W = (pl.dequant_plane(c13, s13, 2 * I, H) if name == "w13"
                         else pl.dequant_plane(c2, s2, H, I)).double()
                assert rel(out[r], arow @ W.t()) < 1e-4, (name, t, j, e)

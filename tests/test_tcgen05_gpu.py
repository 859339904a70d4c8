"""tcgen05 block-scaled GEMM kernels vs fp64 references (2-bit experts and dense FP8)."""
import pytest
import torch

from vllm_moet_b200.formats import codebook, fp8, planes

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def C():
    from vllm_moet_b200.ops import native
    return native()


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


@pytest.mark.parametrize("N,K", [(8, 128), (64, 256), (128, 512)])
def test_tc_block_scaled_mma_basic(C, N, K):
    g = torch.Generator().manual_seed(N + K)
    a = (torch.randn(128, K, generator=g) * 2).to(torch.float8_e4m3fn)
    b = (torch.randn(N, K, generator=g) * 2).to(torch.float8_e4m3fn)
    sa = torch.randint(122, 132, (128, K // 32), generator=g, dtype=torch.uint8)
    sb = torch.randint(122, 132, (N, K // 32), generator=g, dtype=torch.uint8)
    out = torch.zeros(N, 128, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    import moet_testkit       # test-only extension (tests/csrc)
    moet_testkit.tc_gemm_test(a.view(torch.uint8).to(DEV), sa.to(DEV), b.view(torch.uint8).to(DEV), sb.to(DEV), out, st, 3)
    A = a.double() * torch.exp2(sa.double() - 127).repeat_interleave(32, 1)
    B = b.double() * torch.exp2(sb.double() - 127).repeat_interleave(32, 1)
    assert int(st) == 0
    assert rel(out.cpu(), B @ A.t()) < 1e-5


@pytest.mark.parametrize("T,k,E,N,K,NT", [(1, 8, 16, 128, 256, 8), (3, 8, 16, 256, 512, 8), (20, 4, 8, 128, 384, 16),
                                          (96, 8, 16, 256, 128, 64), (300, 8, 16, 128, 256, 128)])
def test_tc_moe_w2(C, T, k, E, N, K, NT):
    g = torch.Generator().manual_seed(T * 7 + N)
    codes = torch.randint(0, 4, (E, N, K), generator=g, dtype=torch.uint8)
    sc = torch.randint(118, 132, (E, N, K // 32), generator=g, dtype=torch.uint8)
    pool = torch.stack([torch.cat([planes.pack_codes(codes[e]), planes.pack_scales(sc[e])]) for e in range(E)]).to(DEV)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int().to(DEV)
    R = T * k
    P = R // NT + min(E, R)
    rank, stok, posof = (torch.empty(R, dtype=torch.int32, device=DEV) for _ in range(3))
    pairs = torch.empty(P, 4, dtype=torch.int32, device=DEV); npairs = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs(ids, E, NT, rank, stok, posof, pairs, npairs, st)
    x = torch.randn(T, K, generator=g)
    q, s = fp8.quant_act_fp8(x)
    qw2 = fp8.to_w2_layout(q.view(torch.uint8)).to(DEV)
    out = torch.full((R, N), float("nan"), device=DEV)
    slots = torch.arange(E, dtype=torch.int32, device=DEV)
    miss = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.tc_moe_w2(qw2, s.to(DEV), stok, pairs, npairs, pool, 0, N * K // 4, slots, out, N, K, NT, miss, st, 0)
    torch.cuda.synchronize()
    assert int(st) == 0 and int(miss) == 0
    A = fp8.dequant_act_fp8(q, s).double()
    po = posof.cpu().long()
    ids_c = ids.cpu()
    for tt in range(T):
        for j in range(k):
            W = codebook.dequant_codes(codes[int(ids_c[tt, j])], sc[int(ids_c[tt, j])]).double()
            assert rel(out[po[tt * k + j]].cpu(), A[tt] @ W.t()) < 1e-4, (tt, j)
    # the mma.sync GEMV gives the same answer
    ref2 = torch.empty(R, N, device=DEV)
    if NT <= 32:
        C.moe_w2_gemv(qw2, s.to(DEV), stok, pairs, npairs, pool, 0, N * K // 4, slots, ref2, N, K, NT, miss)
        assert rel(out, ref2) < 1e-5


@pytest.mark.parametrize("T,N,K,NT", [(1, 128, 128, 8), (5, 384, 512, 8), (70, 256, 1024, 64), (300, 200, 256, 128)])
def test_tc_gemm_fp8(C, T, N, K, NT):
    g = torch.Generator().manual_seed(T + N)
    a = (torch.randn(T, K, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    sa = torch.randint(120, 134, (T, K // 64), generator=g, dtype=torch.uint8)
    w = (torch.randn(N, K, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    sw = torch.randint(118, 130, ((N + 127) // 128, K // 128), generator=g, dtype=torch.uint8)
    out = torch.empty(T, N, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.tc_gemm_fp8(a.to(DEV), sa.to(DEV), w.to(DEV), sw.to(DEV), out, None, NT, st)
    torch.cuda.synchronize()
    A = fp8.dequant_act_fp8(a.view(torch.float8_e4m3fn), sa).double()
    Wd = w.view(torch.float8_e4m3fn).double() * torch.exp2(sw.double() - 127).repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)
    assert int(st) == 0
    assert rel(out.cpu(), A @ Wd.t()) < 1e-4
    res = torch.randn(T, N, generator=g).to(torch.bfloat16).to(DEV)
    outb = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    C.tc_gemm_fp8(a.to(DEV), sa.to(DEV), w.to(DEV), sw.to(DEV), outb, res, NT, st)
    assert rel(outb.cpu().float(), (A @ Wd.t()).float() + res.cpu().float()) < 1e-2


@pytest.mark.parametrize("T,k,E,N,K,NT", [(1, 8, 16, 128, 256, 8), (3, 8, 32, 256, 1536, 8), (20, 4, 8, 384, 512, 16),
                                          (40, 8, 16, 128, 4096, 16), (300, 8, 16, 256, 512, 128)])
def test_ws_moe_w2_padded(C, T, k, E, N, K, NT):
    g = torch.Generator().manual_seed(T * 11 + N)
    codes = torch.randint(0, 4, (E, N, K), generator=g, dtype=torch.uint8)
    sc = torch.randint(118, 132, (E, N, K // 32), generator=g, dtype=torch.uint8)
    pool = torch.stack([torch.cat([planes.pack_codes(codes[e]), planes.pack_scales(sc[e])]) for e in range(E)]).to(DEV)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int().to(DEV)
    R = T * k
    P = R // NT + min(E, R)
    Rp = P * NT
    rank = torch.empty(R, dtype=torch.int32, device=DEV)
    stok = torch.empty(Rp, dtype=torch.int32, device=DEV)
    posof = torch.empty(R, dtype=torch.int32, device=DEV)
    pairs = torch.empty(P, 4, dtype=torch.int32, device=DEV)
    npairs = torch.zeros(1, dtype=torch.int32, device=DEV); nrows = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    C.build_pairs_padded(ids, E, NT, rank, stok, posof, pairs, npairs, nrows, st)
    assert int(nrows) % NT == 0 and int(nrows) <= Rp
    pr = pairs[: int(npairs)].cpu()
    assert (pr[:, 1] % NT == 0).all()
    x = torch.randn(T, K, generator=g)
    q, s = fp8.quant_act_fp8(x)
    qw2 = fp8.to_w2_layout(q.view(torch.uint8)).to(DEV)
    aq = torch.empty(Rp, K, dtype=torch.uint8, device=DEV); as_ = torch.empty(Rp, K // 64, dtype=torch.uint8, device=DEV)
    C.gather_rows(qw2, s.to(DEV), stok, nrows, aq, as_)
    out = torch.full((Rp, N), float("nan"), device=DEV)
    slots = torch.arange(E, dtype=torch.int32, device=DEV)
    slots[int(ids[0, 0])] = -1           # one missing expert -> zero rows + miss count
    miss = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):
        C.ws_moe_w2(aq, as_, pairs, npairs, pool, 0, N * K // 4, slots, out, N, K, NT, miss, st, None)
    torch.cuda.synchronize()
    assert int(st) == 0 and int(miss) >= 1
    A = fp8.dequant_act_fp8(q, s).double()
    po = posof.cpu().long()
    ids_c = ids.cpu()
    for tt in range(T):
        for j in range(k):
            e = int(ids_c[tt, j])
            got = out[po[tt * k + j]].cpu()
            if e == int(ids_c[0, 0]):
                assert (got == 0).all()
                continue
            W = codebook.dequant_codes(codes[e], sc[e]).double()
            assert rel(got, A[tt] @ W.t()) < 1e-4, (tt, j)


@pytest.mark.parametrize("T,N,K", [(1, 128, 128), (130, 384, 512), (300, 200, 1024), (256, 4096, 4096),
                                   (96, 2112, 4096), (96, 4096, 11008)])
def test_ws_gemm_fp8(C, T, N, K):
    g = torch.Generator().manual_seed(T + N + K)
    Tp = (T + 127) // 128 * 128
    a = torch.zeros(Tp, K, dtype=torch.uint8)
    a[:T] = (torch.randn(T, K, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    sap = torch.full((Tp, K // 64), 127, dtype=torch.uint8)
    sap[:T] = torch.randint(120, 134, (T, K // 64), generator=g, dtype=torch.uint8)
    sa = sap[:T]
    w = (torch.randn(N, K, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    sw = torch.randint(118, 130, ((N + 127) // 128, K // 128), generator=g, dtype=torch.uint8)
    out = torch.empty(T, N, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ad = a.to(DEV)
    C.ws_gemm_fp8(ad, sap.to(DEV), w.to(DEV), sw.to(DEV), out, None, T, st)
    torch.cuda.synchronize()
    A = fp8.dequant_act_fp8(a[:T].view(torch.float8_e4m3fn), sa).double()
    Wd = w.view(torch.float8_e4m3fn).double() * torch.exp2(sw.double() - 127).repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)
    assert int(st) == 0
    assert rel(out.cpu(), A @ Wd.t()) < 1e-4

"""Golden tests of the expert formats (CPU)."""
import pytest
import torch

from vllm_moet_b200.formats import codebook, fp8, kv_nvfp4, planes


def test_nibble_to_code_table():
    # +0,.5,1,1.5,2 -> +1 ; 3,4,6 -> +4 ; negatives mirror
    assert codebook.NIBBLE_TO_CODE.tolist() == [2, 2, 2, 2, 2, 3, 3, 3, 1, 1, 1, 1, 1, 0, 0, 0]
    # code -> level -> nibble of that level
    vals = codebook.E2M1_VALUES[codebook.CODE_TO_NIBBLE.long()].tolist()
    assert vals == [-4.0, -1.0, 1.0, 4.0]
    lut = codebook.E4M3_LUT_WORD
    got = [torch.tensor([(lut >> (8 * i)) & 0xFF], dtype=torch.uint8).view(torch.float8_e4m3fn).float().item()
           for i in range(4)]
    assert got == [-4.0, -1.0, 1.0, 4.0]


def test_fragment_major_layout_positions():
    N, K = 32, 128
    codes = torch.randint(0, 4, (N, K), dtype=torch.uint8)
    p = planes.pack_codes(codes)
    assert p.numel() == N * K // 4
    # lane (g,t) of block (nb, kb): byte (tile, k32, half) holds k = kb*64 + k32*32 + half*16 + 4t + j
    nb, kb, g, t, tile, k32, half = 1, 1, 5, 2, 1, 0, 1
    byte = p[(((nb * (K // 64) + kb) * 8 + g) * 4 + t) * 8 + tile * 4 + k32 * 2 + half].item()
    row = nb * 16 + tile * 8 + g
    for j in range(4):
        k = kb * 64 + k32 * 32 + half * 16 + 4 * t + j
        assert (byte >> (2 * j)) & 3 == codes[row, k].item()
    assert torch.equal(planes.unpack_codes(p, N, K), codes)


def test_scale_plane_layout():
    N, K = 32, 128
    s = torch.randint(0, 255, (N, K // 32), dtype=torch.uint8)
    p = planes.pack_scales(s)
    nb, ks, r = 1, 3, 9
    assert p[(nb * (K // 32) + ks) * 16 + r].item() == s[nb * 16 + r, ks].item()
    assert torch.equal(planes.unpack_scales(p, N, K), s)


def test_fp4_roundtrip():
    n = torch.randint(0, 16, (48, 192), dtype=torch.uint8)
    assert torch.equal(planes.unpack_fp4(planes.pack_fp4(n), 48, 192), n)


def test_quintal_exact_for_all_nibbles():
    n = torch.arange(16, dtype=torch.uint8).repeat(16 * 64 // 16).view(16, 64)
    n = n[torch.randperm(16)][:, torch.randperm(64)]
    q = planes.pack_quintal(n)
    assert q.numel() == planes.quintal_plane_bytes(16, 64)
    d = planes.unpack_quintal_digits(q, 16, 64)
    rec = planes.quintal_reconstruct(codebook.nibbles_to_codes(n), d)
    assert torch.equal(rec, n)
    x = torch.arange(1024)
    assert torch.equal(planes.div5_magic(x), x // 5)


def test_requant_midpoints_and_scales():
    # block of 32 with amax 6 -> exponent 0; |u| == 2.5 snaps to 2 (small class, +-1)
    w = torch.zeros(16, 32, dtype=torch.float64)
    w[:, 0] = 6.0
    w[:, 1] = 2.5
    w[:, 2] = -3.5
    w[:, 3] = 0.2
    codes, sc, nib = codebook.f64_to_codes_scales(w, mode="sign", want_nibbles=True)
    assert int(sc[0, 0]) == 127
    assert codes[0, :4].tolist() == [3, 2, 0, 2]
    assert nib[0, 1].item() == 4 and nib[0, 2].item() == (5 | 8)


def test_zero_sign_balancing_auto():
    w = torch.zeros(16, 64, dtype=torch.float64)
    w[:, ::2] = 1.0  # positive zeros only at odd k
    codes, _, _ = codebook.f64_to_codes_scales(w, mode="auto")
    zk = codes[:, 1::2]
    # one-signed zeros -> alternate by k parity: odd k -> negative (-1 -> code 1)
    assert (zk == 1).all()
    codes_s, _, _ = codebook.f64_to_codes_scales(w, mode="sign")
    assert (codes_s[:, 1::2] == 2).all()


def test_fp8_block_rectangular_matches_direct():
    weight = torch.linspace(-2, 2, 64 * 128, dtype=torch.float32).reshape(64, 128).to(torch.float8_e4m3fn)
    scales = torch.tensor([[0.5, 1.0], [2.0, 4.0]])
    got = codebook.fp8_block_to_codes_scales(weight, scales, block_shape=(32, 64), mode="sign")
    exp = codebook.f64_to_codes_scales(weight.double() * scales.repeat_interleave(32, 0).repeat_interleave(64, 1).double(), mode="sign")
    assert torch.equal(got[0], exp[0]) and torch.equal(got[1], exp[1])
    with pytest.raises(ValueError, match="scale shape"):
        codebook.fp8_block_to_codes_scales(weight, torch.ones(1, 1), block_shape=(32, 64))


def test_nvfp4_pipeline_dequant_error():
    torch.manual_seed(0)
    w = torch.randn(64, 256) * 0.02
    packed, sf, ts = codebook.f32_to_nvfp4(w)
    codes, sc, _ = codebook.nvfp4_to_codes_scales(packed, sf, ts, mode="auto")
    deq = codebook.dequant_codes(codes, sc)
    rel = (deq - w).norm() / w.norm()
    assert rel < 0.6  # 4-level codebook on Gaussian data


def test_ue8m0_exponent_exact():
    a = torch.tensor([448.0, 448.0 * 2, 449.0, 1.0, 0.0, 1e-30])
    e = fp8.ue8m0_exponent(a)
    assert e.tolist()[:4] == [0, 1, 1, -8]
    assert e[4].item() == -127
    # the bound holds
    for v, ee in zip(a.tolist(), e.tolist()):
        if v > 0:
            assert v / 2.0 ** ee <= 448.0


def test_w2_activation_layout_is_permutation():
    perm = fp8.w2_perm32()
    assert sorted(perm.tolist()) == list(range(32))


def test_nvfp4_kv_row_roundtrip():
    torch.manual_seed(0)
    lat, rope = torch.randn(7, 512), torch.randn(7, 64)
    rows = kv_nvfp4.encode(lat, rope)
    assert rows.shape == (7, 352) and rows.dtype == torch.uint8
    l2, r2 = kv_nvfp4.decode(rows)
    assert ((l2 - lat).norm() / lat.norm()) < 0.15
    assert ((r2 - rope).norm() / rope.norm()) < 0.05

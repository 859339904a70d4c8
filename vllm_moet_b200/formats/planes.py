"""Fragment-major expert planes: the in-memory AND on-disk expert format.

A plane stores one expert weight matrix [N, K] (N output rows, K the
contraction).  It is cut into 16-row x 64-k blocks ``(nb, kb)``, in that
order; inside a block each of 32 "lanes" ``(g, t)`` (g = 0..7, t = 0..3)
owns the elements an m16n8k32 MMA A-fragment needs for two k32 steps:

    rows  g (tile 0) and g + 8 (tile 1)
    k     kb*64 + k32*32 + half*16 + 4*t + j    (k32, half in {0,1}, j in 0..3)

Byte order within a lane is (tile, k32, half) -> 8 groups of 4 consecutive
k.  This is the reference layout (P:12015-12039, P:12204-12244,
P:12113-12186, P:12400-12408); a pack row written by either engine can be
copied into a GPU slot and served unchanged.

* 2-bit codes: 4 codes per byte, little-endian -> N*K/4 bytes.
* FP4 (e2m1) nibbles: 2 per byte, low nibble first -> N*K/2 bytes.
* Quintal refinement: per group of 4 the base-5 number of e2m1 magnitude
  indices within the code's class (10 bits), 8 words per lane packed into
  an 80-bit little-endian record; a block stores 32x8 low bytes, then
  32x2 high bytes -> N*K*5/16 bytes.
* UE8M0 scales [N, K/32] -> byte at ``(nb*(K/32) + ks)*16 + r``.
"""
from __future__ import annotations

import torch

from .codebook import NIBBLE_TO_CODE, dequant_codes


def _to_lane_order(x: torch.Tensor) -> torch.Tensor:
    """[N, K] -> [N/16, K/64, 8(g), 4(t), 2(tile), 2(k32), 2(half), 4(j)] (contiguous)."""
    N, K = x.shape
    if N % 16 or K % 64:
        raise ValueError(f"plane dims must be multiples of (16, 64), got {(N, K)}")
    # source axes: nb, tile, g, kb, k32, half, t, j
    v = x.reshape(N // 16, 2, 8, K // 64, 2, 2, 4, 4)
    return v.permute(0, 3, 2, 6, 1, 4, 5, 7).contiguous()


def _from_lane_order(v: torch.Tensor, N: int, K: int) -> torch.Tensor:
    v = v.reshape(N // 16, K // 64, 8, 4, 2, 2, 2, 4)
    return v.permute(0, 4, 2, 1, 5, 6, 3, 7).contiguous().reshape(N, K)


def pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """[N, K] u8 codes 0..3 -> plane [N*K/4] u8."""
    q = _to_lane_order(codes).reshape(-1, 4).to(torch.int32)
    return (q[:, 0] | (q[:, 1] << 2) | (q[:, 2] << 4) | (q[:, 3] << 6)).to(torch.uint8)


def unpack_codes(plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    b = plane.reshape(-1, 1).to(torch.int32)
    q = torch.cat([(b >> s) & 3 for s in (0, 2, 4, 6)], dim=1).to(torch.uint8)
    return _from_lane_order(q, N, K)


def pack_fp4(nibbles: torch.Tensor) -> torch.Tensor:
    """[N, K] u8 e2m1 nibbles -> plane [N*K/2] u8 (low nibble first)."""
    q = _to_lane_order(nibbles).reshape(-1, 2).to(torch.int32)
    return (q[:, 0] | (q[:, 1] << 4)).to(torch.uint8)


def unpack_fp4(plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    b = plane.reshape(-1, 1)
    q = torch.cat([b & 0xF, b >> 4], dim=1)
    return _from_lane_order(q, N, K)


def pack_scales(scales: torch.Tensor) -> torch.Tensor:
    """[N, K/32] u8 -> [N*K/32] u8 with byte (nb, ks, r) at (nb*KS + ks)*16 + r."""
    N, KS = scales.shape
    if N % 16:
        raise ValueError("N must be a multiple of 16")
    return scales.reshape(N // 16, 16, KS).transpose(1, 2).contiguous().reshape(-1)


def unpack_scales(plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    KS = K // 32
    return plane.reshape(N // 16, KS, 16).transpose(1, 2).contiguous().reshape(N, KS)


# ---- quintal (radix-5) split-FP4 refinement --------------------------------

_POW5 = (1, 5, 25, 125)


def quintal_digits(nibbles: torch.Tensor) -> torch.Tensor:
    """e2m1 nibbles -> magnitude index within the base code's class (0..4)."""
    mag = (nibbles & 7).long()
    code = NIBBLE_TO_CODE.to(nibbles.device)[nibbles.long()]
    big = (code == 0) | (code == 3)
    return torch.where(big, mag - 5, mag)


def pack_quintal(nibbles: torch.Tensor) -> torch.Tensor:
    """[N, K] e2m1 nibbles -> quintal plane [N*K*5/16] u8."""
    N, K = nibbles.shape
    d = _to_lane_order(quintal_digits(nibbles)).reshape(-1, 8, 4)
    words = sum(d[..., i] * _POW5[i] for i in range(4))           # [lanes, 8] < 625
    rec = torch.zeros(words.shape[0], dtype=torch.int64, device=nibbles.device)
    hi = torch.zeros_like(rec)
    for w in range(8):                     # 80-bit little-endian record: 64 low + 16 high
        bit = 10 * w
        val = words[:, w].long()
        if bit + 10 <= 64:
            rec |= val << bit
        elif bit >= 64:
            hi |= val << (bit - 64)
        else:                              # straddles bit 64
            lo_bits = 64 - bit
            rec |= (val & ((1 << lo_bits) - 1)) << bit
            hi |= val >> lo_bits
    lo_bytes = torch.stack([(rec >> (8 * i)) & 0xFF for i in range(8)], dim=1)
    hi_bytes = torch.stack([(hi >> (8 * i)) & 0xFF for i in range(2)], dim=1)
    lo_bytes = lo_bytes.to(torch.uint8).reshape(-1, 32 * 8)
    hi_bytes = hi_bytes.to(torch.uint8).reshape(-1, 32 * 2)
    return torch.cat([lo_bytes, hi_bytes], dim=1).reshape(-1)


def unpack_quintal_digits(plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    blk = plane.reshape(-1, 320)
    lo = blk[:, :256].reshape(-1, 8).long()
    hi = blk[:, 256:].reshape(-1, 2).long()
    rec = sum(lo[:, i] << (8 * i) for i in range(8))
    hiv = hi[:, 0] | (hi[:, 1] << 8)
    words = []
    for w in range(8):
        bit = 10 * w
        if bit + 10 <= 64:
            v = (rec >> bit) & 0x3FF
        elif bit >= 64:
            v = (hiv >> (bit - 64)) & 0x3FF
        else:
            lo_bits = 64 - bit
            v = ((rec >> bit) & ((1 << lo_bits) - 1)) | ((hiv << lo_bits) & 0x3FF)
        words.append(v)
    words = torch.stack(words, dim=1)                                   # [lanes, 8]
    digits = torch.stack([(words // p) % 5 for p in _POW5], dim=-1)      # [lanes, 8, 4]
    return _from_lane_order(digits.to(torch.uint8).reshape(-1), N, K)


def quintal_reconstruct(codes: torch.Tensor, digits: torch.Tensor) -> torch.Tensor:
    """Base codes + quintal digits -> exact e2m1 nibbles."""
    big = (codes == 0) | (codes == 3)
    mag = torch.where(big, digits.long() + 5, digits.long())
    neg = codes <= 1
    return (mag | (neg.long() << 3)).to(torch.uint8)


def div5_magic(x: torch.Tensor) -> torch.Tensor:
    """x // 5 via (x * 0x334) >> 12, exact for 0 <= x < 1024 (integer identity)."""
    return (x * 0x334) >> 12


# ---- sizes ------------------------------------------------------------------

def codes_plane_bytes(n: int, k: int) -> int:
    return n * k // 4


def scale_plane_bytes(n: int, k: int) -> int:
    return n * k // 32


def fp4_plane_bytes(n: int, k: int) -> int:
    return n * k // 2


def quintal_plane_bytes(n: int, k: int) -> int:
    if (n * k) % 16:
        raise ValueError("n*k must be a multiple of 16")
    return n * k * 5 // 16


def dequant_plane(codes_plane: torch.Tensor, scale_plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    return dequant_codes(unpack_codes(codes_plane, N, K), unpack_scales(scale_plane, N, K))


# ---------------------------------------------------------------------------
# FP4 delta tier in an 8-bit container ("direct-8" plane).
#
# An MXFP4 weight (e2m1 value x UE8M0 block-32 scale) is exactly representable
# as an e4m3 byte times the same scale, so the delta tier stores e4m3 bytes in
# the order the 2-bit decode would produce A-fragments: per 16-row x 64-k
# block and lane (g, t), 32 bytes = registers A0[0..3] (k32 = 0) then
# A1[0..3] (k32 = 1), each register = tile (row g / g+8) x j-parity (j in
# {0,2} or {1,3}), bytes [half0 j_a, half0 j_b, half1 j_a, half1 j_b].  The
# expert GEMV then loads two 16-byte vectors per chunk and needs no decode;
# activations keep the 2-bit path's "w2 layout".  2x the bytes of a nibble
# plane, which HBM affords for the hot fraction of experts.

def mxfp4_quantize(w: torch.Tensor):
    """[N, K] float -> (e2m1 nibbles [N, K] u8, UE8M0 block-32 scales [N, K/32] u8)."""
    from .codebook import e2m1_round
    N, K = w.shape
    x = w.double().reshape(N, K // 32, 32)
    amax = x.abs().amax(-1)
    # smallest power of two with amax / 2^e <= 6 (e2m1 max)
    e = torch.ceil(torch.log2(torch.where(amax > 0, amax / 6.0, torch.ones_like(amax)))).clamp(-127, 127)
    e = torch.where(amax > 0, e, torch.full_like(e, -127))
    nib = e2m1_round((x / torch.exp2(e)[..., None]).float()).reshape(N, K)
    return nib.to(torch.uint8), (e + 127).to(torch.uint8)


def e2m1_to_e4m3_bytes(nib: torch.Tensor) -> torch.Tensor:
    from .codebook import E2M1_VALUES
    v = E2M1_VALUES.float().to(nib.device)[nib.long()]
    return v.to(torch.float8_e4m3fn).view(torch.uint8)


def pack_direct8(e4m3: torch.Tensor) -> torch.Tensor:
    """[N, K] e4m3 bytes -> direct-8 plane [N*K] u8 (fragment register order)."""
    v = _to_lane_order(e4m3)                      # [nb, kb, g, t, tile, k32, half, j]
    v = v.reshape(*v.shape[:4], 2, 2, 2, 2, 2)    # j -> (j_hi, parity): j = 2*j_hi + parity
    # target per lane: [k32][parity][tile][half][j_hi]
    v = v.permute(0, 1, 2, 3, 5, 8, 4, 6, 7).contiguous()
    return v.reshape(-1)


def unpack_direct8(plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    v = plane.reshape(N // 16, K // 64, 8, 4, 2, 2, 2, 2, 2)     # k32, parity, tile, half, j_hi
    v = v.permute(0, 1, 2, 3, 6, 4, 7, 8, 5).contiguous()        # tile, k32, half, j_hi, parity
    return _from_lane_order(v.reshape(N // 16, K // 64, 8, 4, 2, 2, 2, 4), N, K)


def direct8_plane_bytes(n: int, k: int) -> int:
    return n * k


def dequant_direct8(plane: torch.Tensor, scale_plane: torch.Tensor, N: int, K: int) -> torch.Tensor:
    b = unpack_direct8(plane, N, K).view(torch.float8_e4m3fn).float()
    s = torch.exp2(unpack_scales(scale_plane, N, K).float() - 127.0)
    return (b.view(N, K // 32, 32) * s[..., None]).view(N, K)


# ---- split FP4 (w4q) device decode, restated on the host ------------------------
#
# The expert GEMV's quintal mode builds each lane's MMA A-fragment registers from
# the lane's 8 base-code bytes and its 10-byte quintal record.  This is the same
# integer arithmetic, one lane at a time, so the device decode has an exact oracle:
# the registers must equal the lane's bytes of the direct-8 container of the
# reconstructed e2m1 values.

E4M3_LUT_WORD = 0x4838B8C8                   # code -> e4m3 level {-4, -1, +1, +4}
E2M1_MAG_E4M3 = (0x3C383000, 0x4C484440)     # magnitude index 0..7 -> e4m3 byte {0, .5, 1, 1.5, 2, 3, 4, 6}


def prmt(a: int, b: int, sel: int) -> int:
    """PTX prmt (default mode) on Python ints: output byte i = byte (sel nibble i & 7) of {b:a}."""
    pool = (a & 0xFFFFFFFF) | ((b & 0xFFFFFFFF) << 32)
    out = 0
    for i in range(4):
        s = (sel >> (4 * i)) & 0xF
        byte = (pool >> (8 * (s & 7))) & 0xFF
        if s & 8:                                 # sign-replicate mode (not used by the decode)
            byte = 0xFF if byte & 0x80 else 0x00
        out |= byte << (8 * i)
    return out


def quintal_digit_word(w: int) -> int:
    """10-bit quintal word -> (d0 | d2 << 4) | (d1 | d3 << 4) << 8, digits by the
    multiply-shift divide by 5 ((x * 0x334) >> 12, exact below 1024)."""
    q1 = (w * 0x334) >> 12
    d0 = w - 5 * q1
    q2 = (q1 * 0x334) >> 12
    d1 = q1 - 5 * q2
    q3 = (q2 * 0x334) >> 12
    d2 = q2 - 5 * q3
    d3 = q3
    return (d0 | (d2 << 4)) | ((d1 | (d3 << 4)) << 8)


def quintal_lane_registers(code_bytes: bytes, rec: bytes):
    """One lane: 8 base-code bytes + 10-byte quintal record -> (A0[4], A1[4]) e4m3 words."""
    lo = int.from_bytes(code_bytes[:4], "little")
    hi = int.from_bytes(code_bytes[4:8], "little")
    r = int.from_bytes(rec[:8], "little") | (int.from_bytes(rec[8:10], "little") << 64)
    T = [quintal_digit_word((r >> (10 * b)) & 0x3FF) for b in range(8)]

    def reg(c_sel: int, ga: int, gb: int, odd: bool) -> int:
        base = prmt(E4M3_LUT_WORD, E4M3_LUT_WORD, c_sel)
        dsel = prmt(T[ga], T[gb], 0x0051 if odd else 0x0040) & 0xFFFF
        big = ~(c_sel ^ (c_sel >> 1)) & 0x1111          # code 0 or 3: the {3, 4, 6} class
        mag = prmt(E2M1_MAG_E4M3[0], E2M1_MAG_E4M3[1], dsel + 5 * big)
        return mag | (base & 0x80808080)

    m = 0x3333
    A0 = [reg(lo & m, 0, 1, False), reg(hi & m, 4, 5, False), reg((lo >> 2) & m, 0, 1, True),
          reg((hi >> 2) & m, 4, 5, True)]
    A1 = [reg((lo >> 16) & m, 2, 3, False), reg((hi >> 16) & m, 6, 7, False), reg((lo >> 18) & m, 2, 3, True),
          reg((hi >> 18) & m, 6, 7, True)]
    return A0, A1

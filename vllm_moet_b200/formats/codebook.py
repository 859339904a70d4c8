"""Sign-symmetric 2-bit expert codebook {-4, -1, +1, +4}.

Semantics (reference ``moe_w2_planes.py``, P:12014-12074 and
P:12256-12397):

* Code order is ``{0: -4, 1: -1, 2: +1, 3: +4}``.
* An e2m1 nibble maps to the nearest level by magnitude class: magnitudes
  {0, .5, 1, 1.5, 2} are the small class (+-1) and {3, 4, 6} the big class
  (+-4); the sign bit of the nibble gives the sign (so +0 -> +1, -0 -> -1).
* Block-32 scales along K are UE8M0 bytes (``2**(byte-127)``).  For
  dequantized (f64) weights the exponent is ``round(log2(amax/6))`` clamped
  to [-127, 127]; all-zero blocks get exponent -127.
* Snap to the e2m1 grid uses the midpoints between magnitudes with ties to
  the lower magnitude (|u| == 2.5 -> 2).
* Zero-sign balancing: when >95% of a tensor's exact zeros carry one sign,
  zeros alternate sign by k parity ("auto"); "sign" keeps the sign bit and
  "alt" always alternates.

These functions are the golden CPU/GPU (torch) implementation.  The
load-time CUDA quantizer (``csrc/kernels/quant_pack.cu``) is tested against
them byte for byte.
"""
from __future__ import annotations

import os

import torch

QUANTIZER_ABI = "tsym4-e8m0-fragmajor-a32-v2"
"""Identity tag hashed into persistent packs / planes caches.  It names the
quantizer, scale encoding and plane layout, which are byte-compatible with
the reference's packs (same string as P:12050)."""

LEVELS = (-4.0, -1.0, 1.0, 4.0)

# e2m1 nibble (sign in bit 3) -> code
NIBBLE_TO_CODE = torch.tensor([2, 2, 2, 2, 2, 3, 3, 3, 1, 1, 1, 1, 1, 0, 0, 0], dtype=torch.uint8)
# code -> e2m1 nibble of its level (-4 = 0xE, -1 = 0xA, +1 = 0x2, +4 = 0x6)
CODE_TO_NIBBLE = torch.tensor([0xE, 0xA, 0x2, 0x6], dtype=torch.uint8)
# code -> e4m3 byte of its level, as one little-endian word (byte i = code i)
E4M3_LUT_WORD = 0x4838B8C8

E2M1_MAGS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                            -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float64)
_E2M1_MIDPOINTS = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=torch.float64)

ZERO_MODES = ("auto", "sign", "alt")


def zero_mode() -> str:
    mode = os.getenv("VLLM_MOE_W2_ZERO_MODE", "auto").strip().lower()
    if mode not in ZERO_MODES:
        raise ValueError(f"VLLM_MOE_W2_ZERO_MODE must be one of auto|sign|alt, got {mode!r}")
    return mode


def nibbles_to_codes(nib: torch.Tensor) -> torch.Tensor:
    return NIBBLE_TO_CODE.to(nib.device)[nib.long()]


def split_packed_e2m1(packed: torch.Tensor) -> torch.Tensor:
    """[..., K/2] u8 (low nibble = even k) -> [..., K] u8 nibbles."""
    return torch.stack((packed & 0xF, packed >> 4), dim=-1).flatten(-2)


def mxfp4_to_codes(packed: torch.Tensor) -> torch.Tensor:
    """MXFP4 [..., K/2] u8 -> 2-bit codes [..., K] (scales are kept verbatim)."""
    return nibbles_to_codes(split_packed_e2m1(packed))


def f64_to_codes_scales(w: torch.Tensor, mode: str | None = None, want_nibbles: bool = False):
    """Dequantized weights [N, K] (float64) -> (codes u8 [N,K], ue8m0 u8 [N,K/32], nibbles|None)."""
    if w.dtype != torch.float64:
        raise TypeError("f64_to_codes_scales expects float64 weights (exact midpoint tests)")
    N, K = w.shape
    if K % 32:
        raise ValueError("K must be a multiple of 32")
    mode = zero_mode() if mode is None else mode
    blocks = w.reshape(N, K // 32, 32)
    amax = blocks.abs().amax(dim=2)
    exp = torch.full_like(amax, -127.0)
    nz = amax > 0
    exp[nz] = torch.round(torch.log2(amax[nz] / 6.0 + 1e-30))
    exp.clamp_(-127.0, 127.0)
    scale_bytes = (exp + 127.0).to(torch.uint8)
    unit = (blocks / torch.exp2(exp)[..., None]).reshape(N, K)
    mag_idx = torch.bucketize(unit.abs(), _E2M1_MIDPOINTS.to(w.device)).to(torch.uint8)
    negative = torch.signbit(unit)
    if mode != "sign":
        zeros = unit == 0.0
        n_zero = int(zeros.sum())
        if n_zero:
            n_neg = int((negative & zeros).sum())
            if mode == "alt" or min(n_neg, n_zero - n_neg) < 0.05 * n_zero:
                odd_k = (torch.arange(K, device=w.device) % 2 == 1).expand(N, K)
                negative = torch.where(zeros, odd_k, negative)
    nibbles = mag_idx | (negative.to(torch.uint8) << 3)
    codes = nibbles_to_codes(nibbles)
    return codes, scale_bytes, (nibbles if want_nibbles else None)


def fp8_block_to_codes_scales(w_fp8: torch.Tensor, s_block: torch.Tensor, block_shape=(128, 128),
                              mode: str | None = None, want_nibbles: bool = False):
    """FP8 e4m3 weights with f32 block scales -> 2-bit codes + UE8M0 scales."""
    N, K = w_fp8.shape
    if isinstance(block_shape, int):
        bn = bk = block_shape
    else:
        if len(block_shape) != 2:
            raise ValueError(f"FP8 block shape must have two dimensions, got {block_shape!r}")
        bn, bk = int(block_shape[0]), int(block_shape[1])
    if bn <= 0 or bk <= 0:
        raise ValueError(f"invalid FP8 block shape {(bn, bk)}")
    want = (-(-N // bn), -(-K // bk))
    if tuple(s_block.shape) != want:
        raise ValueError(f"FP8 block scale shape {tuple(s_block.shape)} does not match weight "
                         f"{(N, K)} / block {(bn, bk)} -> {want}")
    s = s_block.double().repeat_interleave(bn, 0)[:N].repeat_interleave(bk, 1)[:, :K]
    return f64_to_codes_scales(w_fp8.double() * s, mode, want_nibbles)


def nvfp4_to_codes_scales(packed: torch.Tensor, s_block: torch.Tensor, s2: torch.Tensor,
                          group: int = 16, mode: str | None = None, want_nibbles: bool = False):
    """NVFP4 (e2m1 + e4m3 block-16 + f32 tensor scale) -> 2-bit codes + UE8M0 scales.

    The UE8M0 block-32 scales absorb the tensor scale, so serving needs no
    extra per-tensor factor."""
    N, K = packed.shape[0], packed.shape[1] * 2
    if tuple(s_block.shape) != (N, K // group):
        raise ValueError(f"NVFP4 scale shape {tuple(s_block.shape)} != {(N, K // group)}")
    vals = E2M1_VALUES.to(packed.device)[split_packed_e2m1(packed).long()]
    vals = vals * s_block.double().repeat_interleave(group, dim=1)
    s2 = s2.double().to(packed.device)
    vals = vals * (s2.reshape(()) if s2.numel() == 1 else s2.reshape(N, 1))
    return f64_to_codes_scales(vals, mode, want_nibbles)


def dequant_codes(codes: torch.Tensor, scale_bytes: torch.Tensor) -> torch.Tensor:
    """codes [N,K] + UE8M0 [N,K/32] -> f32 weights (golden dequant)."""
    lv = torch.tensor(LEVELS, device=codes.device)[codes.long()]
    s = torch.exp2(scale_bytes.float() - 127.0)
    N, K = codes.shape
    return (lv.view(N, K // 32, 32) * s[..., None]).view(N, K)


# ---- BASELINE config-1 variant: fp16 group-32 scale = max|w| / 4 ----------

def f32_to_codes_fp16_amax4(w: torch.Tensor, group: int = 32):
    """[N,K] float -> (codes, fp16 scales [N,K/group]); level = nearest of {-4,-1,1,4}*scale."""
    N, K = w.shape
    wb = w.float().reshape(N, K // group, group)
    scale = (wb.abs().amax(-1) / 4.0).to(torch.float16)
    s = scale.float().clamp_min(torch.finfo(torch.float16).tiny)[..., None]
    u = wb / s
    big = u.abs() > 2.5
    neg = torch.signbit(u)
    codes = torch.where(neg, torch.where(big, 0, 1), torch.where(big, 3, 2)).to(torch.uint8)
    return codes.reshape(N, K), scale


def dequant_codes_fp16(codes: torch.Tensor, scale: torch.Tensor, group: int = 32) -> torch.Tensor:
    N, K = codes.shape
    lv = torch.tensor(LEVELS, device=codes.device)[codes.long()]
    return (lv.view(N, K // group, group) * scale.float()[..., None]).view(N, K)


# ---- e2m1 / NVFP4 helpers ---------------------------------------------------

def f32_to_nvfp4(w: torch.Tensor, tensor_scale: float | None = None, group: int = 16):
    """Float [N, K] -> NVFP4 (packed e2m1 u8 [N,K/2], e4m3 block scales [N,K/16], f32 scalar).

    Round-to-nearest-even onto the e2m1 grid (saturating), block scale =
    amax/6 rounded to e4m3 after dividing by the tensor scale."""
    N, K = w.shape
    w = w.float()
    if tensor_scale is None:
        tensor_scale = float(w.abs().max()) / (6.0 * 448.0) or 1.0
    wb = w.view(N, K // group, group)
    sf = (wb.abs().amax(-1) / 6.0 / tensor_scale).clamp(max=448.0).to(torch.float8_e4m3fn)
    scale = sf.float() * tensor_scale
    inv = torch.where(scale > 0, 1.0 / scale, torch.zeros_like(scale))
    u = wb * inv[..., None]
    nib = e2m1_round(u).view(N, K)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8)
    return packed, sf, torch.tensor(tensor_scale, dtype=torch.float32)


def e2m1_round(u: torch.Tensor) -> torch.Tensor:
    """float -> e2m1 nibble, round-to-nearest-even, saturating at 6."""
    a = u.abs().clamp(max=6.0)
    mags = torch.tensor(E2M1_MAGS, device=u.device, dtype=torch.float32)
    d = (a[..., None] - mags).abs()
    best = d.min(-1, keepdim=True).values
    tie = (d == best)
    # ties to even mantissa: candidate indices with even code (idx & 1 == 0)
    idx = torch.arange(8, device=u.device)
    score = torch.where(tie, (idx % 2) * 1 + 0, torch.full_like(idx, 99).expand_as(tie))
    mag_idx = score.argmin(-1).to(torch.uint8)
    neg = torch.signbit(u)
    return mag_idx | (neg.to(torch.uint8) << 3)

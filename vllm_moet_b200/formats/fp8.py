"""FP8 e4m3 with power-of-two (UE8M0) block scales: the dense-stack format.

Weights: [N, K] e4m3 with one UE8M0 exponent per 128x128 block.
Activations: [T, K] e4m3 with one UE8M0 exponent per (token, 128-k group).

Power-of-two scales make every block an exact MX-style operand for the
tcgen05 ``kind::mxf8f6f4`` block-scaled MMA (scale vector 32, the 128 block
exponent repeated four times) and keep requantisation exact.  The scale is
chosen as the smallest power of two with amax / scale <= 448.
"""
from __future__ import annotations

import math

import torch

E4M3_MAX = 448.0


def ue8m0_exponent(amax: torch.Tensor) -> torch.Tensor:
    """Smallest e with fl32(amax / 448) <= 2**e (int32, clamped to [-127, 127]).

    Computed exactly from the float's exponent/mantissa bits (no log2), the
    same way the CUDA quantisers do, so host and device agree bit for bit.
    All-zero groups get e = -127."""
    r = (amax.float() / E4M3_MAX).contiguous()
    bits = r.view(torch.int32)
    ex = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    e = ex - 127 + (mant != 0).to(torch.int32)
    e = torch.where(ex == 0, torch.full_like(e, -126), e)
    e = torch.where(amax > 0, e, torch.full_like(e, -127))
    return e.clamp(-127, 127).to(torch.int32)


def quant_weight_fp8(w: torch.Tensor, block: int = 128):
    """[N, K] float -> (e4m3 [N, K], ue8m0 bytes [ceil(N/128), ceil(K/128)] u8)."""
    N, K = w.shape
    nb, kb = math.ceil(N / block), math.ceil(K / block)
    wp = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    wp[:N, :K] = w.float()
    blk = wp.view(nb, block, kb, block)
    e = ue8m0_exponent(blk.abs().amax(dim=(1, 3)))
    q = (blk / torch.exp2(e.float())[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX)
    q = q.view(nb * block, kb * block)[:N, :K].to(torch.float8_e4m3fn)
    return q.contiguous(), (e + 127).to(torch.uint8)


def dequant_weight_fp8(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    sc = torch.exp2(s.float() - 127.0)
    sc = sc.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * sc


ACT_GROUP = 64


def w2_perm32() -> torch.Tensor:
    """Position -> logical k inside a 32-block for the expert-GEMV operand
    layout ("w2 layout"): lane t of the MMA reads 8 bytes at 8t holding
    k = [4t, 4t+2, 16+4t, 16+4t+2, 4t+1, 4t+3, 16+4t+1, 16+4t+3], which is the
    order the 2-bit decode produces A-fragment bytes in."""
    out = []
    for t in range(4):
        out += [4 * t, 4 * t + 2, 16 + 4 * t, 16 + 4 * t + 2,
                4 * t + 1, 4 * t + 3, 16 + 4 * t + 1, 16 + 4 * t + 3]
    return torch.tensor(out, dtype=torch.long)


def to_w2_layout(q: torch.Tensor) -> torch.Tensor:
    """Natural [T, K] e4m3 (any byte dtype) -> w2 layout (permute inside 32-blocks)."""
    T, K = q.shape
    perm = w2_perm32().to(q.device)
    return q.view(T, K // 32, 32)[:, :, perm].reshape(T, K)


def quant_act_fp8(x: torch.Tensor, group: int = ACT_GROUP):
    """[T, K] float -> (e4m3 [T, K], ue8m0 bytes [T, K/group])."""
    T, K = x.shape
    xb = x.float().view(T, K // group, group)
    e = ue8m0_exponent(xb.abs().amax(-1))
    q = (xb / torch.exp2(e.float())[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(T, K), (e + 127).to(torch.uint8)


def dequant_act_fp8(q: torch.Tensor, s: torch.Tensor, group: int = ACT_GROUP) -> torch.Tensor:
    T, K = q.shape
    return (q.float().view(T, K // group, group) * torch.exp2(s.float() - 127.0)[..., None]).view(T, K)

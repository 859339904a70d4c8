"""NVFP4 MLA KV-cache row (``nvfp4_ds_mla``): 352 bytes per token.

    [0:256)    512 latent dims as e2m1, even dim in the low nibble
    [256:288)  32 e4m3 block-16 scales; block scale = e4m3 * 2**-6
    [288:352)  64 rope dims as e4m3, scale 1

Encode per 16-dim block: sf = amax / 6; stored byte = e4m3(sf * 64)
(saturating at 448); scale = float(byte) / 64; element nibble =
e2m1_rne(x * (1/scale)) (0 when the scale is 0).  The layout and rounding
rules match the reference's KV writer (P:7-19, P:57-115) so the bytes are
interchangeable.  The sm_100a writer kernel lives in
``csrc/kernels/kv_cache.cu``; this module is its golden CPU encoder.
"""
from __future__ import annotations

import torch

from .codebook import E2M1_VALUES, e2m1_round

ROW_BYTES = 352
LATENT = 512
ROPE = 64
SCALE_OFF = 256
ROPE_OFF = 288
GLOBAL_SCALE = 2.0 ** -6


def encode(latent: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
    """latent [T, 512], rope [T, 64] (any float) -> [T, 352] u8."""
    T = latent.shape[0]
    x = latent.float().view(T, 32, 16)
    sf = x.abs().amax(-1) / 6.0
    sfq = (sf * 64.0).clamp(max=448.0).to(torch.float8_e4m3fn)
    scale = sfq.float() * GLOBAL_SCALE
    inv = torch.where(scale > 0, 1.0 / scale, torch.zeros_like(scale))
    nib = e2m1_round(x * inv[..., None]).view(T, 512)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8)
    r = rope.float().clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    return torch.cat([packed, sfq.view(torch.uint8), r], dim=1)


def decode(rows: torch.Tensor):
    """[T, 352] u8 -> (latent f32 [T, 512], rope f32 [T, 64])."""
    T = rows.shape[0]
    packed = rows[:, :256]
    nib = torch.stack((packed & 0xF, packed >> 4), dim=-1).view(T, 512)
    vals = E2M1_VALUES.float().to(rows.device)[nib.long()].view(T, 32, 16)
    sc = rows[:, SCALE_OFF:ROPE_OFF].contiguous().view(torch.float8_e4m3fn).float() * GLOBAL_SCALE
    lat = (vals * sc[..., None]).view(T, 512)
    rope = rows[:, ROPE_OFF:].contiguous().view(torch.float8_e4m3fn).float()
    return lat, rope

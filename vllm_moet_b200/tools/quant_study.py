"""Offline quantisation study: reconstruction error of expert weight formats.

    python -m vllm_moet_b200.tools.quant_study --rows 1024 --cols 4096 --std 0.02

Compares, on the same random (or heavy-tailed) matrix: NVFP4 (e2m1, e4m3
block-16 scales), MXFP4 (e2m1, UE8M0 block-32: the FP4 delta tier), and the
sign-symmetric 2-bit codebook derived from NVFP4 with each zero-code mode
(the base tier) and, with ``--trellis-L``, the trellis (EXL3-style) base tier at 2 and 3
bits (its bits per weight include the fp16 row / column vectors).  Prints relative Frobenius error and bits per weight
(reference: the offline codebook studies, tools/sweep_nvfp4_codebook.py).
"""
from __future__ import annotations

import argparse

import torch

from ..formats import codebook, planes


def study(w: torch.Tensor, trellis_L: int = 0) -> dict:
    N, K = w.shape
    res = {}
    ts = float(w.abs().max()) / (6.0 * 448.0)
    packed, sf, t2 = codebook.f32_to_nvfp4(w, ts)
    vals = codebook.E2M1_VALUES[codebook.split_packed_e2m1(packed).long()]
    nv = (vals * sf.double().repeat_interleave(16, dim=1) * float(t2)).float()
    res["nvfp4"] = (float((nv - w).norm() / w.norm()), 4.5)
    nib, sc = planes.mxfp4_quantize(w)
    mx = planes.dequant_direct8(planes.pack_direct8(planes.e2m1_to_e4m3_bytes(nib)), planes.pack_scales(sc), N, K)
    res["mxfp4 (delta tier)"] = (float((mx - w).norm() / w.norm()), 4.25)
    for mode in ("sign", "alt", "auto"):
        codes, s, _ = codebook.nvfp4_to_codes_scales(packed, sf, t2, mode=mode)
        d = codebook.dequant_codes(codes, s)
        res[f"2-bit codebook ({mode})"] = (float((d - w).norm() / w.norm()), 2.25)
    if trellis_L:
        from ..formats import trellis
        for bits in (2, 3):
            t = trellis.quantize_linear(w, bits, trellis_L)
            d = trellis.dequant_linear(t, bits, trellis_L)
            res[f"trellis {bits}-bit (L={trellis_L})"] = (float((d - w).norm() / w.norm()),
                                                        8.0 * trellis.linear_bytes(N, K, bits) / (N * K))
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=512)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--std", type=float, default=0.02)
    ap.add_argument("--heavy-tail", action="store_true", help="Student-t (3 dof) weights")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--trellis-L", type=int, default=0, help="also the trellis tier with 2^L states (0: off)")
    a = ap.parse_args(argv)
    g = torch.Generator().manual_seed(a.seed)
    if a.heavy_tail:
        w = torch.distributions.StudentT(3.0).sample((a.rows, a.cols)) * a.std
    else:
        w = torch.randn(a.rows, a.cols, generator=g) * a.std
    for name, (err, bits) in study(w, a.trellis_L).items():
        print(f"{name:28s} rel err {err:.4f}   {bits:.2f} bits/weight")


if __name__ == "__main__":
    main()

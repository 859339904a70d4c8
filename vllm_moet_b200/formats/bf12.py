"""bf12: a lossless ~12-bit container for BF16 weights.

A bf16 word is ``sign | exponent(8) | mantissa(7)``.  Split it as
``hi = sign | exponent[7:1]`` and ``lo = exponent[0] | mantissa``.  Trained
(and N(0, s) random) weights use only a handful of ``hi`` values, so:

* **class plane** -- one nibble per weight: ``sign << 3 | class`` where class
  0..6 indexes the tensor's 7 most frequent exponent-top values and class 7
  means *escape*; two nibbles per byte, even index in the low nibble;
* **LO plane** -- the raw ``lo`` byte of every weight;
* **LUT16** -- 16 bytes: nibble -> ``hi`` (escape entries hold 0);
* **escape scatter** -- (position, hi byte) of every escaped weight.

Decode = ``(LUT16[nibble] << 8 | lo)`` then scatter the escapes; the result
is bit-identical to the input (NaN payloads, infinities and denormals
included).  Size: 12 bits per weight plus 5 bytes per escape -- about 12.05
bits for typical weights.  The decoded tensor feeds the stock BF16 GEMM.
(The reference's bf12 container, patch P:11400-11720, behaviour.)
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class Bf12:
    shape: tuple
    classes: torch.Tensor     # uint8 [ceil(n/2)]
    lo: torch.Tensor          # uint8 [n]
    lut: torch.Tensor         # uint8 [16]
    esc_pos: torch.Tensor     # int64 [m]
    esc_hi: torch.Tensor      # uint8 [m]

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def bits_per_weight(self) -> float:
        nbytes = self.classes.numel() + self.lo.numel() + 16 + self.esc_pos.numel() * 5
        return 8.0 * nbytes / self.numel

    def to(self, device) -> "Bf12":
        return Bf12(self.shape, self.classes.to(device), self.lo.to(device), self.lut.to(device),
                    self.esc_pos.to(device), self.esc_hi.to(device))


def encode(w: torch.Tensor) -> Bf12:
    assert w.dtype == torch.bfloat16
    bits = w.detach().contiguous().view(torch.int16).reshape(-1).cpu().to(torch.int32) & 0xFFFF
    hi = (bits >> 8) & 0xFF                  # sign | exp[7:1]
    lo = (bits & 0xFF).to(torch.uint8)
    sign = hi >> 7
    top = hi & 0x7F
    counts = torch.bincount(top, minlength=128)
    common = torch.argsort(counts, descending=True, stable=True)[:7]
    common = common[counts[common] > 0]
    cls = torch.full((128,), 7, dtype=torch.int32)
    cls[common] = torch.arange(common.numel(), dtype=torch.int32)
    c = cls[top]
    nib = (sign << 3) | c
    lut = torch.zeros(16, dtype=torch.uint8)
    for i, t in enumerate(common.tolist()):
        lut[i] = t
        lut[8 + i] = 0x80 | t
    esc = (c == 7).nonzero().flatten()
    n = nib.numel()
    if n % 2:
        nib = torch.cat([nib, torch.zeros(1, dtype=nib.dtype)])
    packed = (nib[0::2] | (nib[1::2] << 4)).to(torch.uint8)
    return Bf12(tuple(w.shape), packed, lo, lut, esc.to(torch.int64), hi[esc].to(torch.uint8))


def decode(b: Bf12) -> torch.Tensor:
    """Reference decoder (any device)."""
    n = b.numel
    p = b.classes.to(torch.int32)
    nib = torch.stack([p & 0xF, p >> 4], dim=1).reshape(-1)[:n]
    hi = b.lut.to(torch.int32)[nib]
    hi[b.esc_pos] = b.esc_hi.to(torch.int32)
    bits = (hi << 8) | b.lo.to(torch.int32)
    bits = torch.where(bits >= 0x8000, bits - 0x10000, bits).to(torch.int16)
    return bits.view(torch.bfloat16).reshape(b.shape)


class Bf12Linear:
    """y = x W^T with W stored as bf12, decoded into a shared scratch buffer per call."""

    _scratch = {}

    def __init__(self, w: torch.Tensor):
        self.b = encode(w.to(torch.bfloat16)).to(w.device)
        self.shape = tuple(w.shape)

    def decoded(self) -> torch.Tensor:
        dev = self.b.lo.device
        if dev.type == "cuda":
            from ..ops import native
            key = (dev, self.b.numel)
            buf = Bf12Linear._scratch.get(key)
            if buf is None:
                buf = Bf12Linear._scratch[key] = torch.empty(self.b.numel, dtype=torch.bfloat16, device=dev)
            native().bf12_decode(self.b.classes, self.b.lo, self.b.lut, self.b.esc_pos, self.b.esc_hi, buf)
            return buf.view(self.shape)
        return decode(self.b)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.decoded().t()

    def dequant(self) -> torch.Tensor:
        return decode(self.b).float()

    def to(self, device) -> "Bf12Linear":
        out = object.__new__(Bf12Linear)
        out.b, out.shape = self.b.to(device), self.shape
        return out


# Linear attributes of a decoder layer that may hold a dense BF16 matrix.
_LAYER_LINEARS = ("qkv_a", "q_b", "kv_b", "o", "gate_up", "down", "shared_gate_up", "shared_down",
                  "idx_wq", "idx_wk", "idx_ww")


def convert_model(mw, min_numel: int = 1 << 20, exclude=(), verify: bool = True) -> dict:
    """Re-pack every dense linear whose weight is exactly BF16 (a ``FloatLinear`` loaded from a
    BF16 checkpoint) and has at least ``min_numel`` elements into a :class:`Bf12Linear`, after
    load and before any graph capture.  Names containing an ``exclude`` substring stay as they
    are (``layers.3.o``, ``mtp.layer.kv_b``, ...); with ``verify`` each container is decoded
    and compared bit for bit with the live matrix, and a mismatch keeps the original.
    FP8 / NVFP4 linears and the 2-bit experts are not BF16 and are never touched (the GPU
    runner's dense layers are FP8, so there this converts nothing).  The reference's
    behaviour: ``convert_model`` after load, opt-in (patch P:3997-4057).
    -> {"converted", "skipped_verify", "bytes_before", "bytes_after"}."""
    from ..models.weights import FloatLinear
    stats = {"converted": 0, "skipped_verify": 0, "bytes_before": 0, "bytes_after": 0}
    layers = [(f"layers.{i}", lw) for i, lw in enumerate(mw.layers)]
    if getattr(mw, "mtp", None) is not None and getattr(mw.mtp, "layer", None) is not None:
        layers.append(("mtp.layer", mw.mtp.layer))
    for prefix, lw in layers:
        for attr in _LAYER_LINEARS:
            lin = getattr(lw, attr, None)
            name = f"{prefix}.{attr}"
            if not isinstance(lin, FloatLinear) or lin.w.dim() != 2 or lin.w.numel() < min_numel:
                continue
            if any(x in name for x in exclude):
                continue
            w = lin.w
            wb = w.to(torch.bfloat16)
            if not torch.equal(wb.float(), w.float()):
                continue                    # not a BF16 matrix (e.g. fp32 random init)
            new = Bf12Linear(wb)
            if verify and not torch.equal(decode(new.b.to("cpu")).view(torch.int16), wb.cpu().view(torch.int16)):
                stats["skipped_verify"] += 1
                continue
            stats["converted"] += 1
            stats["bytes_before"] += wb.numel() * 2
            b = new.b
            stats["bytes_after"] += b.classes.numel() + b.lo.numel() + 16 + b.esc_pos.numel() * 9
            setattr(lw, attr, new)
    return stats

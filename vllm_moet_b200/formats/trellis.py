"""Trellis-coded expert weights: the format of the EXL3-style base tier.

The reference serves an experimental base tier from EXL3 packs through exllamav3's
kernels (``moe_w2_exl3.py``, patch/vllm-moet-v0.24.0.patch:10374-11205; pack naming
``exl3-l{li:02d}.safetensors``, keys ``e{e}.{w1|w3|w2}.k{K}.{trellis|suh|svh}``, trellis
bytes ``(k/16)(n/16)·16K`` words, fp16 ``suh`` / ``svh`` vectors: P:10411-10433,
P:10660-10668).  This module is our own restatement of that family of formats from the
published method it is based on -- QTIP (Tseng, Sun, Hou, De Sa, "QTIP: Quantization
with Trellises and Incoherence Processing", NeurIPS 2024): incoherence processing by
random-sign Hadamard transforms, then a tail-biting bitshift trellis whose states map to
pseudo-Gaussian values through a computed codebook.  The names, key layout and byte
sizes follow the reference's packs; the bit order inside a tile is ours (written by our
own pack builder), so packs written by exllamav3 are not read (``FORMAT`` is checked).

A linear map ``y = x W^T`` (``W`` [N_out, K_in], torch convention) is stored as

    W^T = diag(su) · Hk · Q · Hn · diag(sv)

with ``Hk`` / ``Hn`` block-diagonal orthonormal Sylvester-Hadamard matrices (block
``hadamard_block(n)`` = the largest power of two <= 128 dividing ``n``), ``su`` [K_in] and
``sv`` [N_out] fp16 vectors (a random sign times a row / column RMS), and ``Q`` [K_in,
N_out] trellis-coded at ``K`` bits per weight.  The serving order is therefore
``x' = Hk(x ⊙ su)``, ``z = x' Q``, ``y = Hn(z) ⊙ sv``.

``Q`` is cut into 16 x 16 tiles in (k-tile, n-tile) row-major order; a tile's 256 values
(row-major inside the tile, index ``i = kk·16 + nn``) are one trellis walk of 256·K bits,
stored as 16·K 16-bit words, bit 0 of the stream being the most significant bit of word
0.  Value ``i`` is ``cb(state_i) / rms(cb)`` where ``state_i`` is the L-bit window of the
stream that ENDS at bit ``(i + 1)·K`` (MSB first), read cyclically: the walk is
tail-biting, so the first states wrap around to the stream's last bits.

Codebooks (both from the QTIP paper, computed, no table):

* ``3inst``: ``x = a·s + b mod 2^32`` (a = 89226354, b = 64248484), ``m = (x & 0x8FFF8FFF)
  ^ 0x3B603B60``, value = fp16(m low half) + fp16(m high half), summed in fp32.
* ``1mad``: ``x = a·s + b mod 2^32`` (a = 34038481, b = 76625530), value = (sum of the
  four bytes of x - 510) / 147.8.

The values are divided by the codebook's RMS over all 2^L states (``codebook_rms``),
which the kernels receive as an fp32 argument.
"""
from __future__ import annotations

import functools
import math
from typing import Optional

import torch

FORMAT = "moet-trellis-v1"
TILE = 16
CODEBOOKS = ("3inst", "1mad")
_M32 = 0xFFFFFFFF


def hadamard_block(n: int) -> int:
    """Largest power of two <= 128 that divides n."""
    b = 1
    while b < 128 and n % (2 * b) == 0:
        b *= 2
    return b


def fwht(x: torch.Tensor, block: Optional[int] = None) -> torch.Tensor:
    """Orthonormal block Walsh-Hadamard transform (Sylvester order) over the last dim.
    Symmetric and its own inverse."""
    n = x.shape[-1]
    b = block or hadamard_block(n)
    assert n % b == 0 and b & (b - 1) == 0
    y = x.reshape(*x.shape[:-1], n // b, b).clone()
    h = 1
    while h < b:
        y = y.view(*y.shape[:-1], b // (2 * h), 2, h)
        a, c = y[..., 0, :], y[..., 1, :]
        y = torch.stack((a + c, a - c), dim=-2)
        y = y.view(*y.shape[:-3], b)
        h *= 2
    return (y * (1.0 / math.sqrt(b))).reshape(x.shape)


def codebook_raw(states: torch.Tensor, codebook: str = "3inst") -> torch.Tensor:
    """Un-normalised codebook values (fp32) of integer trellis states."""
    s = states.to(torch.int64)
    if codebook == "3inst":
        x = (s * 89226354 + 64248484) & _M32
        m = (x & 0x8FFF8FFF) ^ 0x3B603B60
        lo = (m & 0xFFFF).to(torch.int32).to(torch.int16)          # wraps to the fp16 bit pattern
        hi = ((m >> 16) & 0xFFFF).to(torch.int32).to(torch.int16)
        return lo.view(torch.float16).float() + hi.view(torch.float16).float()
    if codebook == "1mad":
        x = (s * 34038481 + 76625530) & _M32
        tot = (x & 0xFF) + ((x >> 8) & 0xFF) + ((x >> 16) & 0xFF) + ((x >> 24) & 0xFF)
        return ((tot - 510).double() / 147.8).float()
    raise ValueError(f"unknown trellis codebook {codebook!r}; expected one of {CODEBOOKS}")


@functools.lru_cache(maxsize=None)
def codebook_rms(L: int, codebook: str = "3inst") -> float:
    """RMS of the codebook over all 2^L states, rounded to fp32."""
    v = codebook_raw(torch.arange(1 << L), codebook).double()
    return float(torch.tensor(float(v.pow(2).mean().sqrt()), dtype=torch.float32))


@functools.lru_cache(maxsize=None)
def codebook_table(L: int, codebook: str = "3inst") -> torch.Tensor:
    """Normalised values of all 2^L states, exactly as the kernels compute them
    (fp32 raw value times the fp32 reciprocal of the RMS)."""
    inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(codebook_rms(L, codebook), dtype=torch.float32)
    return codebook_raw(torch.arange(1 << L), codebook) * inv


def words_per_tile(K: int) -> int:
    return TILE * K


def _check(K: int, L: int):
    if not 1 <= K <= 4:
        raise ValueError(f"trellis bits per weight must be 1..4, got {K}")
    if not K < L <= 16:
        raise ValueError(f"trellis state bits must satisfy K < L <= 16, got L={L}, K={K}")


# ---------------------------------------------------------------- bit streams

def codes_to_words(codes: torch.Tensor, K: int) -> torch.Tensor:
    """codes [B, 256] (K-bit ints) -> words [B, 16K] int16 (MSB-first stream)."""
    B = codes.shape[0]
    dev = codes.device
    bits = ((codes.to(torch.int64)[..., None] >> torch.arange(K - 1, -1, -1, device=dev)) & 1).reshape(B, 256 * K)
    w = (bits.view(B, 16 * K, 16) << torch.arange(15, -1, -1, device=dev)).sum(-1)
    return w.to(torch.int32).to(torch.int16)


def words_to_bits(words: torch.Tensor) -> torch.Tensor:
    """words [..., n] int16 -> bits [..., 16 n] (0/1 int64), MSB of word 0 first."""
    w = words.to(torch.int64) & 0xFFFF
    sh = torch.arange(15, -1, -1, device=words.device)
    return ((w[..., None] >> sh) & 1).reshape(*words.shape[:-1], words.shape[-1] * 16)


@functools.lru_cache(maxsize=None)
def _window_index(K: int, L: int) -> torch.Tensor:
    N = 256 * K
    i = torch.arange(256)[:, None]
    j = torch.arange(L)[None, :]
    return ((i + 1) * K - L + j) % N                          # [256, L] bit positions, MSB first


def tile_states(words: torch.Tensor, K: int, L: int) -> torch.Tensor:
    """words [..., 16K] -> the 256 trellis states of each tile [..., 256]."""
    bits = words_to_bits(words)
    win = bits[..., _window_index(K, L).to(words.device)]     # [..., 256, L]
    return (win << torch.arange(L - 1, -1, -1, device=words.device)).sum(-1)


def decode_tiles(words: torch.Tensor, K: int, L: int, codebook: str = "3inst") -> torch.Tensor:
    """words [..., 16K] -> normalised tile values [..., 256] fp32."""
    return codebook_table(L, codebook).to(words.device)[tile_states(words, K, L)]


# ---------------------------------------------------------------- Viterbi encoder

def _viterbi(target: torch.Tensor, cbv: torch.Tensor, K: int, L: int,
             wrap: Optional[torch.Tensor]) -> tuple:
    """Minimum-squared-error state path through the bitshift trellis.

    target [B, 256] fp32, cbv [2^L] codebook values.  ``wrap`` [B] constrains the walk to be
    tail-biting: the first state's high L-K bits and the last state's low L-K bits both
    equal it.  Returns (states [B, 256] int64, cost [B])."""
    B, n = target.shape
    S, C = 1 << L, 1 << K
    Q = S // C
    s_all = torch.arange(S, device=target.device)
    inf = torch.tensor(float("inf"), device=target.device)
    D = (target[:, 0, None] - cbv[None, :]) ** 2
    if wrap is not None:
        D = torch.where((s_all[None, :] >> K) == wrap[:, None], D, inf)
    back = torch.empty(n, B, Q, dtype=torch.uint8, device=target.device)
    for i in range(1, n):
        # predecessors of s: p = (s >> K) + h·Q for h in [0, 2^K)
        m, h = D.view(B, C, Q).min(dim=1)
        back[i] = h.to(torch.uint8)
        D = m.repeat_interleave(C, dim=1) + (target[:, i, None] - cbv[None, :]) ** 2
    if wrap is not None:
        D = torch.where((s_all[None, :] & (Q - 1)) == wrap[:, None], D, inf)
    cost, s = D.min(dim=1)
    states = torch.empty(B, n, dtype=torch.int64, device=target.device)
    states[:, n - 1] = s
    rows = torch.arange(B, device=target.device)
    for i in range(n - 1, 0, -1):
        q = s >> K
        s = q + back[i][rows, q].to(torch.int64) * Q
        states[:, i - 1] = s
    return states, cost


def encode_tiles(values: torch.Tensor, K: int, L: int, codebook: str = "3inst",
                 chunk: Optional[int] = None) -> torch.Tensor:
    """values [B, 256] (unit-RMS targets) -> words [B, 16K] int16.  Two Viterbi passes per
    tile: a free one, then one constrained to be tail-biting on the first pass's last
    L-K bits (every such walk is a valid cyclic stream)."""
    _check(K, L)
    B = values.shape[0]
    dev = values.device
    cbv = codebook_table(L, codebook).to(dev)
    if chunk is None:   # bound the back-pointer store (256 x chunk x 2^(L-K) bytes) to ~256 MiB
        chunk = max(1, min(B, (256 << 20) // (256 << (L - K))))
    out = torch.empty(B, 16 * K, dtype=torch.int16, device=dev)
    mask = (1 << (L - K)) - 1
    for b0 in range(0, B, chunk):
        t = values[b0:b0 + chunk].float()
        st, _ = _viterbi(t, cbv, K, L, None)
        st, _ = _viterbi(t, cbv, K, L, st[:, -1] & mask)
        out[b0:b0 + chunk] = codes_to_words(st & ((1 << K) - 1), K)
    return out


# ---------------------------------------------------------------- matrices

def _tiles_of(Q: torch.Tensor) -> torch.Tensor:
    """Q [Kin, N] -> tile values [Kin/16, N/16, 256] (row-major inside a tile)."""
    Kin, N = Q.shape
    return Q.reshape(Kin // TILE, TILE, N // TILE, TILE).permute(0, 2, 1, 3).reshape(Kin // TILE, N // TILE, 256)


def _untile(t: torch.Tensor) -> torch.Tensor:
    kt, nt, _ = t.shape
    return t.reshape(kt, nt, TILE, TILE).permute(0, 2, 1, 3).reshape(kt * TILE, nt * TILE)


def _signs(n: int, gen: torch.Generator) -> torch.Tensor:
    return torch.randint(0, 2, (n,), generator=gen).double() * 2 - 1


def quantize_linear(w: torch.Tensor, K: int, L: int = 16, codebook: str = "3inst", seed: int = 0,
                    device=None) -> dict:
    """Trellis-code a torch-convention weight ``w`` [N_out, K_in].

    Returns ``{"trellis": int16 [K_in/16, N_out/16, 16K], "suh": fp16 [K_in], "svh": fp16
    [N_out]}``.  ``device`` runs the Viterbi search there (it is the costly part: 2·256 steps
    over 2^L states per tile)."""
    _check(K, L)
    N, Kin = w.shape
    if Kin % TILE or N % TILE:
        raise ValueError(f"trellis tiles need both dims divisible by {TILE}, got {tuple(w.shape)}")
    gen = torch.Generator().manual_seed(seed)
    dev = device if device is not None else w.device
    wt = w.detach().double().cpu().t()                             # [Kin, N]
    col = wt.pow(2).mean(0).sqrt()
    sv = (_signs(N, gen) * torch.where(col > 0, col, torch.ones_like(col))).half()
    wt = wt / sv.double()[None, :]
    row = wt.pow(2).mean(1).sqrt()
    su = (_signs(Kin, gen) * torch.where(row > 0, row, torch.ones_like(row))).half()
    wt = wt / su.double()[:, None]
    Qm = fwht(fwht(wt.t()).t())                                    # Hk · wt · Hn
    tiles = _tiles_of(Qm.float())
    words = encode_tiles(tiles.reshape(-1, 256).to(dev), K, L, codebook).cpu()
    return {"trellis": words.reshape(Kin // TILE, N // TILE, 16 * K), "suh": su, "svh": sv}


def decode_q(trellis: torch.Tensor, K: int, L: int, codebook: str = "3inst") -> torch.Tensor:
    """trellis [Kt, Nt, 16K] -> Q [Kt·16, Nt·16] fp32."""
    return _untile(decode_tiles(trellis, K, L, codebook))


def dequant_linear(t: dict, K: int, L: int, codebook: str = "3inst") -> torch.Tensor:
    """Inverse of quantize_linear up to the trellis error: W [N_out, K_in] fp32."""
    Qm = decode_q(t["trellis"], K, L, codebook).double()
    wt = fwht(fwht(Qm.t()).t())                                    # Hk · Q · Hn
    wt = t["suh"].double()[:, None] * wt * t["svh"].double()[None, :]
    return wt.t().float()


def apply_linear(x: torch.Tensor, t: dict, K: int, L: int, codebook: str = "3inst",
                 q: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x W^T through the transforms (what the kernels compute), fp32.  ``q`` is the
    decoded Q when the caller keeps it."""
    Qm = q if q is not None else decode_q(t["trellis"], K, L, codebook)
    xr = fwht(x.float() * t["suh"].float())
    return fwht(xr @ Qm) * t["svh"].float()


def linear_bytes(n_out: int, k_in: int, K: int) -> int:
    """Bytes of one trellis-coded linear: trellis + suh + svh."""
    return (k_in // TILE) * (n_out // TILE) * 16 * K * 2 + 2 * k_in + 2 * n_out

"""Offline codebook studies for the 2-bit expert format: K-level codebook search over
the e2m1 grid, the sign-asymmetry sweep, and a K-level repack of FP4 checkpoints.

    # sign-symmetric vs optimal 4-level codebook on synthetic or checkpoint experts
    python -m vllm_moet_b200.tools.codebook_search sweep [--checkpoint DIR --limit 24]
    # degrade a checkpoint's FP4 routed experts to K levels (headers and offsets kept)
    python -m vllm_moet_b200.tools.codebook_search repack --src DIR --dst DIR --levels 4
    # K = 16 must reproduce every file byte for byte
    python -m vllm_moet_b200.tools.codebook_search gate --src DIR

Model (the behaviour of the reference's offline tools, tools/repack_expert_bits.py,
tools/sweep_nvfp4_codebook.py):

* A tensor's values in unit space are e2m1 codes: 16 codes, 15 distinct values (+0 and
  -0 coincide).  Its code histogram is the weight of each value.
* ``optimal_levels`` picks K of the representable values minimising the weighted
  squared error of the histogram when every value moves to a chosen level.  In one
  dimension the optimal assignment sends each level a contiguous run of the sorted
  values, so the search is a dynamic programme over (runs so far, last value covered);
  a run's cost is its best representable centre inside the run.  Ties keep the first
  (lowest) candidate unless ``tie="last"``.
* ``symmetric_levels`` is the best set {-b, -a, a, b} (0 < a < b on the grid), each
  code moving to the nearest level (equal distance: the level with the code's sign, so
  +0 and -0 go to +a and -a as the served quantizer maps them).
* The sweep reports, per tensor, the weighted mean signed error (bias) and the
  relative RMS error of both codebooks: an asymmetric optimum that drops one sign's
  tail gives a one-signed bias that compounds over layers, which is why the served
  codebook is sign-symmetric {-4, -1, 1, 4}.
* ``repack`` remaps every FP4 code of the matched expert tensors to the original e2m1
  code of its nearest chosen level (the sign bit kept when the level is zero) and
  copies all other bytes unchanged, so file sizes, headers and offsets stay identical.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import shutil
import struct
import sys
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..formats import codebook

# value of e2m1 code c (sign in bit 3): magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6
CODE_VALUES: List[float] = [float(v) for v in codebook.E2M1_VALUES.tolist()]
GRID: List[float] = sorted(set(v + 0.0 for v in CODE_VALUES))          # 15 distinct values

EXPERT_PATTERNS = (
    r"^(model\.)?layers\.\d+\.ffn\.experts\.\d+\.(w1|w2|w3)\.weight$",
    r"^(model\.)?(language_model\.model\.)?layers\.\d+\.mlp\.experts\.\d+\.(gate|up|down)_proj\.weight$",
)


# ---------------------------------------------------------------------- codebook search
def value_histogram(hist16: Sequence[float]) -> Dict[float, float]:
    """Code histogram (16 bins) -> weight per distinct value (+0 and -0 merged)."""
    out: Dict[float, float] = {}
    for c, w in enumerate(hist16):
        if w:
            v = CODE_VALUES[c] + 0.0
            out[v] = out.get(v, 0.0) + float(w)
    return out


def optimal_levels(hist16: Sequence[float], K: int, tie: str = "first") -> Tuple[List[float], float]:
    """-> (sorted levels, weighted squared error): the best K representable levels for the
    histogram (exact; see the module docstring)."""
    vh = value_histogram(hist16)
    pts = sorted(vh)
    m = len(pts)
    if m == 0:
        return [0.0], 0.0
    K = max(1, min(K, m))
    w = [vh[v] for v in pts]

    def run_cost(a: int, b: int) -> Tuple[float, float]:
        # best representable centre of pts[a..b] (inclusive)
        best, centre = None, None
        cands = [g for g in GRID if pts[a] <= g <= pts[b]]
        for c in cands:
            e = sum(w[i] * (pts[i] - c) ** 2 for i in range(a, b + 1))
            if best is None or e < best - 1e-15 or (tie == "last" and abs(e - best) <= 1e-15):
                best, centre = e, c
        return best, centre

    cost = {(a, b): run_cost(a, b) for a in range(m) for b in range(a, m)}
    INF = float("inf")
    # f[k][j]: best error covering pts[0..j] with k runs; arg for reconstruction
    f = [[INF] * m for _ in range(K + 1)]
    arg = [[-1] * m for _ in range(K + 1)]
    for j in range(m):
        f[1][j] = cost[(0, j)][0]
    for k in range(2, K + 1):
        for j in range(k - 1, m):
            for i in range(k - 2, j):          # previous run ends at i
                e = f[k - 1][i] + cost[(i + 1, j)][0]
                if e < f[k][j] - 1e-15 or (tie == "last" and abs(e - f[k][j]) <= 1e-15):
                    f[k][j], arg[k][j] = e, i
    levels, j = [], m - 1
    for k in range(K, 0, -1):
        i = arg[k][j] if k > 1 else -1
        levels.append(cost[(i + 1, j)][1])
        j = i
    return sorted(levels), f[K][m - 1]


def level_of(c: int, levels: Sequence[float]) -> float:
    """The level code c moves to: the nearest one; at equal distance the one with the
    code's sign (so +0 and -0 split between +a and -a), then the smaller magnitude."""
    v, neg = CODE_VALUES[c] + 0.0, bool(c & 0x8)
    return min(levels, key=lambda L: (abs(v - L), 0 if (L < 0) == neg or L == 0 else 1, abs(L), L))


def symmetric_levels(hist16: Sequence[float]) -> Tuple[List[float], float]:
    """-> (levels {-b, -a, a, b}, weighted squared error): the best sign-symmetric set."""
    pos = [g for g in GRID if g > 0]
    best = None
    for ai, a in enumerate(pos):
        for b in pos[ai + 1:]:
            lv = [-b, -a, a, b]
            e = sum(w * (CODE_VALUES[c] - level_of(c, lv)) ** 2 for c, w in enumerate(hist16) if w)
            if best is None or e < best[1] - 1e-15:
                best = (lv, e)
    return best


def error_stats(hist16: Sequence[float], levels: Sequence[float]) -> Tuple[float, float]:
    """-> (weighted mean signed error, relative RMS error) of moving every code to its
    level, relative to the histogram's RMS value."""
    W = float(sum(hist16))
    if W == 0:
        return 0.0, 0.0
    d = [(w, level_of(c, levels) - CODE_VALUES[c], CODE_VALUES[c]) for c, w in enumerate(hist16) if w]
    bias = sum(w * e for w, e, _ in d) / W
    mse = sum(w * e * e for w, e, _ in d) / W
    ms = sum(w * v * v for w, _, v in d) / W
    return bias, (mse / ms) ** 0.5 if ms > 0 else 0.0


def code_lut(levels: Sequence[float]) -> List[int]:
    """16-entry code -> code map: each e2m1 code to the original code of its level (a
    zero level keeps the code's sign bit)."""
    lut = []
    for c in range(16):
        L = level_of(c, levels)
        if L == 0.0:
            lut.append(c & 0x8)
        else:
            lut.append(next(i for i in range(16) if CODE_VALUES[i] == L))
    return lut


def remap_packed(packed: torch.Tensor, lut: Sequence[int]) -> torch.Tensor:
    """Apply a 16-entry code map to both nibbles of packed FP4 bytes."""
    t = torch.tensor(lut, dtype=torch.uint8)
    b = packed.view(torch.uint8).long()
    return (t[b & 0xF] | (t[b >> 4] << 4)).view(packed.dtype)


def packed_histogram(packed: torch.Tensor) -> List[int]:
    b = packed.view(torch.uint8).flatten().long()
    return (torch.bincount(b & 0xF, minlength=16) + torch.bincount(b >> 4, minlength=16)).tolist()


def unit_histogram(w: torch.Tensor) -> List[int]:
    """e2m1 code histogram of a weight matrix in unit space: block-32 UE8M0 scales and
    the e2m1 snap of the load-time quantizer (formats.codebook)."""
    _, _, nib = codebook.f64_to_codes_scales(w.double(), mode="sign", want_nibbles=True)
    return torch.bincount(nib.flatten().long(), minlength=16).tolist()


# ---------------------------------------------------------------------- safetensors
def read_header(path: str) -> Tuple[dict, int]:
    """-> (header dict, byte offset of the data section)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        return json.loads(f.read(n)), 8 + n


def _is_expert(name: str, meta: dict, patterns) -> bool:
    return meta.get("dtype") in ("I8", "U8") and any(re.match(p, name) for p in patterns)


def repack_file(src: str, dst: str, lut: Sequence[int], patterns=EXPERT_PATTERNS) -> int:
    """Copy one safetensors file, remapping the codes of the matched tensors -> tensors
    changed.  The header and every other byte are copied unchanged."""
    hdr, base = read_header(src)
    shutil.copyfile(src, dst)
    n = 0
    with open(dst, "r+b") as f:
        for name, meta in hdr.items():
            if name == "__metadata__" or not _is_expert(name, meta, patterns):
                continue
            a, b = meta["data_offsets"]
            f.seek(base + a)
            raw = bytearray(f.read(b - a))
            out = remap_packed(torch.frombuffer(raw, dtype=torch.uint8), lut)
            f.seek(base + a)
            f.write(out.numpy().tobytes())
            n += 1
    return n


def _shards(d: str) -> List[str]:
    return sorted(x for x in os.listdir(d) if x.endswith(".safetensors"))


def repack(src: str, dst: str, K: int, patterns=EXPERT_PATTERNS, per_tensor: bool = False) -> dict:
    """K-level repack of a checkpoint directory: one codebook from the pooled histogram of
    every matched tensor (or one per tensor with ``per_tensor``).  Files without experts and
    non-shard files are copied unchanged."""
    os.makedirs(dst, exist_ok=True)
    pooled = [0] * 16
    per: Dict[Tuple[str, str], List[int]] = {}
    for fn in _shards(src):
        p = os.path.join(src, fn)
        hdr, base = read_header(p)
        with open(p, "rb") as f:
            for name, meta in hdr.items():
                if name == "__metadata__" or not _is_expert(name, meta, patterns):
                    continue
                a, b = meta["data_offsets"]
                f.seek(base + a)
                h = packed_histogram(torch.frombuffer(bytearray(f.read(b - a)), dtype=torch.uint8))
                per[(fn, name)] = h
                pooled = [x + y for x, y in zip(pooled, h)]
    levels, err = optimal_levels(pooled, K)
    changed = 0
    for fn in os.listdir(src):
        s, d = os.path.join(src, fn), os.path.join(dst, fn)
        if not os.path.isfile(s):
            continue
        if fn.endswith(".safetensors") and any(k[0] == fn for k in per):
            if per_tensor:
                hdr, base = read_header(s)
                shutil.copyfile(s, d)
                with open(d, "r+b") as f:
                    for (f_, name), h in per.items():
                        if f_ != fn:
                            continue
                        a, b = hdr[name]["data_offsets"]
                        f.seek(base + a)
                        raw = bytearray(f.read(b - a))
                        f.seek(base + a)
                        f.write(remap_packed(torch.frombuffer(raw, dtype=torch.uint8),
                                             code_lut(optimal_levels(h, K)[0])).numpy().tobytes())
                        changed += 1
            else:
                changed += repack_file(s, d, code_lut(levels), patterns)
        else:
            shutil.copyfile(s, d)
    return {"levels": levels, "pooled_sq_error": err, "tensors": changed, "K": K}


def gate(src: str, patterns=EXPERT_PATTERNS, tmp: Optional[str] = None) -> bool:
    """K = 16 keeps every code: the repacked files must equal the originals byte for byte."""
    import filecmp
    import tempfile
    with tempfile.TemporaryDirectory(dir=tmp) as d:
        repack(src, d, 16, patterns)
        return all(filecmp.cmp(os.path.join(src, fn), os.path.join(d, fn), shallow=False) for fn in _shards(src))


# ---------------------------------------------------------------------- sweep
def sweep_tensor(w: torch.Tensor) -> dict:
    """Optimal (possibly asymmetric) vs sign-symmetric 4-level codebooks of one tensor."""
    h = unit_histogram(w)
    opt, _ = optimal_levels(h, 4)
    sym, _ = symmetric_levels(h)
    b_o, r_o = error_stats(h, opt)
    b_s, r_s = error_stats(h, sym)
    return {"optimal": opt, "optimal_bias": b_o, "optimal_rel_rms": r_o,
            "symmetric": sym, "symmetric_bias": b_s, "symmetric_rel_rms": r_s}


def _synthetic(n: int, rows: int, cols: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    for i in range(n):
        if i % 2:
            yield f"student-t[{i}]", torch.distributions.StudentT(4.0).sample((rows, cols)) * 0.02
        else:
            yield f"normal[{i}]", torch.randn(rows, cols, generator=g) * 0.02


def _checkpoint(d: str, limit: int):
    from ..models.loader import CheckpointReader
    rd = CheckpointReader(d)
    n = 0
    for name in sorted(rd.where):
        if not any(re.match(p, name) for p in EXPERT_PATTERNS):
            continue
        prefix = name[: -len(".weight")]
        yield name, rd.dense64(prefix).float()
        n += 1
        if n >= limit:
            return


def main(argv=None):
    ap = argparse.ArgumentParser(description="2-bit codebook studies")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("sweep", help="optimal vs sign-symmetric 4-level codebooks")
    s.add_argument("--checkpoint", help="checkpoint directory (default: synthetic tensors)")
    s.add_argument("--limit", type=int, default=16)
    s.add_argument("--rows", type=int, default=256)
    s.add_argument("--cols", type=int, default=1024)
    s.add_argument("--seed", type=int, default=0)
    r = sub.add_parser("repack", help="K-level repack of FP4 routed experts")
    r.add_argument("--src", required=True)
    r.add_argument("--dst", required=True)
    r.add_argument("--levels", type=int, default=4)
    r.add_argument("--per-tensor", action="store_true")
    g = sub.add_parser("gate", help="K = 16 round trip must be byte-identical")
    g.add_argument("--src", required=True)
    a = ap.parse_args(argv)
    if a.cmd == "sweep":
        src = _checkpoint(a.checkpoint, a.limit) if a.checkpoint else _synthetic(a.limit, a.rows, a.cols, a.seed)
        rows = []
        for name, w in src:
            res = sweep_tensor(w)
            rows.append(res)
            print(f"{name:48s} opt {res['optimal']} bias {res['optimal_bias']:+.4f} rms {res['optimal_rel_rms']:.4f}"
                  f" | sym {res['symmetric']} bias {res['symmetric_bias']:+.4f} rms {res['symmetric_rel_rms']:.4f}")
        if rows:
            mb = lambda k: sum(abs(x[k]) for x in rows) / len(rows)   # noqa: E731
            print(f"mean |bias|: optimal {mb('optimal_bias'):.4f}, symmetric {mb('symmetric_bias'):.4f}; "
                  f"mean rel rms: optimal {mb('optimal_rel_rms'):.4f}, symmetric {mb('symmetric_rel_rms'):.4f}")
        return 0
    if a.cmd == "repack":
        print(json.dumps(repack(a.src, a.dst, a.levels, per_tensor=a.per_tensor)))
        return 0
    ok = gate(a.src)
    print("gate:", "byte-identical" if ok else "MISMATCH")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

"""Offline codebook tools: the K-level search is the exact optimum (checked against a
brute force over every level subset), the sign-symmetric winner on Gaussian experts is the
served {-4, -1, 1, 4} with a far smaller bias than the asymmetric optimum, the code map is
the identity at K = 16, and a checkpoint repack keeps headers, offsets and non-expert bytes
(K = 16: byte-identical files)."""
import itertools
import os

import pytest
import torch

from vllm_moet_b200.tools import codebook_search as cs


def _brute(hist16, K):
    vh = cs.value_histogram(hist16)
    best = None
    for lv in itertools.combinations(cs.GRID, K):
        e = sum(w * min((v - L) ** 2 for L in lv) for v, w in vh.items())
        best = e if best is None else min(best, e)
    return best


@pytest.mark.parametrize("seed,K", [(0, 2), (1, 3), (2, 4), (3, 5)])
def test_optimal_levels_is_exact(seed, K):
    g = torch.Generator().manual_seed(seed)
    hist = (torch.rand(16, generator=g) * 100).round().tolist()
    hist[int(torch.randint(16, (1,), generator=g))] = 0
    levels, err = cs.optimal_levels(hist, K)
    assert len(levels) == K and all(L in cs.GRID for L in levels)
    assert abs(err - _brute(hist, K)) < 1e-9 * max(1.0, err)
    vh = cs.value_histogram(hist)
    assert abs(err - sum(w * min((v - L) ** 2 for L in levels) for v, w in vh.items())) < 1e-9 * max(1.0, err)


def test_sweep_reproduces_the_symmetric_finding():
    g = torch.Generator().manual_seed(5)
    res = cs.sweep_tensor(torch.randn(256, 1024, generator=g) * 0.02)
    assert res["symmetric"] == [-4.0, -1.0, 1.0, 4.0]
    assert res["optimal"] != res["symmetric"]                       # the optimum is one-sided
    assert abs(res["symmetric_bias"]) * 10 < abs(res["optimal_bias"])
    assert abs(res["symmetric_rel_rms"] - res["optimal_rel_rms"]) < 0.01


def test_code_lut():
    assert cs.code_lut(cs.GRID) == list(range(16))
    lut = cs.code_lut([-4.0, -1.0, 1.0, 4.0])
    vals = [cs.CODE_VALUES[c] for c in lut]
    assert set(vals) == {-4.0, -1.0, 1.0, 4.0}
    assert lut[0] != lut[8] and cs.CODE_VALUES[lut[0]] == 1.0 and cs.CODE_VALUES[lut[8]] == -1.0   # +0 / -0
    packed = torch.tensor([0x00, 0x8F, 0x57], dtype=torch.uint8)
    out = cs.remap_packed(packed, lut)
    for b, o in zip(packed.tolist(), out.tolist()):
        assert o & 0xF == lut[b & 0xF] and o >> 4 == lut[b >> 4]


def test_repack_and_gate(tmp_path):
    from safetensors.torch import save_file
    src, dst = tmp_path / "src", tmp_path / "dst"
    src.mkdir()
    g = torch.Generator().manual_seed(9)
    t = {
        "layers.3.ffn.experts.7.w1.weight": torch.randint(-128, 127, (64, 32), generator=g, dtype=torch.int8),
        "layers.3.ffn.experts.7.w1.scale": torch.randint(0, 255, (64, 2), generator=g, dtype=torch.uint8),
        "layers.3.attn.wq.weight": torch.randn(16, 16, generator=g).to(torch.bfloat16),
        "mtp.0.ffn.experts.1.w2.weight": torch.randint(-128, 127, (8, 8), generator=g, dtype=torch.int8),
    }
    save_file(t, str(src / "model-00001-of-00001.safetensors"))
    (src / "config.json").write_text("{}")
    assert cs.gate(str(src))
    info = cs.repack(str(src), str(dst), 4)
    assert info["tensors"] == 1 and len(info["levels"]) == 4
    a, b = (src / "model-00001-of-00001.safetensors").read_bytes(), (dst / "model-00001-of-00001.safetensors").read_bytes()
    assert len(a) == len(b)
    hdr, base = cs.read_header(str(src / "model-00001-of-00001.safetensors"))
    assert a[:base] == b[:base]                                      # header verbatim
    for name, meta in hdr.items():
        if name == "__metadata__":
            continue
        lo, hi = meta["data_offsets"]
        same = a[base + lo:base + hi] == b[base + lo:base + hi]
        assert same == (name != "layers.3.ffn.experts.7.w1.weight"), name   # MTP experts untouched
    w = torch.frombuffer(bytearray(b[base + hdr["layers.3.ffn.experts.7.w1.weight"]["data_offsets"][0]:
                                     base + hdr["layers.3.ffn.experts.7.w1.weight"]["data_offsets"][1]]),
                         dtype=torch.uint8)
    vals = {cs.CODE_VALUES[c] + 0.0 for c in torch.cat([w & 0xF, w >> 4]).tolist()}
    assert vals <= set(info["levels"]) | {0.0} and len(vals - {0.0}) <= 4
    assert os.path.exists(dst / "config.json")

"""Boot from the persistent quantisation caches: the second build of the same
model loads every MoE layer's expert planes from the planes cache / pack
instead of quantising, and the pools are byte-identical."""
import torch

from vllm_moet_b200.config import tiny_config
from vllm_moet_b200.models import weights as W
from vllm_moet_b200.residency import PlanesCache, make_store
from vllm_moet_b200.residency.sources import PackSource, PlanesSource


def _cfg():
    return tiny_config(expert_scale="ue8m0", dense_dtype="fp8", hidden=128, moe_intermediate=64, num_experts=4)


def _count_quant(monkeypatch):
    calls = {"n": 0}
    real = W.quantize_experts_cpu

    def counting(*a, **k):
        calls["n"] += 1
        return real(*a, **k)
    monkeypatch.setattr(W, "quantize_experts_cpu", counting)
    return calls


def test_planes_cache_boot(tmp_path, monkeypatch):
    calls = _count_quant(monkeypatch)
    src = PlanesSource(PlanesCache(str(tmp_path), "ckpt-a", background=False))
    a = W.random_weights(_cfg(), "cpu", seed=1, expert_source=src)
    first = calls["n"]
    assert first > 0 and src.misses > 0 and src.hits == 0
    src2 = PlanesSource(PlanesCache(str(tmp_path), "ckpt-a", background=False))
    b = W.random_weights(_cfg(), "cpu", seed=1, expert_source=src2)
    assert calls["n"] == first and src2.hits == src.misses and src2.misses == 0
    for la, lb in zip(a.layers + [a.mtp.layer], b.layers + [b.mtp.layer]):
        if la.is_moe:
            assert torch.equal(la.experts.pool, lb.experts.pool)
    # non-expert weights are still drawn identically (the skipped draws keep streams aligned)
    assert torch.equal(a.lm_head.w, b.lm_head.w)


def test_pack_boot(tmp_path, monkeypatch):
    calls = _count_quant(monkeypatch)
    cfg = _cfg()
    lay = W.ExpertLayout(H=cfg.hidden, I=cfg.moe_intermediate)
    st = make_store("pack", cfg.num_layers + 1, cfg.num_experts, lay.slot_bytes, dir=str(tmp_path), ckpt_id="p")
    a = W.random_weights(cfg, "cpu", seed=2, expert_source=PackSource(st))
    first = calls["n"]
    st2 = make_store("pack", cfg.num_layers + 1, cfg.num_experts, lay.slot_bytes, dir=str(tmp_path), ckpt_id="p")
    src = PackSource(st2)
    b = W.random_weights(cfg, "cpu", seed=2, expert_source=src)
    assert calls["n"] == first and src.hits >= 1
    assert torch.equal(a.layers[-1].experts.pool, b.layers[-1].experts.pool)

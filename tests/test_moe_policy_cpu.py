import torch

from vllm_moet_b200.models.moe_policy import apply_topp, check_layer_contract, is_w2_layer, layer_contract_violations


def test_topp_prunes_tail_statically():
    ids = torch.tensor([[3, 7, 1, 9], [2, 4, 6, 8]])
    w = torch.tensor([[0.1, 0.6, 0.25, 0.05], [0.25, 0.25, 0.25, 0.25]])
    pi, pw = apply_topp(ids, w, 0.8)
    # token 0: sorted 0.6 (7), 0.25 (1) -> mass before 3rd = 0.85 >= 0.8: keep {7, 1}
    assert torch.allclose(pw[0], torch.tensor([0.0, 0.6, 0.25, 0.0])) and pi[0].tolist() == [7, 7, 1, 7]
    # token 1: ties keep index order: mass before 4th = 0.75 < 0.8 -> keep all four
    assert pw[1].tolist() == [0.25] * 4
    pi, pw = apply_topp(ids, w, 0.1, min_keep=2)
    assert int((pw[0] > 0).sum()) == 2
    assert apply_topp(ids, w, 0.0)[1] is w


def test_contracts_and_layer_selection(monkeypatch):
    assert layer_contract_violations({"hidden_act": "silu", "torch_dtype": "bfloat16"}) == []
    bad = layer_contract_violations({"hidden_act": "gelu", "expert_bias": True, "torch_dtype": "float32"})
    assert len(bad) == 3
    import pytest
    with pytest.raises(ValueError, match="gelu"):
        check_layer_contract({"hidden_act": "gelu"})
    assert is_w2_layer(3, 32) and not is_w2_layer(32, 32)
    monkeypatch.setenv("VLLM_MOE_W2_DRAFT", "1")
    assert is_w2_layer(32, 32)


def test_oracle_topp_changes_output_only_when_enabled():
    from vllm_moet_b200.config import tiny_config
    from vllm_moet_b200.models import reference as ref
    from vllm_moet_b200.models.weights import random_weights
    cfg = tiny_config()
    mw = random_weights(cfg, "cpu", seed=0)
    toks = torch.tensor([5, 6, 7, 8])
    cs = ref.rope_cos_sin(cfg, 16)
    a, _ = ref.forward(mw, toks, torch.arange(4), cs)
    ref.set_topp(0.3)
    try:
        b, _ = ref.forward(mw, toks, torch.arange(4), cs)
    finally:
        ref.set_topp(0.0)
    assert not torch.allclose(a, b)

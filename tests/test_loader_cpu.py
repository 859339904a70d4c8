"""Loading a DeepSeek-layout Hugging Face checkpoint: config mapping, dense linears
(bf16 and FP8 with UE8M0 block scales kept bit-exactly), routed experts from bf16,
FP8 (arbitrary f32 block scales) and NVFP4 converted exactly as the reference's
converters do, the MTP module, and the engine running the loaded model."""
import json
import os

import pytest
import torch
from safetensors.torch import save_file

from vllm_moet_b200.formats import codebook, fp8, planes
from vllm_moet_b200.models.loader import CheckpointReader, hf_config, load_weights

H, V, NH, QL, KVL, NOPE, ROPE, VD, E, I, DI, L = 256, 512, 4, 128, 64, 32, 16, 32, 8, 128, 256, 2


def _config(quant: bool):
    c = {"model_type": "deepseek_v3", "hidden_size": H, "num_hidden_layers": L, "vocab_size": V,
         "first_k_dense_replace": 1, "intermediate_size": DI, "num_attention_heads": NH, "q_lora_rank": QL,
         "kv_lora_rank": KVL, "qk_nope_head_dim": NOPE, "qk_rope_head_dim": ROPE, "v_head_dim": VD,
         "n_routed_experts": E, "moe_intermediate_size": I, "num_experts_per_tok": 2, "n_shared_experts": 1,
         "scoring_func": "sigmoid", "n_group": 1, "topk_group": 1, "norm_topk_prob": True,
         "routed_scaling_factor": 2.5, "rms_norm_eps": 1e-6, "rope_theta": 10000.0,
         "num_nextn_predict_layers": 1, "max_position_embeddings": 4096}
    if quant:
        c["quantization_config"] = {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128]}
    return c


def _fp8_pow2(w):
    q, s = fp8.quant_weight_fp8(w)
    return q, torch.exp2(s.float() - 127)


def _fp8_any(w):
    """FP8 with arbitrary (non power-of-two) f32 block scales, as FP8 checkpoints store them."""
    N, K = w.shape
    s = w.abs().reshape(N // 128, 128, K // 128, 128).amax((1, 3)) / 448.0
    q = (w / s.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(torch.float8_e4m3fn)
    return q, s.float()


def _make_ckpt(d, quant: bool, nvfp4_experts: bool = False, shards: int = 2, hc: int = 1):
    g = torch.Generator().manual_seed(1)
    rn = lambda *s: torch.randn(*s, generator=g) * 0.05       # noqa: E731
    T = {"model.embed_tokens.weight": rn(V, H).to(torch.bfloat16), "model.norm.weight": 1 + rn(H) * 0.1,
         "lm_head.weight": rn(V, H).to(torch.bfloat16)}
    raw = {}

    def dense(name, w):
        raw[name] = w
        if quant:
            q, s = _fp8_pow2(w)
            T[name + ".weight"], T[name + ".weight_scale_inv"] = q, s
        else:
            T[name + ".weight"] = w.to(torch.bfloat16)
            raw[name] = w.to(torch.bfloat16).float()

    def expert(name, w):
        if nvfp4_experts:
            packed, sf, t2 = codebook.f32_to_nvfp4(w, float(w.abs().max()) / (6 * 448))
            T[name + ".weight"], T[name + ".weight_scale"], T[name + ".weight_scale_2"] = packed, sf, t2
        elif quant:
            q, s = _fp8_any(w)
            T[name + ".weight"], T[name + ".weight_scale_inv"] = q, s
        else:
            T[name + ".weight"] = w.to(torch.bfloat16)

    for li in range(L + 1):                     # layer L is the MTP module
        P = f"model.layers.{li}."
        for n, sh in (("input_layernorm", H), ("post_attention_layernorm", H), ("self_attn.q_a_layernorm", QL),
                      ("self_attn.kv_a_layernorm", KVL)):
            T[P + n + ".weight"] = 1 + rn(sh) * 0.1
        dense(P + "self_attn.q_a_proj", rn(QL, H))
        dense(P + "self_attn.kv_a_proj_with_mqa", rn(KVL + ROPE, H))
        dense(P + "self_attn.q_b_proj", rn(NH * (NOPE + ROPE), QL))
        dense(P + "self_attn.kv_b_proj", rn(NH * (NOPE + VD), KVL))
        dense(P + "self_attn.o_proj", rn(H, NH * VD))
        if li == 0:
            dense(P + "mlp.gate_proj", rn(DI, H)); dense(P + "mlp.up_proj", rn(DI, H))
            dense(P + "mlp.down_proj", rn(H, DI))
        else:
            T[P + "mlp.gate.weight"] = rn(E, H).to(torch.bfloat16)
            T[P + "mlp.gate.e_score_correction_bias"] = rn(E) * 0.1
            dense(P + "mlp.shared_experts.gate_proj", rn(I, H)); dense(P + "mlp.shared_experts.up_proj", rn(I, H))
            dense(P + "mlp.shared_experts.down_proj", rn(H, I))
            for e in range(E):
                expert(P + f"mlp.experts.{e}.gate_proj", rn(I, H))
                expert(P + f"mlp.experts.{e}.up_proj", rn(I, H))
                expert(P + f"mlp.experts.{e}.down_proj", rn(H, I))
        if hc > 1:
            for site in ("hc_attn", "hc_ffn"):
                T[P + site + "_fn"], T[P + site + "_base"] = rn((2 + hc) * hc, hc * H), rn((2 + hc) * hc) * 10
                T[P + site + "_scale"] = 1 + rn(3)
            if li == L:
                T[P + "hc_head_fn"], T[P + "hc_head_base"], T[P + "hc_head_scale"] = rn(hc, hc * H), rn(hc), 1 + rn(1)
        if li == L:
            T[P + "enorm.weight"] = 1 + rn(H) * 0.1
            T[P + "hnorm.weight"] = 1 + rn(H) * 0.1
            T[P + "shared_head.norm.weight"] = 1 + rn(H) * 0.1
            dense(P + "eh_proj", rn(H, 2 * H))
    os.makedirs(d, exist_ok=True)
    names = sorted(T)
    wm = {}
    for k in range(shards):
        part = {n: T[n].contiguous() for n in names[k::shards]}
        fn = f"model-{k + 1:05d}-of-{shards:05d}.safetensors"
        save_file(part, os.path.join(d, fn))
        wm.update({n: fn for n in part})
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": wm}, f)
    if hc > 1:
        T["model.hc_head_fn"], T["model.hc_head_base"], T["model.hc_head_scale"] = rn(hc, hc * H), rn(hc), 1 + rn(1)
        for n in ("model.hc_head_fn", "model.hc_head_base", "model.hc_head_scale"):
            fn = "hc.safetensors"
            wm[n] = fn
        save_file({n: T[n] for n in wm if wm[n] == "hc.safetensors"}, os.path.join(d, "hc.safetensors"))
        with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": wm}, f)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(dict(_config(quant), **({"hc_mult": hc, "hc_sinkhorn_iters": 10} if hc > 1 else {})), f)
    return T, raw


def test_config_mapping(tmp_path):
    _make_ckpt(str(tmp_path), quant=True)
    cfg = hf_config(str(tmp_path))
    assert (cfg.hidden, cfg.num_layers, cfg.num_dense_layers, cfg.num_experts, cfg.top_k) == (H, L, 1, E, 2)
    assert (cfg.qk_nope_dim, cfg.v_head_dim, cfg.router, cfg.routed_scaling, cfg.dense_dtype) == \
        (NOPE, VD, "sigmoid", 2.5, "fp8")
    assert cfg.num_mtp_layers == 1


def test_fp8_checkpoint_maps_exactly(tmp_path):
    T, raw = _make_ckpt(str(tmp_path), quant=True)
    mw = load_weights(str(tmp_path))
    lw0, lw1 = mw.layers
    # UE8M0 FP8 linears keep their bytes: dequant == the checkpoint's block product
    want_qkv = torch.cat([raw["model.layers.0.self_attn.q_a_proj"], raw["model.layers.0.self_attn.kv_a_proj_with_mqa"]])
    q, s = _fp8_pow2(want_qkv)
    assert torch.equal(lw0.qkv_a.w, q.view(torch.uint8))
    for name, lin in (("self_attn.q_b_proj", lw0.q_b), ("self_attn.o_proj", lw0.o), ("self_attn.kv_b_proj", lw1.kv_b)):
        li = 0 if lin is not lw1.kv_b else 1
        ref = CheckpointReader(str(tmp_path)).dense64(f"model.layers.{li}.{name}").float()
        assert torch.equal(lin.dequant(), ref), name
    assert torch.equal(lw1.router_bias, T["model.layers.1.mlp.gate.e_score_correction_bias"].float())
    assert torch.equal(lw0.attn_norm.float(), T["model.layers.0.input_layernorm.weight"].to(torch.bfloat16).float())
    # experts: FP8 blocks with arbitrary scales -> exact float64 products -> 2-bit codes
    rd = CheckpointReader(str(tmp_path))
    for e in (0, 5):
        P = f"model.layers.1.mlp.experts.{e}."
        w13 = torch.cat([rd.dense64(P + "gate_proj"), rd.dense64(P + "up_proj")])
        q13 = T[P + "gate_proj.weight"].double()
        assert torch.equal(w13[:I], q13 * T[P + "gate_proj.weight_scale_inv"].double().repeat_interleave(128, 0)
                           .repeat_interleave(128, 1))
        codes, sc, _ = codebook.f64_to_codes_scales(w13)
        got13, _ = lw1.experts.dequant_expert(e)
        assert torch.equal(got13, codebook.dequant_codes(codes, sc))
    assert mw.mtp is not None and torch.equal(mw.mtp.enorm.float(),
                                              T["model.layers.2.enorm.weight"].to(torch.bfloat16).float())


def test_nvfp4_experts_match_reference_converter(tmp_path):
    T, _ = _make_ckpt(str(tmp_path), quant=False, nvfp4_experts=True)
    mw = load_weights(str(tmp_path), with_mtp=False)
    P = "model.layers.1.mlp.experts.3."
    c_g, s_g, _ = codebook.nvfp4_to_codes_scales(T[P + "gate_proj.weight"], T[P + "gate_proj.weight_scale"],
                                                 T[P + "gate_proj.weight_scale_2"])
    got13, got2 = mw.layers[1].experts.dequant_expert(3)
    assert torch.equal(got13[:I], codebook.dequant_codes(c_g, s_g))
    c_d, s_d, _ = codebook.nvfp4_to_codes_scales(T[P + "down_proj.weight"], T[P + "down_proj.weight_scale"],
                                                 T[P + "down_proj.weight_scale_2"])
    assert torch.equal(got2, codebook.dequant_codes(c_d, s_d))


def test_engine_serves_the_checkpoint(tmp_path):
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    _make_ckpt(str(tmp_path), quant=False)
    llm = LLM(str(tmp_path), device="cpu", num_speculative_tokens=1, max_model_len=128)
    assert llm.cfg.hidden == H and llm.mw.mtp is not None
    p = [5, 9, 17, 33, 65]
    out = llm.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids
    assert out == reference.greedy_generate(llm.mw, p, 6)


def _tp_ckpt(rank, world, d):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM(d, device="cpu", num_speculative_tokens=1, max_model_len=128, tensor_parallel_size=world,
              tp_group=dist.group.WORLD, tp_rank=rank)
    return llm.generate([[5, 9, 17, 33, 65]], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids


def test_tp2_slices_of_the_checkpoint_match_one_rank(tmp_path):
    from mp_util import run_ranks
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    _make_ckpt(str(tmp_path), quant=False)
    want = LLM(str(tmp_path), device="cpu", num_speculative_tokens=1, max_model_len=128).generate(
        [[5, 9, 17, 33, 65]], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids
    assert run_ranks(_tp_ckpt, 2, str(tmp_path)) == [want, want]


def test_checkpoint_tokenizer_is_used(tmp_path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    _make_ckpt(str(tmp_path), quant=False)
    words = ["<s>", "</s>", "<pad>"] + [f"w{i}" for i in range(100)]
    tk = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<pad>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tk, bos_token="<s>", eos_token="</s>", pad_token="<pad>") \
        .save_pretrained(str(tmp_path))
    llm = LLM(str(tmp_path), device="cpu", num_speculative_tokens=1, max_model_len=128)
    assert llm.tokenizer.encode("w5 w7") == [8, 10] and llm.tokenizer.eos_token_id == 1
    out = llm.generate(["w5 w7 w9"], SamplingParams(max_tokens=4, ignore_eos=True))[0]
    assert out.prompt_token_ids == [0, 8, 10, 12]
    assert out.outputs[0].text == llm.tokenizer.decode(out.outputs[0].token_ids)


def test_nvfp4_dense_linear_roundtrip_and_loader(tmp_path):
    from vllm_moet_b200.models.weights import Nvfp4Linear, make_linear
    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 128, generator=g) * 0.05
    lin = make_linear(w, "nvfp4")
    assert isinstance(lin, Nvfp4Linear) and lin.shape == (64, 128)
    packed, sf, t2 = codebook.f32_to_nvfp4(w)
    ref = codebook.E2M1_VALUES[codebook.split_packed_e2m1(packed).long()].float() * \
        sf.float().repeat_interleave(16, 1) * t2
    assert torch.equal(lin.dequant(), ref) and float((lin.dequant() - w).abs().max()) < 0.05
    # the loader keeps NVFP4 dense tensors as they are when the model's dense format is NVFP4
    from safetensors.torch import save_file
    save_file({"x.weight": packed, "x.weight_scale": sf, "x.weight_scale_2": t2}, str(tmp_path / "m.safetensors"))
    rd = CheckpointReader(str(tmp_path))
    got = rd.linear("x", "nvfp4")
    assert isinstance(got, Nvfp4Linear) and torch.equal(got.dequant(), ref)
    assert torch.equal(rd.dense64("x").float(), ref)


def test_loader_refuses_layouts_it_cannot_represent(tmp_path):
    T, _ = _make_ckpt(str(tmp_path), quant=False, shards=1)
    from safetensors.torch import save_file
    save_file({"model.layers.0.hc_pre_fn": torch.zeros(4)}, str(tmp_path / "extra.safetensors"))
    idx = json.load(open(tmp_path / "model.safetensors.index.json"))
    idx["weight_map"]["model.layers.0.hc_pre_fn"] = "extra.safetensors"
    json.dump(idx, open(tmp_path / "model.safetensors.index.json", "w"))
    with pytest.raises(ValueError, match="hyper-connection"):      # hc tensors, config without hc_mult
        load_weights(str(tmp_path))


def test_hyper_connection_checkpoint(tmp_path):
    """mHC (hc_mult 2): the hc_* tensors land on every layer, the head and the MTP module,
    and the engine serving the loaded model decodes the oracle's greedy chain."""
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference as ref
    from vllm_moet_b200 import SamplingParams
    T, _ = _make_ckpt(str(tmp_path), quant=False, shards=1, hc=2)
    cfg = hf_config(str(tmp_path))
    assert (cfg.hc_mult, cfg.hc_sinkhorn_iters) == (2, 10)
    mw = load_weights(str(tmp_path))
    assert torch.equal(mw.layers[1].hc_ffn.fn, T["model.layers.1.hc_ffn_fn"].float())
    assert torch.equal(mw.extra["hc_head"].base, T["model.hc_head_base"].float())
    assert torch.equal(mw.mtp.hc_head.scale, T[f"model.layers.{L}.hc_head_scale"].float())
    llm = LLM(str(tmp_path), device="cpu", num_speculative_tokens=2, max_model_len=128)
    prompt = [5, 17, 33, 2, 9]
    out = llm.generate([prompt], SamplingParams(max_tokens=12, ignore_eos=True))[0].outputs[0].token_ids
    assert out == ref.greedy_generate(llm.mw, prompt, 12)

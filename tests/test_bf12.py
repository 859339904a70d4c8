"""bf12 lossless BF16 container: CPU round trip (special values included),
size, and the GPU decode kernel against the reference decoder."""
import pytest
import torch

from vllm_moet_b200.formats import bf12


def _weights(n=4099, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    w[:6] = torch.tensor([float("nan"), float("inf"), -float("inf"), 0.0, -0.0, 1e-40]).to(torch.bfloat16)
    w[6] = 3.0e38
    return w


def test_roundtrip_bit_exact_and_size():
    w = _weights()
    b = bf12.encode(w)
    d = bf12.decode(b)
    assert torch.equal(d.view(torch.int16), w.view(torch.int16))
    big = (torch.randn(1 << 16) * 0.02).to(torch.bfloat16)
    assert bf12.encode(big).bits_per_weight() < 12.3


def test_linear_matches_bf16():
    w = (torch.randn(64, 32) * 0.02).to(torch.bfloat16)
    x = torch.randn(3, 32).to(torch.bfloat16)
    lin = bf12.Bf12Linear(w)
    assert torch.equal(lin(x), x @ w.t())


@pytest.mark.gpu
@pytest.mark.parametrize("n", [8, 4099, 1 << 20])
def test_gpu_decode_kernel(n):
    w = _weights(max(n, 8))[:n].contiguous()
    b = bf12.encode(w).to("cuda")
    from vllm_moet_b200.ops import native
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    native().bf12_decode(b.classes, b.lo, b.lut, b.esc_pos, b.esc_hi, out)
    assert torch.equal(out.cpu().view(torch.int16), w.view(torch.int16))
    lin = bf12.Bf12Linear(w.view(1, n).cuda())
    assert torch.equal(lin.decoded().cpu().view(torch.int16), w.view(1, n).view(torch.int16))


def test_convert_model_is_lossless_in_the_engine(monkeypatch):
    """VLLM_MOE_W2_BF12=1: after load every dense BF16 linear above the size floor is
    re-packed into the 12-bit container (verified bit for bit), excluded names stay BF16,
    and the engine emits exactly the tokens of the unconverted model."""
    import torch
    from vllm_moet_b200 import LLM, SamplingParams
    from vllm_moet_b200.config import get_preset
    from vllm_moet_b200.formats.bf12 import Bf12Linear
    from vllm_moet_b200.models.weights import FloatLinear, random_weights
    cfg = get_preset("tiny-moe").replace(dense_dtype="bf16")

    def bf16_model():
        mw = random_weights(cfg, "cpu", seed=4, with_mtp=True)
        for lw in list(mw.layers) + [mw.mtp.layer]:
            for a in ("qkv_a", "q_b", "kv_b", "o", "gate_up", "down", "shared_gate_up", "shared_down"):
                lin = getattr(lw, a, None)
                if isinstance(lin, FloatLinear):       # a BF16 checkpoint's dense matrices
                    lin.w = lin.w.to(torch.bfloat16).float()
        return mw

    prompts = [[5, 9, 13, 200, 7, 31], [3, 3, 4, 8]]
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    plain = LLM(cfg, device="cpu", weights=bf16_model(), num_speculative_tokens=2)
    want = [o.outputs[0].token_ids for o in plain.generate(prompts, sp)]
    monkeypatch.setenv("VLLM_MOE_W2_BF12", "1")
    monkeypatch.setenv("VLLM_MOE_W2_BF12_MIN_NUMEL", "1024")
    monkeypatch.setenv("VLLM_MOE_W2_BF12_EXCLUDE", "layers.0.o")
    conv = LLM(cfg, device="cpu", weights=bf16_model(), num_speculative_tokens=2)
    st = conv.bf12_stats
    assert st["converted"] > 0 and st["skipped_verify"] == 0
    assert st["bytes_after"] < 0.8 * st["bytes_before"]
    assert isinstance(conv.mw.layers[0].q_b, Bf12Linear) and isinstance(conv.mw.layers[0].o, FloatLinear)
    got = [o.outputs[0].token_ids for o in conv.generate(prompts, sp)]
    assert got == want

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

"""Trellis base tier kernels (csrc/kernels/trellis.cu) against the fp32 CPU path of the
same packs: the input / output rotations, the decode GEMV over expert groups (1, 3 and
9 tokens: one row, several rows, and experts split over two groups), both codebooks,
2 / 3 / 4 bits, widths whose Hadamard block is below 128 and n-tile counts that do not
fill the last CTA."""
import pytest
import torch

from vllm_moet_b200.formats import trellis as tf
from vllm_moet_b200.residency import trellis_tier as tt

pytestmark = pytest.mark.gpu


def _random_pack(d, E, H, I, K13, K2, L, codebook, seed):
    """A pack of random words and scale vectors: the kernels' arithmetic does not depend
    on the words being a good encoding."""
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    out = {}
    for e in range(E):
        for name, (n, k, K) in {"w1": (I, H, K13), "w3": (I, H, K13), "w2": (H, I, K2)}.items():
            out[f"e{e}.{name}.k{K}.trellis"] = torch.randint(-32768, 32768, (k // 16, n // 16, 16 * K), generator=g,
                                                             dtype=torch.int64).to(torch.int16)
            out[f"e{e}.{name}.k{K}.suh"] = ((torch.rand(k, generator=g) + 0.5) *
                                           (torch.randint(0, 2, (k,), generator=g) * 2 - 1)).half() * 0.1
            out[f"e{e}.{name}.k{K}.svh"] = ((torch.rand(n, generator=g) + 0.5) *
                                           (torch.randint(0, 2, (n,), generator=g) * 2 - 1)).half() * 0.1
    save_file(out, tt.pack_path(str(d), 0), metadata={
        "format": tf.FORMAT, "L": str(L), "codebook": codebook, "num_experts": str(E),
        "w13_k": str(K13), "w2_k": str(K2)})


def _rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().norm().clamp_min(1e-30))


def test_trellis_rotations_match_fwht():
    from vllm_moet_b200.ops import native
    C = native()
    torch.manual_seed(0)
    for n in (96, 384, 4096):
        x = torch.randn(3, n, device="cuda")
        su = (torch.randn(5, n, device="cuda")).half()
        src = torch.tensor([2, 0, -1, 1], dtype=torch.int32, device="cuda")
        eid = torch.tensor([4, 0, 1, 3], dtype=torch.int32, device="cuda")
        out = torch.empty(4, n, device="cuda")
        C.trellis_rot_in(x, src, eid, su, out)
        for p in range(4):
            if int(src[p]) < 0:
                assert (out[p] == 0).all()
                continue
            want = tf.fwht((x[int(src[p])] * su[int(eid[p])].float()).double().cpu())
            assert _rel(out[p], want) < 1e-5
        sc = torch.rand(4, device="cuda")
        y = torch.empty_like(out)
        C.trellis_rot_out(out, eid, su, sc, y)
        for p in range(4):
            want = tf.fwht(out[p].double().cpu()) * su[int(eid[p])].double().cpu() * float(sc[p])
            assert _rel(y[p], want) < 1e-5


@pytest.mark.parametrize("K13,K2,L,codebook", [(2, 2, 16, "3inst"), (3, 4, 12, "1mad"), (2, 3, 16, "1mad")])
def test_trellis_tier_gpu_matches_cpu(tmp_path, K13, K2, L, codebook):
    E, H, I = 8, 384, 96
    _random_pack(tmp_path, E, H, I, K13, K2, L, codebook, seed=K13 * 10 + K2)
    cpu = tt.TrellisBaseTier(str(tmp_path), [0], act_limit=7.0)
    gpu = tt.TrellisBaseTier(str(tmp_path), [0], device="cuda", act_limit=7.0)
    g = torch.Generator().manual_seed(3)
    for T in (1, 3, 9):
        x = torch.randn(T, H, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:4] for _ in range(T)])
        w = torch.rand(T, 4, generator=g)
        mask = torch.zeros(T, 4, dtype=torch.bool)
        mask[0, 1] = True
        for m in (None, mask):
            want = cpu.forward_topk(0, x, ids, w, fp4_mask=m)
            got = gpu.forward_topk(0, x.cuda(), ids.cuda(), w.cuda(),
                                   fp4_mask=None if m is None else m.cuda())
            torch.cuda.synchronize()
            assert got.shape == (T, H) and got.is_cuda
            assert _rel(got, want) < 1e-4, (T, m is not None)
        # deterministic: fixed-order sums everywhere
        again = gpu.forward_topk(0, x.cuda(), ids.cuda(), w.cuda())
        assert torch.equal(again, gpu.forward_topk(0, x.cuda(), ids.cuda(), w.cuda()))


def test_trellis_delta_pool_gpu_matches_cpu(tmp_path):
    E, H, I = 8, 256, 128
    _random_pack(tmp_path, E, H, I, 2, 2, 12, "3inst", seed=11)
    g = torch.Generator().manual_seed(4)
    true = [(torch.randn(2 * I, H, generator=g) * 0.01, torch.randn(H, I, generator=g) * 0.01) for _ in range(3)]
    tiers = {}
    for dev in ("cpu", "cuda"):
        t = tt.TrellisBaseTier(str(tmp_path), [0], device=dev, act_limit=7.0)
        pool = tt.TrellisDeltaPool(t, slots=2, dk13=2, dk2=3, L=8)
        for e in (2, 5, 7):                       # the third promotion evicts expert 2
            pool.promote(0, e, *true[(2, 5, 7).index(e)])
        tiers[dev] = (t, pool)
    assert torch.equal(tiers["cuda"][1].slot_of[0], tiers["cpu"][1].slot_of[0])
    for T in (1, 4):
        x = torch.randn(T, H, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:4] for _ in range(T)])
        ids[0] = torch.tensor([5, 7, 0, 2])        # both pooled experts, one evicted, one never pooled
        w = torch.rand(T, 4, generator=g)
        want = tiers["cpu"][0].forward_topk(0, x, ids, w, delta=tiers["cpu"][1])
        got = tiers["cuda"][0].forward_topk(0, x.cuda(), ids.cuda(), w.cuda(), delta=tiers["cuda"][1])
        torch.cuda.synchronize()
        assert _rel(got, want) < 1e-4, T

"""Router lookahead, host logic on CPU: the in-graph bookkeeping (recall of the previous
step's routing and of layer L+1's router on layer L's input, the prediction buffers and
the PILOT log) run through the runner's own code with the kernels replaced by torch, and
the PILOT consumer (read once, clear, skip resident and out-of-range experts, cap, gate on
a cold pool)."""
import types

import torch

from vllm_moet_b200.config import tiny_config
from vllm_moet_b200.engine.gpu_runner import NativeRunner
from vllm_moet_b200.models.weights import random_weights
from vllm_moet_b200.residency import Pilot


def _stub(K=6):
    cfg = tiny_config(num_layers=4)
    mw = random_weights(cfg, "cpu", seed=1)
    st = types.SimpleNamespace(cfg=cfg, mw=mw, dev=torch.device("cpu"), _route_tag="")
    st.ws = types.SimpleNamespace(get=lambda name, shape, dtype: torch.zeros(shape, dtype=dtype))

    def router_logits(hb, lw, out):
        out.copy_(hb.float() @ NativeRunner._router_w(st, lw).float().t())

    def router_topk(lg, bias, k, sigmoid, ng, tg, norm, scaling, ids, wts):
        s = torch.sigmoid(lg) if sigmoid else torch.softmax(lg, -1)
        ids.copy_(torch.topk(s + (bias if bias is not None else 0), k, dim=-1).indices.int())

    st._router_logits = router_logits
    st._router_w = lambda lw: NativeRunner._router_w(st, lw)
    st.C = types.SimpleNamespace(router_topk=router_topk)
    NativeRunner.enable_looka(st, K, True, 12)
    return st


def test_lookahead_bookkeeping():
    st = _stub()
    L = st._looka
    assert L["n_main"] >= 3
    T, k, H = 4, st.cfg.top_k, st.cfg.hidden
    ctx = types.SimpleNamespace(mode="decode")
    g = torch.Generator().manual_seed(0)
    hb = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids0 = torch.randint(0, st.cfg.num_experts, (T, k), generator=g).int()
    NativeRunner._looka_step(st, 0, hb, ids0, ctx)
    assert st.looka_tot.tolist() == [T * k, 0]                 # layer 0: no lookahead target
    assert st.looka_hits[0] == 0                               # nothing routed before
    want = torch.topk(torch.sigmoid(hb.float() @ st._router_w(L["layers"][1]).float().t()), L["K"]).indices
    assert torch.equal(st._looka_pred[:T].long().sort(-1).values, want.sort(-1).values)
    assert torch.equal(st.pilot_log[1, :T], st._looka_pred[:T])
    # layer 1 routed exactly to the first k predicted experts: lookahead recall 1
    ids1 = st._looka_pred[:T, :k].clone()
    NativeRunner._looka_step(st, 1, hb, ids1, ctx)
    assert st.looka_hits[1] == T * k and st.looka_tot[1] == T * k
    # the same routing at layer 0 next step: previous-step recall 1 for those rows
    NativeRunner._looka_step(st, 0, hb, ids0, ctx)
    assert st.looka_hits[0] == T * k
    r = NativeRunner.looka_recall(st)
    assert 0 < r["previous_step"] <= 1 and r["router_lookahead"] == 1.0
    # MTP draft passes and prefill are not scored
    before = st.looka_tot.clone()
    st._route_tag = ".p1"
    NativeRunner._looka_step(st, 0, hb, ids0, ctx)
    st._route_tag = ""
    NativeRunner._looka_step(st, 0, hb, ids0, types.SimpleNamespace(mode="prefill"))
    assert torch.equal(st.looka_tot, before)


class _Cache:
    E = 8

    def __init__(self, resident):
        self.res, self.requests = set(resident), []

    def resident(self, li, e):
        return (li, e) in self.res

    def request_prefetch(self, pairs):
        self.requests.append(list(pairs))


def test_pilot_consumer():
    log = torch.full((3, 4, 2), -1, dtype=torch.int32)
    log[1, 0] = torch.tensor([2, 5])
    log[1, 1] = torch.tensor([5, 9])          # 9 is out of range
    log[2, 0] = torch.tensor([1, 3])
    cache = _Cache({(2, 3)})
    p = Pilot(cache, log, cap=2, min_replay=30.0)
    assert p.consume() == 2
    assert cache.requests == [[(1, 2), (1, 5)]]               # capped, in layer order
    assert (log == -1).all()                                   # consumed once
    assert p.consume() == 0 and len(cache.requests) == 1
    for _ in range(200):
        p.observe(False)                                       # the pool warmed up
    log[2, 0] = torch.tensor([1, 4])
    assert p.consume() == 0 and p.stats["warm_skips"] == 1 and (log == -1).all()

"""Residency tiers on the CPU: host stores (byte identity across backends,
cold / warm / reboot / evict / overflow / scan / preheat, injected read
faults, concurrent writers), planes cache identity, the expert cache's slot
policy and fail-closed fetch, miss replay to a fixed point (1 rank and a
2-rank gloo consensus), the confidence gate, the speculation guard and the
pool floors."""
import os

import pytest
import torch

from mp_util import run_ranks
from vllm_moet_b200.residency import (ConfidenceGate, DraftAffinity, ExpertCache, FetchError, LookaheadPrefetcher,
                                      PlanesCache, ReplayEngine, SpecGuard, gate_fire_floor, make_store,
                                      pack_has_layer, working_set_floor)
from vllm_moet_b200.residency.stores import pack_paths

L, E, SB = 3, 8, 5000


def layer_rows(li, seed=0):
    g = torch.Generator().manual_seed(seed * 100 + li)
    return torch.randint(0, 256, (E, SB), generator=g, dtype=torch.uint8)


def fill(store, layers=range(L)):
    for li in layers:
        store.add_layer(li, layer_rows(li))


@pytest.mark.parametrize("kind", ["pinned", "pack", "tiered"])
def test_backends_byte_identical(tmp_path, kind):
    st = make_store(kind, L, E, SB, dir=str(tmp_path), ckpt_id="t", arena_rows=5)
    fill(st)
    for li in range(L):
        want = layer_rows(li)
        for experts in ([0, 3, 7], [7, 0], [1, 2, 3, 4, 5, 6]):
            b = st.rows_for(li, experts)
            assert not b.failed
            for e, r in zip(experts, b.rows):
                assert torch.equal(r, want[e]), (kind, li, e)


def test_pack_reboot_and_identity(tmp_path):
    d = str(tmp_path)
    st = make_store("pack", L, E, SB, dir=d, ckpt_id="ck1")
    fill(st, [0, 2])
    st.release()
    assert pack_has_layer(d, "base", L, E, SB, 0, ckpt_id="ck1")
    assert not pack_has_layer(d, "base", L, E, SB, 1, ckpt_id="ck1")
    assert not pack_has_layer(d, "base", L, E, SB, 0, ckpt_id="other")   # another checkpoint never matches
    st2 = make_store("pack", L, E, SB, dir=d, ckpt_id="ck1")              # "reboot"
    assert st2.has_layer(0) and st2.has_layer(2) and not st2.has_layer(1)
    assert torch.equal(st2.rows_for(2, [5]).rows[0], layer_rows(2)[5])
    pack, side, _, _ = pack_paths(d, "base", L, E, SB, "ck1")
    assert os.path.getsize(pack) >= 3 * E * 8192 - 8192     # rows at (li*E+e)*stride, 4 KiB stride
    with open(side, "w") as f:
        f.write("{corrupt")
    st3 = make_store("pack", L, E, SB, dir=d, ckpt_id="ck1")              # corrupt sidecar -> rebuild
    assert not st3.has_layer(0)


def test_tiered_evict_scan_and_preheat(tmp_path):
    st = make_store("tiered", L, E, SB, dir=str(tmp_path), ckpt_id="t", arena_rows=4)
    fill(st)
    st.rows_for(0, [0, 1, 2, 3])
    assert st.stats()["arena_misses"] == 4
    st.rows_for(0, [0, 1])
    assert st.stats()["arena_hits"] == 2
    st.rows_for(1, [0])                     # evicts the LRU row (0, 2)
    assert st.stats()["arena_evictions"] == 1 and (0, 2) not in st.lru
    before = dict(st.lru)
    b = st.rows_for(2, [0, 1, 2, 3, 4, 5], scan=True)   # a sweep larger than the arena: no pollution
    assert not b.failed and dict(st.lru) == before
    assert torch.equal(b.rows[5], layer_rows(2)[5])
    b = st.rows_for(2, [6], scan=True)
    assert (2, 6) not in st.lru
    st.dump_heat()
    st2 = make_store("tiered", L, E, SB, dir=str(tmp_path), ckpt_id="t", arena_rows=4)
    assert st2.preheat() >= 3
    assert st2.rows_for(1, [0]).rows[0] is not None and st2.stats()["arena_hits"] >= 1


def test_injected_read_faults_never_publish(tmp_path):
    st = make_store("tiered", L, E, SB, dir=str(tmp_path), ckpt_id="t", arena_rows=6)
    fill(st)
    st.inject_read_faults(2)                # every 2nd read fails with EIO
    b = st.rows_for(0, [0, 1, 2, 3])
    assert len(b.failed) == 2
    for e, r in zip([0, 1, 2, 3], b.rows):
        assert (r is None) == (e in b.failed)
        if r is not None:
            assert torch.equal(r, layer_rows(0)[e])
    for e in b.failed:
        assert (0, e) not in st.lru         # a failed read is not in the arena
    st.inject_read_faults(0)
    b2 = st.rows_for(0, b.failed)
    assert not b2.failed and all(torch.equal(r, layer_rows(0)[e]) for e, r in zip(b.failed, b2.rows))


def _writer(rank, world, d):
    st = make_store("pack", L, E, SB, dir=d, ckpt_id="mp", suffix="rank0of1")
    st.add_layer(rank, layer_rows(rank))
    return sorted(st.layers)


def test_concurrent_writers_share_one_sidecar(tmp_path):
    run_ranks(_writer, 2, str(tmp_path))
    st = make_store("pack", L, E, SB, dir=str(tmp_path), ckpt_id="mp", suffix="rank0of1")
    assert st.has_layer(0) and st.has_layer(1)
    assert torch.equal(st.rows_for(1, [4]).rows[0], layer_rows(1)[4])


def test_planes_cache(tmp_path):
    pc = PlanesCache(str(tmp_path), "ck", tp_world=2, tp_rank=1)
    parts = {"codes13": torch.arange(100, dtype=torch.uint8), "sc13": torch.ones(7, dtype=torch.uint8)}
    assert pc.try_load(0, {"codes13": 100, "sc13": 7}) is None
    pc.store(0, parts)
    pc.flush()
    got = pc.try_load(0, {"codes13": 100, "sc13": 7})
    assert got is not None and torch.equal(got["codes13"], parts["codes13"])
    assert pc.try_load(0, {"codes13": 101, "sc13": 7}) is None        # exact sizes required
    assert "tp2-rank1" in pc.rank_dir and os.path.exists(os.path.join(pc.base, "meta.json"))
    pc2 = PlanesCache(str(tmp_path), "other-ckpt", tp_world=2, tp_rank=1)
    assert pc2.base != pc.base and pc2.try_load(0, {"codes13": 100, "sc13": 7}) is None
    assert PlanesCache(str(tmp_path), None).try_load(0, {"codes13": 100}) is None   # unverified: never cached
    pc.close()


def _cache(tmp_path, slots=6, policy="lru"):
    st = make_store("pinned", L, E, SB)
    fill(st)
    return ExpertCache(st, L, E, SB, slots, device="cpu", policy=policy, manager=False)


def test_expert_cache_promote_evict_pin(tmp_path):
    c = _cache(tmp_path)
    assert c.promote([(0, 1), (0, 2), (1, 3)]) == 3
    assert int(c.slot_table[0, 1]) >= 0 and torch.equal(c.pool[int(c.slot_table[0, 1])], layer_rows(0)[1])
    c.step_end()
    c.promote([(2, 0), (2, 1), (2, 2)])      # fills the pool
    c.step_end()
    c.note_routed(0, [1])                    # pinned for this step
    c.promote([(1, 7)])                      # evicts an unpinned slot, never (0, 1)
    assert c.resident(0, 1) and c.resident(1, 7) and c.stats["evictions"] == 1
    for li in range(L):
        for e in range(E):
            s = int(c.slot_table[li, e])
            assert (s >= 0) == c.resident(li, e)
            if s >= 0:
                assert torch.equal(c.pool[s], layer_rows(li)[e])
    with pytest.raises(FetchError):
        c.promote([(li, e) for li in range(L) for e in range(E)])   # more than the pool


def test_failed_fetch_publishes_nothing(tmp_path):
    st = make_store("pack", L, E, SB, dir=str(tmp_path), ckpt_id="f")
    fill(st)
    c = ExpertCache(st, L, E, SB, 8, device="cpu", manager=False)
    st.inject_read_faults(3)
    with pytest.raises(FetchError):
        c.promote([(0, 0), (0, 1), (0, 2), (0, 3)])
    assert int((c.slot_table >= 0).sum()) == 0 and c.stats["fetch_failures"] >= 1


class FakeModel:
    """A "step" routes fixed experts per layer; the fake kernel counts routed experts
    whose slot is -1 into miss_count (what the native expert GEMVs do in-graph)."""

    def __init__(self, cache, routes):
        self.cache, self.routes, self.state, self.outputs = cache, routes, 0, []

    def step(self):
        for li, ids in enumerate(self.routes):
            self.cache.miss_count += int((self.cache.slot_table[li, ids] < 0).sum())
        self.outputs.append(self.state)
        self.state += 1

    def restore(self):
        self.state -= 1


def test_replay_converges_single_rank(tmp_path):
    c = _cache(tmp_path, slots=12)
    routes = [torch.tensor([0, 1]), torch.tensor([2, 3, 4]), torch.tensor([5])]
    m = FakeModel(c, routes)
    r = ReplayEngine(c, fp_max=4)
    assert r.run(m.step, m.restore, lambda: routes) == 1      # one replay after fetching all 6
    assert m.outputs == [0, 0] and m.state == 1
    assert r.run(m.step, m.restore, lambda: routes) == 0      # warm: no replay
    c2 = _cache(tmp_path, slots=12)
    with pytest.raises(RuntimeError):
        ReplayEngine(c2, fp_max=0).run(FakeModel(c2, routes).step, lambda: None, lambda: routes)


def _replay_rank(rank, world):
    import torch.distributed as dist
    st = make_store("pinned", L, E, SB)
    fill(st)
    c = ExpertCache(st, L, E, SB, 12, device="cpu", manager=False)
    if rank == 1:
        c.promote([(0, 0)])      # ranks start with different caches
        c.step_end()
    routes = [torch.tensor([0, 1]), torch.tensor([2]), torch.tensor([3 + rank])]   # rank-specific routing
    m = FakeModel(c, routes)
    r = ReplayEngine(c, tp_group=dist.group.WORLD, fp_max=4, comm_device="cpu")
    n = r.run(m.step, m.restore, lambda: routes)
    return n, sorted(map(tuple, (c.slot_table >= 0).nonzero().tolist()))


def test_replay_tp_consensus_gloo():
    (n0, res0), (n1, res1) = run_ranks(_replay_rank, 2)
    assert n0 == n1 == 1                       # both ranks replay the same number of times
    assert res0 == res1                        # and fetched the union of the missing sets
    assert (2, 3) in res0 and (2, 4) in res0


def test_confidence_gate_and_floors():
    g = ConfidenceGate(tau=0.5)
    sure = torch.tensor([[10.0, 0.0, 0.0]])
    unsure = torch.tensor([[1.0, 1.0, 0.9]])
    assert g.score(sure) > 0.99 and g.score(unsure) < 0.5
    calls = {"promote": 0, "restore": 0}
    logits = [unsure, sure]
    n = g.run(lambda: logits[min(calls["restore"], 1)], lambda: calls.__setitem__("restore", calls["restore"] + 1),
              lambda: [(0, 1)], lambda p: calls.__setitem__("promote", calls["promote"] + 1) or 1)
    assert n == 1 and calls == {"promote": 1, "restore": 1}
    gm = ConfidenceGate(tau=0.2, signal="margin", agg="q0.5")
    assert gm.score(torch.tensor([[5.0, 0.0], [0.0, 0.0]])) < 0.6
    assert working_set_floor(31, 8, 2, 1) == int(1.15 * 31 * 8 * 3 + 0.999)
    assert gate_fire_floor(31, 8, 3, 3) >= 31 * 8 * 3


def test_spec_guard_latch_and_resume():
    sg = SpecGuard(alpha=0.5, patience=4)
    allowed = [sg.observe(True) for _ in range(4)]
    assert allowed[-1] is False and sg.suppressed
    for _ in range(6):
        sg.observe(False)
    assert not sg.suppressed
    sg2 = SpecGuard(alpha=0.5, patience=2)
    for _ in range(20):
        sg2.observe(True)
    assert sg2.backoff > 1                     # suppression that does not warm the pool backs off


def test_prefetchers(tmp_path):
    c = _cache(tmp_path, slots=16)
    routers = [None, torch.eye(E)[:, :4].repeat(1, 1)[:E, :4].t().contiguous().float().repeat(1, 1), None]
    routers[1] = torch.randn(E, 4)
    lp = LookaheadPrefetcher(c, routers, top_k=2, extra=0)
    h = torch.randn(1, 4)
    want = {(1, int(e)) for e in torch.topk(h @ routers[1].t(), 2).indices.view(-1)}
    lp.step(0, h)
    assert all(c.resident(*p) for p in want)
    da = DraftAffinity(c)
    da.record([42], [torch.tensor([[5]]), None, torch.tensor([[6]])])
    assert da.prefetch([42]) == 2 and c.resident(0, 5) and c.resident(2, 6)


def test_floor_caps_at_expert_count():
    assert working_set_floor(3, 4, 2, 2, num_experts=16) == int(1.15 * 3 * 16 + 0.999)


def _pp_gate(rank, world, fail_rank):
    import torch.distributed as dist
    from vllm_moet_b200.residency import FetchError, pp_gate_barrier
    calls = []

    def promote():
        calls.append(rank)
        if rank == fail_rank:
            raise FetchError("injected promotion failure")
    # only the last stage's vote counts
    fire = (rank == world - 1)
    out = pp_gate_barrier(fire, promote, pp_group=dist.group.WORLD)
    return out, calls


def test_pp_gate_barrier_consensus_and_fail_closed():
    res = run_ranks(_pp_gate, 3, -1)
    assert all(o for o, _ in res) and all(c for _, c in res)     # every stage promoted and replays
    res = run_ranks(_pp_gate, 3, 1)
    assert not any(o for o, _ in res)                             # one failure -> nobody replays


def test_split_fp4_slot_roundtrip_and_register_decode():
    """Split-FP4 rows rebuild the exact MXFP4 values from the base codes + scales, and
    the device decode (restated per lane) yields the direct-8 registers of those values."""
    from vllm_moet_b200.formats import codebook, planes
    from vllm_moet_b200.residency.delta import dequant_split_slot, pack_split_slot, split_layout
    g = torch.Generator().manual_seed(3)
    H, I = 128, 64
    nib13 = torch.randint(0, 16, (2 * I, H), generator=g, dtype=torch.uint8)
    nib2 = torch.randint(0, 16, (H, I), generator=g, dtype=torch.uint8)
    sc13 = torch.randint(115, 135, (2 * I, H // 32), generator=g, dtype=torch.uint8)
    sc2 = torch.randint(115, 135, (H, I // 32), generator=g, dtype=torch.uint8)
    row = pack_split_slot(nib13, nib2)
    assert row.numel() == split_layout(H, I)[0] == (2 * I * H + H * I) * 5 // 16
    w13, w2 = dequant_split_slot(row, codebook.nibbles_to_codes(nib13), sc13, codebook.nibbles_to_codes(nib2), sc2,
                                 H, I)
    for w, nib, sc in ((w13, nib13, sc13), (w2, nib2, sc2)):
        N, K = nib.shape
        want = codebook.E2M1_VALUES[nib.long()].float().view(N, K // 32, 32) * torch.exp2(sc.float() - 127)[..., None]
        assert torch.equal(w, want.view(N, K))
    # per-lane device decode == direct-8 registers, every lane of every block of w13
    N, K = nib13.shape
    cp = planes.pack_codes(codebook.nibbles_to_codes(nib13))
    qp = planes.pack_quintal(nib13)
    d8 = planes.pack_direct8(planes.e2m1_to_e4m3_bytes(nib13))
    for blk in range((N // 16) * (K // 64)):
        for lane in range(32):
            cb = bytes(cp[blk * 256 + lane * 8: blk * 256 + lane * 8 + 8].tolist())
            rec = bytes(qp[blk * 320 + lane * 8: blk * 320 + lane * 8 + 8].tolist()) + \
                bytes(qp[blk * 320 + 256 + lane * 2: blk * 320 + 258 + lane * 2].tolist())
            A0, A1 = planes.quintal_lane_registers(cb, rec)
            got = b"".join(x.to_bytes(4, "little") for x in A0 + A1)
            assert list(got) == d8[blk * 1024 + lane * 32: blk * 1024 + lane * 32 + 32].tolist(), (blk, lane)
    for w in range(625):                      # the multiply-shift divide by 5 gives the base-5 digits
        t = planes.quintal_digit_word(w)
        d = [t & 0xF, (t >> 8) & 0xF, (t >> 4) & 0xF, (t >> 12) & 0xF]
        assert sum(di * 5 ** i for i, di in enumerate(d)) == w and max(d) < 5


def test_split_delta_coupling_protects_the_base(tmp_path):
    """A split-FP4 promotion makes the base resident first, and the base cache
    never evicts an expert that has a delta slot."""
    from vllm_moet_b200.residency.delta import DeltaTier, split_layout
    H = I = 64
    sbq = split_layout(H, I)[0]
    base = _cache(tmp_path, slots=4)
    rows = [torch.randint(0, 256, (E, sbq), dtype=torch.uint8) for _ in range(L)]
    delta = DeltaTier(rows, H, I, 3, device="cpu", policy="need", split=True)
    try:
        delta.couple(base)
        assert delta.promote([(0, 1), (1, 2)]) == 2
        assert base.resident(0, 1) and base.resident(1, 2) and delta.resident(0, 1)
        base.step_end(), delta.step_end()
        base.promote([(2, 0), (2, 1)])          # fills the base pool
        base.step_end()
        base.promote([(2, 2)])                  # must evict (2, 0) or (2, 1), never a coupled expert
        assert base.resident(0, 1) and base.resident(1, 2) and base.resident(2, 2)
        base.step_end()
        base.note_routed(2, [2])
        before = base.mirror.clone()
        with pytest.raises(FetchError):         # one unprotected, unpinned slot for two experts
            base.promote([(2, 3), (2, 4)])
        assert torch.equal(base.mirror, before)     # all or nothing: the victim taken first is restored
        for li in range(L):
            for e in range(E):
                assert int(base.slot_table[li, e]) == int(base.mirror[li, e])
    finally:
        delta.close()


def test_storm_invariants_hold_every_iteration(tmp_path):
    """Random promotions, manager-thread prefetches, routed pins, injected pack read
    faults and split-FP4 promotions over a tiered base cache; the residency
    invariants (pool bytes, mirror / owner / free / slot-table coherence, split
    coupling, store integrity) are checked after every iteration."""
    import random
    from vllm_moet_b200.residency.delta import DeltaTier, split_layout
    rnd = random.Random(1234)
    st = make_store("tiered", L, E, SB, dir=str(tmp_path), ckpt_id="storm", arena_rows=7)
    fill(st)
    base = ExpertCache(st, L, E, SB, 9, device="cpu", policy="freq", manager=True)
    H = I = 64
    sbq = split_layout(H, I)[0]
    drows = [torch.randint(0, 256, (E, sbq), generator=torch.Generator().manual_seed(50 + li), dtype=torch.uint8)
             for li in range(L)]
    delta = DeltaTier(drows, H, I, 4, device="cpu", policy="lru", split=True)
    delta.couple(base)
    failures = 0
    try:
        for it in range(150):
            base.step_begin()
            op = rnd.random()
            pairs = [(rnd.randrange(L), rnd.randrange(E)) for _ in range(rnd.randint(1, 4))]
            try:
                if op < 0.35:
                    base.promote(pairs)
                elif op < 0.55:
                    base.request_prefetch(pairs)
                elif op < 0.70:
                    delta.promote(pairs[:2])
                elif op < 0.80:
                    li = rnd.randrange(L)
                    base.ensure_resident(li, [rnd.randrange(E) for _ in range(3)])
                elif op < 0.90:
                    for li, e in pairs:
                        base.note_routed(li, [e])
                else:
                    st.inject_read_faults(rnd.choice([1, 2, 3]))
                    base.promote(pairs)
            except FetchError:
                failures += 1
            finally:
                st.inject_read_faults(0)
            assert base.wait_idle(10)
            base.step_end()
            delta.step_end()
            base.check_invariants(host_row=lambda li, e: layer_rows(li)[e])
            delta.check_invariants(host_row=lambda li, e: drows[li][e], base=base)
        for li in range(L):                      # store integrity after the storm
            got = st.rows_for(li, list(range(E)))
            assert not got.failed and all(torch.equal(r, layer_rows(li)[e]) for e, r in enumerate(got.rows))
        assert base.stats["evictions"] > 0 and delta.stats["fetched_rows"] > 0 and failures > 0
    finally:
        delta.close()
        base.close()
        st.release()


def _gate_tp(rank, world, fail_rank, empty_rank):
    import torch.distributed as dist
    from vllm_moet_b200.residency import FetchError, gate_promote_consensus

    def promote():
        if rank == fail_rank:
            raise FetchError("injected promotion failure")
        return 0 if rank == empty_rank else 3
    return gate_promote_consensus(promote, dist.group.WORLD)


def test_gate_promote_consensus_fail_safe():
    assert all(run_ranks(_gate_tp, 3, -1, -1))                  # everyone promoted -> everyone replays
    assert not any(run_ranks(_gate_tp, 3, 1, -1))               # one failed read -> nobody replays
    assert all(run_ranks(_gate_tp, 3, -1, 2))                   # nothing new on one rank still replays together
    from vllm_moet_b200.residency import gate_promote_consensus
    assert gate_promote_consensus(lambda: 2) and not gate_promote_consensus(lambda: 0)


def _replay_pp_stage(rank, world, fault_stage, base_dir):
    """Pipeline stages with their own layers' caches: stage 0's experts are resident,
    stage 1 misses.  Both stages replay the step together (and, with an injected read
    fault on one stage, both refuse to replay)."""
    import torch.distributed as dist
    st = make_store("pack", L, E, SB, dir=os.path.join(base_dir, f"stage{rank}"), ckpt_id="pp")
    fill(st)
    c = ExpertCache(st, L, E, SB, 12, device="cpu", manager=False)
    routes = [torch.tensor([0, 1]), torch.tensor([2]), torch.tensor([3])]
    if rank == 0:
        c.promote([(0, 0), (0, 1), (1, 2), (2, 3)])     # everything this stage routes is resident
        c.step_end()
    if rank == fault_stage:
        st.inject_read_faults(1)
    m = FakeModel(c, routes)
    r = ReplayEngine(c, pp_group=dist.group.WORLD, fp_max=4, comm_device="cpu")
    try:
        n = r.run(m.step, m.restore, lambda: routes)
        out = ("ok", n, len(m.outputs))
    except FetchError:
        out = ("refused", 0, len(m.outputs))
    finally:
        st.release()
    return out


def test_replay_pp_whole_pipeline_consensus(tmp_path):
    res = run_ranks(_replay_pp_stage, 2, -1, str(tmp_path / "a"))
    assert res[0] == res[1] == ("ok", 1, 2)           # stage 0 had no miss but replays with stage 1
    res = run_ranks(_replay_pp_stage, 2, 1, str(tmp_path / "b"))
    assert res[0][0] == res[1][0] == "refused"         # a failed read on stage 1: nobody replays


def test_gate_score_from_vocab_shards_is_exact():
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(5, 101, generator=g) * 3
    shards = torch.tensor_split(logits, 3, dim=1)
    parts = torch.stack([ConfidenceGate.row_stats(s) for s in shards])
    merged = ConfidenceGate.merge_stats(parts)
    assert torch.allclose(merged, ConfidenceGate.row_stats(logits), atol=1e-5)
    for sig in ("maxprob", "margin"):
        gt = ConfidenceGate(signal=sig)
        assert abs(gt.score_stats(merged) - gt.score(logits)) < 1e-6


def _gate_score_tp(rank, world):
    import torch.distributed as dist
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(4, 64, generator=g) * 2
    shard = torch.tensor_split(logits, world, dim=1)[rank]
    gt = ConfidenceGate(signal="margin", agg="q0.5")
    return gt.score(shard, tp_group=dist.group.WORLD), gt.score(logits)


def test_gate_score_tp_ranks_agree():
    res = run_ranks(_gate_score_tp, 3)
    assert all(abs(a - b) < 1e-6 for a, b in res) and len({round(a, 9) for a, _ in res}) == 1


def test_warm_state_dump_and_preload_across_boots(tmp_path):
    """Pool heat and the tiered arena's heat survive a restart: shutdown dumps both, the
    next boot preheats the arena and preloads the hottest experts into the cold pool; a
    first boot (no heat files) starts cold."""
    import types
    from vllm_moet_b200.config import MoetConfig
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.residency import ExpertCache, make_store
    L, E, SB = 2, 8, 512

    def boot():
        st = make_store("tiered", L, E, SB, dir=str(tmp_path), ckpt_id="ck", arena_rows=8)
        for li in range(L):
            if not st.has_layer(li):
                st.add_layer(li, torch.arange(E * SB, dtype=torch.int32).to(torch.uint8).view(E, SB) + li)
        cache = ExpertCache(st, L, E, SB, 6, device="cpu", manager=False)
        ns = types.SimpleNamespace(cache=cache, ecfg=types.SimpleNamespace(moet=MoetConfig()),
                                   mw=types.SimpleNamespace(tp_rank=0, tp_size=1))
        ns._heat_path = types.MethodType(LLM._heat_path, ns)
        return ns
    a = boot()
    LLM._warm_start(a, a.ecfg.moet)
    assert int((a.cache.slot_table >= 0).sum()) == 0                 # first boot: cold
    a.cache.promote([(0, 3), (1, 5), (1, 6)])
    a.cache.freq.zero_()
    a.cache.freq[0, 3], a.cache.freq[1, 5] = 9.0, 4.0
    LLM._dump_heat(a)
    assert os.path.exists(LLM._heat_path(a)) and os.path.exists(a.cache.store.heat_path)
    a.cache.store.release()
    b = boot()
    LLM._warm_start(b, b.ecfg.moet)
    assert b.cache.resident(0, 3) and b.cache.resident(1, 5)
    assert b.stats_warm["pool_experts"] >= 2 and b.stats_warm["arena_rows"] >= 1
    b.cache.store.release()
    # the knobs turn it off
    c = boot()
    c.ecfg.moet = MoetConfig(pool_heat=False, tier_preheat=False)
    LLM._warm_start(c, c.ecfg.moet)
    assert int((c.cache.slot_table >= 0).sum()) == 0
    c.cache.store.release()


def test_promotion_hysteresis_blocks_near_equal_displacement():
    """PROMO_HYST: with the delta pool full, a background (tick) candidate displaces a
    resident only when hotter than h x the weakest evictable resident + 4; mandatory
    promote() calls are never gated; h = 0 keeps the plain policy."""
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    H = I = 64
    sb = delta_layout(H, I)[0]
    for h, expect_blocked in ((1.25, True), (0.0, False)):
        rows = [torch.zeros(4, sb, dtype=torch.uint8) for _ in range(2)]
        t = DeltaTier(rows, H, I, 2, device="cpu", policy="freq", promo_hyst=h)
        try:
            t.promote([(0, 0), (0, 1)])
            t.step_end()
            t.freq.zero_()
            t.freq[0, 0], t.freq[0, 1] = 10.0, 10.0
            t.freq[1, 2] = 14.0                      # hotter, but < 1.25 x 10 + 4
            t.tick()
            t.step_end()
            assert t.resident(1, 2) != expect_blocked
            if expect_blocked:
                assert t.stats["hyst_blocked"] == 1
                t.freq[1, 2] = 20.0                  # > 16.5: displaces now
                t.tick()
                t.step_end()
                assert t.resident(1, 2)
                t.promote([(1, 3)])                  # mandatory: never gated
                assert t.resident(1, 3)
        finally:
            t.close()


def test_delta_pool_sizing_from_gib_or_auto():
    from vllm_moet_b200.residency.delta import delta_slots_for
    G = 1 << 30
    assert delta_slots_for("2", 1 << 20, 0) == 2048
    assert delta_slots_for("auto", 1 << 20, 10 * G, reserve_gb=3.0) == 7 * 1024
    assert delta_slots_for("auto", 1 << 20, 10 * G, reserve_gb=3.0, max_gb=1.5) == 1536
    assert delta_slots_for("auto", 1 << 20, 2 * G, reserve_gb=3.0) == 0
    with pytest.raises(ValueError):
        delta_slots_for("lots", 1 << 20, G)


def test_prefill_fp4_ensure_makes_the_chunk_fp4_resident(monkeypatch):
    """VLLM_MOE_W2_PREFILL_FP4=ensure: an eager prefill chunk makes its routed experts
    resident in the delta tier before the layer's experts run (the most-routed ones when
    the pool is smaller than the chunk's set); decode passes and mode 1 do not."""
    import types
    from vllm_moet_b200.config import MoetConfig
    from vllm_moet_b200.engine.gpu_runner import NativeRunner
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    H = I = 64
    sb = delta_layout(H, I)[0]
    delta = DeltaTier([torch.zeros(8, sb, dtype=torch.uint8) for _ in range(2)], H, I, 3, device="cpu",
                      policy="need")
    try:
        fake = types.SimpleNamespace(cache=None, delta=delta,
                                     ecfg=types.SimpleNamespace(moet=MoetConfig(prefill_fp4="ensure")))
        ids = torch.tensor([[1, 2], [1, 5], [1, 2], [6, 2]])
        NativeRunner._ensure_experts(fake, 0, ids, "decode")
        assert not any(delta.resident(0, e) for e in range(8))
        NativeRunner._ensure_experts(fake, 0, ids, "prefill")
        assert delta.resident(0, 1) and delta.resident(0, 2)           # the two most routed
        assert sum(delta.resident(0, e) for e in range(8)) == 3          # capped at the pool
        fake.ecfg.moet = MoetConfig(prefill_fp4="1")
        NativeRunner._ensure_experts(fake, 1, ids, "prefill")
        assert not any(delta.resident(1, e) for e in range(8))
    finally:
        delta.close()
    with pytest.raises(ValueError):
        MoetConfig(prefill_fp4="sometimes").validate()

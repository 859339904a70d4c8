"""Runtime-tunable knobs from files (GATE_TAU_FILE, GATE_MAX_PROMOTE_FILE,
BASE_MISS_TOL_FILE): re-read on change, default when missing, last good value on garbage,
and the gate / replay engine reading them."""
import os

from vllm_moet_b200.config import MoetConfig
from vllm_moet_b200.residency.control import ConfidenceGate
from vllm_moet_b200.utils.tunable import TunableFile, resolve, tunable


class Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t


def _write(path, text, bump):
    with open(path, "w") as f:
        f.write(text)
    st = os.stat(path)
    os.utime(path, ns=(st.st_atime_ns, st.st_mtime_ns + bump))      # a distinct mtime per edit


def test_tunable_file_semantics(tmp_path):
    p = str(tmp_path / "tau")
    clk = Clock()
    t = TunableFile(p, 0.6, float, interval=1.0, clock=clk, check=lambda v: 0 <= v <= 1)
    assert t.get() == 0.6                                  # missing file: the default
    _write(p, "0.25\n", 1)
    assert t.get() == 0.6                                  # not re-checked within the interval
    clk.t = 1.5
    assert t.get() == 0.25 and t.reloads == 1
    _write(p, "half", 2_000_000)                           # garbage: keep the last good value
    clk.t = 3.0
    assert t.get() == 0.25
    _write(p, "7.0", 4_000_000)                            # out of range: kept as well
    clk.t = 4.5
    assert t.get() == 0.25
    _write(p, "0.9", 6_000_000)
    clk.t = 6.0
    assert t.get() == 0.9 and t.reloads == 2
    os.remove(p)
    clk.t = 7.5
    assert t.get() == 0.6                                  # removed: back to the default
    assert tunable(3, None) == 3 and resolve(3) == 3 and isinstance(tunable(3, p), TunableFile)


def test_gate_reads_its_files_and_accepts_fixed_values(tmp_path):
    tau_f, mp_f = str(tmp_path / "tau"), str(tmp_path / "mp")
    _write(tau_f, "0.3", 1)
    _write(mp_f, "5", 1)
    g = ConfidenceGate(tau=0.6, max_promote=64, tau_file=tau_f, max_promote_file=mp_f)
    assert g.tau == 0.3 and g.max_promote == 5
    g.tau = 2.0                                            # a fixed value replaces the file
    assert g.tau == 2.0 and g.max_promote == 5


def test_replay_miss_tol_file(tmp_path):
    import torch
    from vllm_moet_b200.residency import ExpertCache, ReplayEngine, make_store
    st = make_store("pinned", 1, 4, 64)
    st.add_layer(0, torch.zeros(4, 64, dtype=torch.uint8))
    cache = ExpertCache(st, 1, 4, 64, 2, device="cpu", manager=False)
    f = str(tmp_path / "tol")
    _write(f, "3", 1)
    r = ReplayEngine(cache, mode="approximate", miss_tol=0, comm_device="cpu", miss_tol_file=f)
    assert r.miss_tol == 3
    r.miss_tol = 1
    assert r.miss_tol == 1


def test_env_aliases_of_the_files(monkeypatch):
    monkeypatch.setenv("VLLM_MOE_W2_GATE_TAU_FILE", "/tmp/tau")
    monkeypatch.setenv("VLLM_MOE_W2_BASE_MISS_TOL_FILE", "/tmp/tol")
    m = MoetConfig.from_env()
    assert m.gate_tau_file == "/tmp/tau" and m.base_miss_tol_file == "/tmp/tol" and m.gate_max_promote_file is None


def _scripted_replay(tmp_path, misses, **kw):
    import torch
    from vllm_moet_b200.residency import ExpertCache, ReplayEngine, make_store
    st = make_store("pinned", 1, 4, 64)
    st.add_layer(0, torch.zeros(4, 64, dtype=torch.uint8))
    cache = ExpertCache(st, 1, 4, 64, 2, device="cpu", manager=False)
    r = ReplayEngine(cache, comm_device="cpu", **kw)
    seq = iter(misses)

    def step():
        cache.miss_count += next(seq)
    return r, r.run(step, lambda: None, lambda: [None])


def test_approximate_replay_chases_only_within_fp_thresh(tmp_path):
    # beyond closing distance after the mandatory first replay: kept (working set moving)
    r, n = _scripted_replay(tmp_path, [5, 3], mode="approximate", fp_thresh=2, fp_max=8)
    assert n == 1 and r.stats["fp_giveup"] == 1
    # within closing distance: chased until miss-free
    r, n = _scripted_replay(tmp_path, [5, 3, 1, 0], mode="approximate", fp_thresh=4, fp_max=8)
    assert n == 3 and r.stats["second_order_replays"] == 2 and r.stats["fp_giveup"] == 0
    # within closing distance but never converging: fp_max, counted, no exception
    r, n = _scripted_replay(tmp_path, [2] * 10, mode="approximate", fp_thresh=4, fp_max=3)
    assert n == 3 and r.stats["fp_unfixed"] == 1
    # the threshold from a file
    f = str(tmp_path / "th")
    _write(f, "4", 1)
    r, n = _scripted_replay(tmp_path, [5, 3, 0], mode="approximate", fp_thresh=0, fp_thresh_file=f, fp_max=8)
    assert r.fp_thresh == 4 and n == 2
    # strict mode is untouched: every miss is chased, failing closed at fp_max
    import pytest
    with pytest.raises(RuntimeError):
        _scripted_replay(tmp_path, [2] * 10, mode="strict", fp_max=3)

"""DSpark's hardware-aware verify-length policy.

Each step the engine verifies every live request at a batch-uniform length L (a
captured shape); per-request widths (``dspark.allocate_widths``) then trim inside it.
L is chosen to maximise generated tokens per second:

    tokens(L) = R * (1 + accept[L])           accept[L] = sum of the first L calibrated
                                               prefix-survival probabilities
    time(L)   = T(R, L) + c0 + c1 * tokens(L)

* ``T(R, L)`` is a cost table measured at start-up on a grid of request counts R
  (:func:`profile_cost_table`); lookups round R up to the next grid bucket (the engine
  pads a batch to its bucket, so cost is a step function of R; interpolation would
  smooth over the cliff between buckets) and extrapolate linearly past the last one.
* ``c0 + c1 * tokens`` is the engine's own overhead (sampling, detokenising, host
  loop), which the table cannot see: each step's wall time minus the table's
  prediction is regressed on the step's token count over a ring of recent samples
  (least squares, c1 clamped to [0, 1e-3] s/token, c0 >= 0; residuals that are
  negative or above 0.25 s -- idle gaps -- are dropped).
* survival: an exponential moving average of the drafter's predicted per-position
  survival, times a per-position calibration ratio (realised / predicted acceptance
  over the positions actually verified at full width, clamped to [0.25, 4], blended
  slowly, updated only after enough observations).
* hysteresis: the incumbent L is kept unless a challenger beats its throughput by more
  than 5 %, so survival jitter cannot flap the shape; a change of R re-evaluates both.

:func:`derive_schedule` turns the cost table and a survival curve into a batch-size ->
L table with adjacent equal entries merged (dynamic speculative decoding), and
:class:`LiveRederivation` re-derives it from the acceptance actually measured.
Reference: the DSpark scheduler policy (patch P:19619-20013) and the dynamic-SD
derivation (P:18008-18145); the constants below are that policy's.
"""
from __future__ import annotations

import math
import time
from collections import deque
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from .dspark import allocate_widths

# prefix-survival prior (per draft position) used until acceptance has been measured
SURVIVAL_PRIOR = [0.78, 0.55, 0.37, 0.24, 0.16, 0.11, 0.08]
EMA_DECAY = 0.9
CAL_DECAY, CAL_MIN_OBS, CAL_RATIO = 0.8, 64.0, (0.25, 4.0)
RING, GATE_S, MIN_SAMPLES, C1_MAX = 129, 0.25, 16, 1e-3
HYSTERESIS = 0.05
PRIOR_C0, PRIOR_C1 = 0.003, 5e-5


def accept_curve(survival: Sequence[float], gamma: int) -> List[float]:
    """accept[L] = expected accepted drafts per request at verify length L (L = 0..gamma)."""
    out, run = [0.0], 0.0
    for j in range(gamma):
        run += min(float(survival[j]), 1.0) if j < len(survival) else 0.0
        out.append(run)
    return out


def bucket_cost(r_grid: Sequence[int], times: Sequence[float], num_reqs: int) -> float:
    """One table row's step time at `num_reqs` requests (see _step_times)."""
    return float(_step_times(r_grid, [times], num_reqs)[0])


def _step_times(r_grid: Sequence[int], times_by_l: Sequence[Sequence[float]], num_reqs: int) -> torch.Tensor:
    """Table step time of every L at `num_reqs` requests: column of the first grid bucket
    holding num_reqs, or the last column scaled by num_reqs / last bucket beyond the grid."""
    table = torch.as_tensor(times_by_l, dtype=torch.float64)          # [gamma + 1, len(r_grid)]
    grid = torch.as_tensor(r_grid, dtype=torch.int64)
    col = int(torch.searchsorted(grid, torch.tensor([num_reqs]), right=False))
    if col < len(r_grid):
        return table[:, col]
    return table[:, -1] * (num_reqs / r_grid[-1])


def uniform_length(accept: Sequence[float], num_reqs: int, gamma: int, r_grid: Optional[Sequence[int]],
                   times_by_l: Optional[Sequence[Sequence[float]]], overhead: Tuple[float, float] = (0.0, 0.0),
                   current: Optional[int] = None, hysteresis: float = HYSTERESIS) -> Tuple[int, float]:
    """-> (L maximising tokens / s, that L's predicted step time with overhead).
    Without a cost table: (gamma, 0).  Every L is scored at once: throughput(L) =
    tokens(L) / (T(R, L) + c0 + c1 tokens(L)); L with a non-positive table time is
    never chosen; ties go to the shorter L; the incumbent stays unless beaten by more
    than `hysteresis`."""
    if not r_grid or not times_by_l:
        return gamma, 0.0
    c0, c1 = overhead
    base = _step_times(r_grid, times_by_l, num_reqs)[: gamma + 1]
    tokens = num_reqs * (1.0 + torch.as_tensor(accept[: gamma + 1], dtype=torch.float64))
    total = base + c0 + c1 * tokens
    valid = base > 0
    if not bool(valid.any()):
        return gamma, 0.0
    rate = torch.where(valid, tokens / total, torch.full_like(total, -math.inf))
    best = int(torch.argmax(rate))             # argmax returns the first (shortest) maximum
    if current is not None and 0 <= current <= gamma and bool(valid[current]):
        if float(rate[best]) <= float(rate[current]) * (1.0 + hysteresis):
            best = current
    return best, float(total[best])


def derive_schedule(r_grid: Sequence[int], times_by_l: Sequence[Sequence[float]], survival: Sequence[float],
                    max_num_reqs: int, c0: float = PRIOR_C0, c1: float = PRIOR_C1) -> List[Tuple[int, int, int]]:
    """-> [(first R, last R, L)] covering 1..max_num_reqs, one entry per run of equal L."""
    gamma = len(times_by_l) - 1
    acc = accept_curve(survival, gamma)
    rows: List[list] = []
    lo = 1
    for i, r in enumerate(r_grid):
        hi = r if i < len(r_grid) - 1 else max(max_num_reqs, r)
        L, _ = uniform_length(acc, r, gamma, [r], [[times_by_l[k][i]] for k in range(gamma + 1)], (c0, c1))
        if rows and rows[-1][2] == L:
            rows[-1][1] = hi
        else:
            rows.append([lo, hi, L])
        lo = hi + 1
    return [tuple(x) for x in rows]


def schedule_lookup(table: Sequence[Tuple[int, int, int]], max_num_reqs: int, gamma: int) -> List[int]:
    """Dense lookup: out[R] = L for R = 0..max_num_reqs (R = 0 maps to gamma)."""
    out = [gamma] * (max_num_reqs + 1)
    for lo, hi, L in table:
        for r in range(max(lo, 1), min(hi, max_num_reqs) + 1):
            out[r] = min(L, gamma)
    return out


class LiveRederivation:
    """Re-derives the batch-size -> L table from measured per-position acceptance every
    `every` verified requests (positions with at least `min_obs` observations replace
    their prior; counts then halve, so the estimate tracks drift)."""

    def __init__(self, r_grid, times_by_l, max_num_reqs: int, every: int = 16384, min_obs: float = 512.0):
        self.r_grid, self.times_by_l, self.max_num_reqs = list(r_grid), [list(t) for t in times_by_l], max_num_reqs
        self.gamma = len(times_by_l) - 1
        self.every, self.min_obs = every, min_obs
        self.survival = list(SURVIVAL_PRIOR[: self.gamma])
        while len(self.survival) < self.gamma:
            self.survival.append(self.survival[-1] * 0.7 if self.survival else 0.5)
        self.obs = [0.0] * self.gamma
        self.acc = [0.0] * self.gamma
        self.n = 0

    def observe(self, drafted: int, accepted: int) -> Optional[List[int]]:
        for j in range(min(drafted, self.gamma)):
            self.obs[j] += 1
        for j in range(min(accepted, drafted, self.gamma)):
            self.acc[j] += 1
        self.n += 1
        if self.n < self.every:
            return None
        self.n = 0
        for j in range(self.gamma):
            if self.obs[j] >= self.min_obs:
                self.survival[j] = self.acc[j] / self.obs[j]
            self.obs[j] *= 0.5
            self.acc[j] *= 0.5
        table = derive_schedule(self.r_grid, self.times_by_l, self.survival, self.max_num_reqs)
        return schedule_lookup(table, self.max_num_reqs, self.gamma)


class DSparkPolicy:
    """Per-step verify-length choice and per-request widths (host-side, synchronous)."""

    def __init__(self, gamma: int, tau: float = 0.0, budget_frac: float = 1.0,
                 clock: Callable[[], float] = time.perf_counter):
        self.gamma, self.tau, self.budget_frac, self.clock = gamma, tau, budget_frac, clock
        self.r_grid: Optional[List[int]] = None
        self.times_by_l: Optional[List[List[float]]] = None
        self.c0 = self.c1 = 0.0
        self.samples: "deque[Tuple[float, float]]" = deque()
        self._sums = [0.0, 0.0, 0.0, 0.0]        # running sums of x, y, x*x, x*y over `samples`
        self.ema: Optional[torch.Tensor] = None
        self.cal = torch.ones(gamma)
        self.acc = torch.zeros(gamma)
        self.obs = torch.zeros(gamma)
        self.pred = torch.zeros(gamma)
        self._cal_base = (torch.zeros(gamma), torch.zeros(gamma), torch.zeros(gamma))
        self.current: Optional[int] = None
        self._t_last: Optional[float] = None
        self._gpu_pred = 0.0
        self._tokens = 0.0
        self.history: List[int] = []

    def set_cost_table(self, r_grid: Sequence[int], times_by_l: Sequence[Sequence[float]]) -> None:
        if len(times_by_l) != self.gamma + 1 or any(len(t) != len(r_grid) for t in times_by_l):
            raise ValueError("cost table: gamma + 1 rows of len(r_grid) step times")
        self.r_grid, self.times_by_l = list(r_grid), [list(map(float, t)) for t in times_by_l]

    # -------------------------------------------------------------- overhead regression
    def _observe_overhead(self, now: float) -> None:
        """Fit the engine overhead o = c0 + c1 * tokens to the last RING steps.  Running
        sums of x, y, x^2 and xy over the ring are updated as samples enter and leave, so
        each step costs O(1); the fit is the closed-form least-squares line through them."""
        if self._t_last is not None and self._gpu_pred > 0:
            o = (now - self._t_last) - self._gpu_pred
            if 0.0 <= o < GATE_S:
                self._fit_add(self._tokens, o)
                n = len(self.samples)
                if n >= MIN_SAMPLES:
                    sx, sy, sxx, sxy = self._sums
                    sxx_c = sxx - sx * sx / n           # sum of squared deviations of x
                    if sxx_c > 1e-6:
                        slope = (sxy - sx * sy / n) / sxx_c
                        self.c1 = min(max(slope, 0.0), C1_MAX)
                    self.c0 = max(sy / n - self.c1 * sx / n, 0.0)
        self._t_last = now

    def _fit_add(self, x: float, y: float) -> None:
        if len(self.samples) == RING:
            ox, oy = self.samples.popleft()
            self._sums = [a - b for a, b in zip(self._sums, (ox, oy, ox * ox, ox * oy))]
        self.samples.append((x, y))
        self._sums = [a + b for a, b in zip(self._sums, (x, y, x * x, x * y))]

    def survival_curve(self) -> Optional[List[float]]:
        if self.ema is None:
            return None
        return [min(float(s) * float(c), 1.0) for s, c in zip(self.ema, self.cal)]

    def begin_step(self, num_reqs: int, now: Optional[float] = None) -> int:
        """-> this step's uniform verify length L (0..gamma)."""
        self._observe_overhead(self.clock() if now is None else now)
        L = self.gamma
        curve = self.survival_curve()
        if curve is not None and self.r_grid:
            acc = accept_curve(curve, self.gamma)
            L, pred = uniform_length(acc, num_reqs, self.gamma, self.r_grid, self.times_by_l, (self.c0, self.c1),
                                     self.current)
            self._tokens = num_reqs * (1.0 + acc[L])
            self._gpu_pred = pred - (self.c0 + self.c1 * self._tokens)
        else:
            self._gpu_pred = 0.0
        self.current = L
        self.history.append(L)
        return L

    def allocate(self, survival: torch.Tensor, num_reqs: int, length: int) -> torch.Tensor:
        return allocate_widths(survival, self.cal, num_reqs, length, self.tau, self.budget_frac)

    # -------------------------------------------------------------- survival and calibration
    def observe(self, survival: torch.Tensor, widths: torch.Tensor, accepted: torch.Tensor, length: int) -> None:
        """After a verify: survival [R, gamma] predicted for the step's drafts, widths [R]
        verified, accepted [R] drafts accepted.  A position j (1-based) of request r counts
        as observed when r was verified at the step's full length and j <= its width."""
        s = survival.detach().float().cpu()
        m = s.mean(0)
        self.ema = m.clone() if self.ema is None else self.ema * EMA_DECAY + m * (1 - EMA_DECAY)
        if length <= 0:
            return
        w, a = widths.cpu().long(), accepted.cpu().long()
        j = torch.arange(1, self.gamma + 1)
        seen = (w[:, None] >= j[None, :]) & (w[:, None] == length)
        self.obs += seen.sum(0).float()
        self.acc += ((a[:, None] >= j[None, :]) & seen).sum(0).float()
        self.pred += (s * seen.float()).sum(0)
        o0, a0, p0 = self._cal_base
        d_obs, d_acc, d_pred = self.obs - o0, self.acc - a0, self.pred - p0
        upd = (d_obs >= CAL_MIN_OBS) & (d_pred > 1e-3)
        if bool(upd.any()):
            ratio = (d_acc / d_pred.clamp_min(1e-3)).clamp(*CAL_RATIO)
            self.cal = torch.where(upd, CAL_DECAY * self.cal + (1 - CAL_DECAY) * ratio, self.cal)
            self._cal_base = (torch.where(upd, self.obs, o0), torch.where(upd, self.acc, a0),
                              torch.where(upd, self.pred, p0))


def profile_cost_table(step: Callable[[int, int], None], r_grid: Sequence[int], gamma: int, repeats: int = 3,
                       sync: Optional[Callable[[], None]] = None,
                       clock: Callable[[], float] = time.perf_counter) -> List[List[float]]:
    """times_by_l[L][i] = median seconds of `step(r_grid[i], L)` (one verify step of R
    requests at length L), after one warm-up call per shape."""
    out = []
    for L in range(gamma + 1):
        row = []
        for R in r_grid:
            step(R, L)
            ts = []
            for _ in range(repeats):
                if sync:
                    sync()
                t0 = clock()
                step(R, L)
                if sync:
                    sync()
                ts.append(clock() - t0)
            row.append(sorted(ts)[len(ts) // 2])
        out.append(row)
    return out

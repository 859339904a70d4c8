"""Runtime-tunable knobs: a value read from a one-line text file and re-read when the file
changes, so an operator can retune a serving process without restarting it.

The reference reads ``VLLM_MOE_W2_GATE_TAU_FILE``, ``_GATE_MAX_PROMOTE_FILE`` and
``_BASE_MISS_TOL_FILE`` through mtime-cached file reads (patch P:9884-9904, P:9936-9950,
P:11489-11502); the same knobs here are ``MoetConfig.gate_tau_file`` /
``gate_max_promote_file`` / ``base_miss_tol_file`` (those env names are aliases).

``TunableFile.get()`` stats the file at most once per ``interval`` seconds and parses it
again only when its (mtime, size) changed.  A missing file gives the default; a file
that does not parse keeps the last good value (and logs once per bad version), so a
half-written edit never changes the knob to garbage.
"""
from __future__ import annotations

import logging
import os
import time
from typing import Any, Callable, Optional

log = logging.getLogger("vllm_moet_b200")


class TunableFile:
    def __init__(self, path: str, default: Any, parse: Callable[[str], Any] = float, interval: float = 0.5,
                 clock: Callable[[], float] = time.monotonic,
                 check: Optional[Callable[[Any], bool]] = None):
        self.path, self.default, self.parse = path, default, parse
        self.interval, self.clock, self.check = float(interval), clock, check
        self.value = default
        self._stamp = None          # (mtime_ns, size) of the version parsed last
        self._next = -float("inf")  # clock time of the next stat
        self.reloads = 0

    def get(self) -> Any:
        now = self.clock()
        if now < self._next:
            return self.value
        self._next = now + self.interval
        try:
            st = os.stat(self.path)
        except OSError:
            if self._stamp is not None:
                log.info("tunable %s removed: back to the default %r", self.path, self.default)
            self.value, self._stamp = self.default, None
            return self.value
        stamp = (st.st_mtime_ns, st.st_size)
        if stamp == self._stamp:
            return self.value
        self._stamp = stamp
        try:
            with open(self.path) as f:
                v = self.parse(f.read().strip())
            if self.check is not None and not self.check(v):
                raise ValueError(f"{v!r} out of range")
        except (OSError, ValueError) as e:
            log.warning("tunable %s: keeping %r (%s)", self.path, self.value, e)
            return self.value
        if v != self.value:
            log.info("tunable %s: %r -> %r", self.path, self.value, v)
        self.value = v
        self.reloads += 1
        return self.value


def tunable(value, path: Optional[str], parse=float, check=None):
    """``path`` set: a TunableFile defaulting to ``value``; else ``value`` itself."""
    return TunableFile(path, value, parse, check=check) if path else value


def resolve(v):
    """The current value of a knob that may be a TunableFile."""
    return v.get() if isinstance(v, TunableFile) else v

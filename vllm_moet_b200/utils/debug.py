"""Debug proxy around the native module: after every call, synchronise and
raise at the first kernel that set the device status word or wrote
non-finite floats into one of its tensor arguments (eager runs only)."""
from __future__ import annotations

import torch


class CheckedNative:
    def __init__(self, mod, status: torch.Tensor):
        self._mod = mod
        self._status = status
        self.calls = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def wrapped(*args, **kw):
            out = fn(*args, **kw)
            self.calls += 1
            torch.cuda.synchronize()
            code = int(self._status.item())
            if code:
                raise RuntimeError(f"status {code} after native call #{self.calls} {name}")
            skip = {"mla_decode": {6}}.get(name, set())  # m = -inf marks an empty split
            for i, a in enumerate(args):
                if i in skip:
                    continue
                if isinstance(a, torch.Tensor) and a.is_floating_point() and a.numel():
                    if not bool(torch.isfinite(a.float()).all()):
                        bad = (~torch.isfinite(a.float())).reshape(a.shape[0], -1).any(-1).nonzero().flatten()
                        raise FloatingPointError(f"non-finite arg {i} {tuple(a.shape)} after native call "
                                                 f"#{self.calls} {name}; rows {bad[:8].tolist()} of {bad.numel()}")
            return out
        return wrapped

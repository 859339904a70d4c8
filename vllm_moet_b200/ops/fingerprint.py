"""Native source fingerprint: sha256 over every file under csrc/ (sorted by
path).  setup.py compiles the same digest into the extension
(``_C.source_fingerprint``); :func:`check_build` compares the two so that a
stale build -- sources changed since the .so was made -- fails loudly
instead of silently running old kernels (the role of the reference's patch
guard, tools/check_patch_files.py, for this repository's native code)."""
from __future__ import annotations

import hashlib
import os

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def source_fingerprint(root: str = ROOT) -> str:
    h = hashlib.sha256()
    base = os.path.join(root, "csrc")
    if not os.path.isdir(base):
        return "no-sources"
    for d, _, files in sorted(os.walk(base)):
        for fn in sorted(files):
            if not fn.endswith((".cu", ".cuh", ".cpp", ".h")):
                continue
            p = os.path.join(d, fn)
            h.update(os.path.relpath(p, root).encode())
            with open(p, "rb") as f:
                h.update(hashlib.sha256(f.read()).digest())
    return h.hexdigest()[:32]


def check_build(mod) -> None:
    built = getattr(mod, "source_fingerprint", None)
    if built is None or os.environ.get("MOET_SKIP_BUILD_CHECK") == "1":
        return
    now = source_fingerprint()
    if now != "no-sources" and built != now:
        raise RuntimeError(f"vllm_moet_b200._C is stale: built from sources {built}, tree has {now}; "
                           "rebuild with `python setup.py build_ext --inplace` (MOET_SKIP_BUILD_CHECK=1 overrides)")

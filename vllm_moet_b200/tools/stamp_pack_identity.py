"""Stamp existing expert packs with a checkpoint identity, so a restart reuses them.

    python -m vllm_moet_b200.tools.stamp_pack_identity --store-dir DIR \\
        (--checkpoint CKPT_DIR | --ckpt-id ID) [--force] [--dry-run]

A pack store keys its files by the checkpoint identity, the quantizer ABI and the
zero-code mode (``residency/stores.py::pack_paths``).  A pack written without an
identity (its sidecar says ``ckpt_id: null``) lives under a process-local name and is
never reused.  For packs an operator knows were written from a given checkpoint, this
tool records the identity in the sidecar and moves the pack and sidecar to the names the
store computes for that identity -- the next boot finds them instead of rebuilding.

It refuses a sidecar that already names a DIFFERENT checkpoint (that directory served
another model: rebuild instead) unless ``--force``, and always refuses one whose
quantizer ABI or zero-code mode differs from this build's (its bytes would be read
wrongly).  (Reference: tools/stamp_pack_identity.py, the same operator workflow for its
pack sidecars.)
"""
from __future__ import annotations

import argparse
import os
import re
import sys
from typing import List

from ..residency.fsutil import atomic_write_json, read_json
from ..residency.identity import checkpoint_id, identity_fields
from ..residency.stores import pack_paths

_NAME = re.compile(r"^(?P<tag>.+)\.v2\.(?P<h>[0-9a-f]{20})\.(?P<suffix>.+)\.json$")


def stamp(store_dir: str, ckpt_id: str, force: bool = False, dry_run: bool = False) -> List[dict]:
    """-> one record per sidecar: {"sidecar", "action" (stamped | current | refused),
    "reason"}."""
    out = []
    cur = identity_fields(ckpt_id)
    for fn in sorted(os.listdir(store_dir)):
        m = _NAME.match(fn)
        if not m:
            continue
        side = os.path.join(store_dir, fn)
        meta = read_json(side)
        rec = {"sidecar": fn}
        if meta is None:
            out.append(dict(rec, action="refused", reason="unreadable sidecar"))
            continue
        if meta.get("quantizer_abi") != cur["quantizer_abi"] or meta.get("zero_mode") != cur["zero_mode"]:
            out.append(dict(rec, action="refused", reason="quantizer ABI / zero mode differ from this build"))
            continue
        old = meta.get("ckpt_id")
        if old == ckpt_id:
            out.append(dict(rec, action="current", reason=""))
            continue
        if old is not None and not force:
            out.append(dict(rec, action="refused", reason=f"names another checkpoint ({old}); --force to override"))
            continue
        pack_old = side[:-len(".json")] + ".pack"
        new_pack, new_side, new_lock, _ = pack_paths(store_dir, meta["tag"], int(meta["n_layers"]), int(meta["E"]),
                                                     int(meta["slot_bytes"]), ckpt_id, m.group("suffix"))
        if os.path.exists(new_side) and os.path.abspath(new_side) != os.path.abspath(side):
            out.append(dict(rec, action="refused", reason=f"{os.path.basename(new_side)} exists"))
            continue
        if not dry_run:
            if os.path.exists(pack_old):
                os.replace(pack_old, new_pack)
            atomic_write_json(new_side, dict(meta, ckpt_id=ckpt_id))
            if os.path.abspath(new_side) != os.path.abspath(side):
                os.remove(side)
            lock_old = side[:-len(".json")] + ".lock"
            if os.path.exists(lock_old) and os.path.abspath(lock_old) != os.path.abspath(new_lock):
                os.remove(lock_old)
        out.append(dict(rec, action="stamped", reason=os.path.basename(new_side)))
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--store-dir", required=True)
    g = ap.add_mutually_exclusive_group(required=True)
    g.add_argument("--checkpoint", help="checkpoint directory (its identity is computed as the server does)")
    g.add_argument("--ckpt-id", help="identity string (as MOET_CKPT_ID would give)")
    ap.add_argument("--force", action="store_true", help="overwrite an identity naming another checkpoint")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    cid = a.ckpt_id or checkpoint_id(model_path=a.checkpoint)
    if cid is None:
        print("no identity: not a checkpoint directory", file=sys.stderr)
        return 2
    recs = stamp(a.store_dir, cid, a.force, a.dry_run)
    for r in recs:
        print(f"{r['action']:8s} {r['sidecar']} {r['reason']}")
    return 1 if any(r["action"] == "refused" for r in recs) else 0


if __name__ == "__main__":
    sys.exit(main())

"""Stamping an identity-less pack with a checkpoint identity: the store opened with that
identity finds the written layers (same bytes); a pack naming another checkpoint is
refused unless forced; an already-stamped pack is left alone."""
import os

import torch

from vllm_moet_b200.residency.stores import MmapPackStore
from vllm_moet_b200.tools.stamp_pack_identity import main, stamp


def _write(d, ckpt_id):
    st = MmapPackStore(str(d), "experts", 2, 4, 256, ckpt_id=ckpt_id)
    rows = torch.arange(4 * 256, dtype=torch.int32).to(torch.uint8).view(4, 256)
    st.add_layer(1, rows)
    st.release()
    return rows


def test_stamp_makes_the_pack_reusable(tmp_path):
    rows = _write(tmp_path, None)
    assert not MmapPackStore(str(tmp_path), "experts", 2, 4, 256, ckpt_id="ckpt:abc").has_layer(1)
    recs = stamp(str(tmp_path), "ckpt:abc")
    assert [r["action"] for r in recs] == ["stamped"]
    st = MmapPackStore(str(tmp_path), "experts", 2, 4, 256, ckpt_id="ckpt:abc")
    assert st.has_layer(1) and not st.has_layer(0)
    got = st.rows_for(1, [0, 3])
    assert torch.equal(got.rows[0], rows[0]) and torch.equal(got.rows[1], rows[3])
    st.release()
    assert [r["action"] for r in stamp(str(tmp_path), "ckpt:abc")] == ["current"]
    assert len([f for f in os.listdir(tmp_path) if f.endswith(".json")]) == 1


def test_stamp_refuses_another_checkpoint_unless_forced(tmp_path):
    _write(tmp_path, "ckpt:other")
    assert [r["action"] for r in stamp(str(tmp_path), "ckpt:abc")] == ["refused"]
    assert main(["--store-dir", str(tmp_path), "--ckpt-id", "ckpt:abc"]) == 1
    assert [r["action"] for r in stamp(str(tmp_path), "ckpt:abc", force=True)] == ["stamped"]
    assert MmapPackStore(str(tmp_path), "experts", 2, 4, 256, ckpt_id="ckpt:abc").has_layer(1)

"""Inter-host pipeline-parallel prototype: a model split into stages on different
hosts, activations over plain TCP with an injectable WAN round-trip time.

This measures the mechanics of serving across hosts, not a performance build:
every stage runs its layer range with the reference (eager) layer code, there is
no CUDA graph and no speculation.  Per generated token the driver reports
``stage compute`` (the sum of every stage's own layer time, carried back in the
replies) and ``link`` (the rest of the round trip), which is the term the
prototype exists to validate.  Reference: ``tools/pp_proto_exl3.py`` (patch
P:1491-1735) -- there two stages of DS4-Flash with EXL3-served experts; here
any number of stages of any preset, experts from the 2-bit planes or, with
``--trellis-pack``, from the trellis (EXL3-style) base tier.

Wire format (no pickle: a peer's bytes are never executed): one frame is
``u64 total | u32 header bytes | JSON header | tensor bytes``; the header lists
each tensor as ``{"name", "dtype", "shape", "nbytes"}`` in payload order, so
bf16 activations cross the link bit-exactly as raw bytes.

Chain: stage 0 (embedding + first layers) drives; stage ``s > 0`` listens on
its port and, unless it is last, connects to stage ``s + 1``; the last stage
applies the final norm and the head and answers with the greedy token; the
answer travels back along the chain.

    # the last stage first (listens), then the middle ones, then the driver
    python -m vllm_moet_b200.parallel.interhost_pp --stage 1 --stages 2 --port 29777 --rtt-ms 46.6
    python -m vllm_moet_b200.parallel.interhost_pp --stage 0 --stages 2 --peer 127.0.0.1:29777 \\
        --rtt-ms 46.6 --new-tokens 48
"""
from __future__ import annotations

import argparse
import json
import socket
import struct
import time
from typing import Dict, List, Optional, Tuple

import torch

from ..config import ModelConfig, get_preset
from ..models import reference as ref
from ..models.weights import random_weights

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16,
           "int32": torch.int32, "int64": torch.int64, "uint8": torch.uint8}
MAX_FRAME = 1 << 34          # refuse absurd lengths from a broken peer


# ------------------------------------------------------------------ framing
def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(min(1 << 20, n - len(buf)))
        if not chunk:
            raise ConnectionError("peer closed the connection")
        buf += chunk
    return bytes(buf)


def send_frame(sock: socket.socket, header: dict, tensors: Optional[Dict[str, torch.Tensor]] = None,
               one_way_s: float = 0.0) -> int:
    """-> bytes sent.  `one_way_s` is the injected one-way link delay."""
    specs, blobs = [], []
    for name, t in (tensors or {}).items():
        t = t.detach().contiguous().cpu()
        dt = str(t.dtype).replace("torch.", "")
        if dt not in _DTYPES:
            raise TypeError(f"unsupported tensor dtype {t.dtype}")
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        specs.append({"name": name, "dtype": dt, "shape": list(t.shape), "nbytes": len(raw)})
        blobs.append(raw)
    head = json.dumps(dict(header, tensors=specs)).encode()
    body = struct.pack("<I", len(head)) + head + b"".join(blobs)
    if one_way_s > 0:
        time.sleep(one_way_s)
    sock.sendall(struct.pack("<Q", len(body)) + body)
    return 8 + len(body)


def recv_frame(sock: socket.socket) -> Tuple[dict, Dict[str, torch.Tensor]]:
    (n,) = struct.unpack("<Q", _recv_exact(sock, 8))
    if n > MAX_FRAME:
        raise ValueError(f"frame of {n} bytes refused")
    body = _recv_exact(sock, n)
    (hn,) = struct.unpack("<I", body[:4])
    header = json.loads(body[4:4 + hn].decode())
    off, tensors = 4 + hn, {}
    for spec in header.pop("tensors", []):
        dt = _DTYPES[spec["dtype"]]
        raw = bytearray(body[off:off + spec["nbytes"]])
        off += spec["nbytes"]
        t = torch.frombuffer(raw, dtype=torch.uint8) if raw else torch.empty(0, dtype=torch.uint8)
        tensors[spec["name"]] = t.view(dt).reshape(spec["shape"]) if raw else torch.empty(spec["shape"], dtype=dt)
    return header, tensors


# ------------------------------------------------------------------ stages
class Stage:
    """Layers [lo, hi) of a `stages`-way split (the engine's PP layer ranges)."""

    def __init__(self, cfg: ModelConfig, stage: int, stages: int, device="cpu", seed: int = 0,
                 max_pos: int = 4096, trellis_pack: Optional[str] = None):
        self.cfg, self.stage, self.stages = cfg, stage, stages
        self.dev = torch.device(device)
        self.mw = random_weights(cfg, self.dev, seed=seed, with_mtp=False, pp_rank=stage, pp_size=stages)
        self.lo, self.hi = self.mw.extra["layer_range"]
        self.moe_fn = None
        if trellis_pack:            # this stage's MoE layers from the trellis packs (global layer ids)
            import os
            from ..residency.trellis_tier import TrellisBaseTier, pack_path
            mine = [self.lo + i for i, lw in enumerate(self.mw.layers)
                    if lw.is_moe and os.path.exists(pack_path(trellis_pack, self.lo + i))]
            if mine:
                tier = TrellisBaseTier(trellis_pack, mine, device=self.dev, act_limit=cfg.swiglu_limit)
                self.moe_fn = tier.moe_fn(self.mw, layer_offset=self.lo)
        self.first, self.last = stage == 0, stage == stages - 1
        self.cs = ref.rope_cos_sin(cfg, max_pos, self.dev)
        self.reset()

    def reset(self):
        self.cache = ref.RefKV(self.hi - self.lo)

    @torch.inference_mode()
    def run(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """First stage: x = token ids [T]; others: x = hidden [T, H] (bf16 on the wire).
        -> hidden [T, H] bf16 (the tensor that crosses the link)."""
        h = self.mw.embed[x.to(self.dev).long()].float() if self.first else x.to(self.dev).float()
        if self.first and self.cfg.hc_mult > 1:           # hyper-connections: [T, n, H] streams on the wire
            h = h[:, None, :].expand(-1, self.cfg.hc_mult, -1)
        pos = positions.to(self.dev)
        import contextlib
        with ref.moe_context(self.moe_fn) if self.moe_fn is not None else contextlib.nullcontext():
            for i, lw in enumerate(self.mw.layers):
                h = ref.decoder_layer(self.cfg, lw, h, pos, self.cs, self.cache, i)
        return h.to(torch.bfloat16)

    @torch.inference_mode()
    def head(self, h: torch.Tensor) -> int:
        h = h[-1:].float()
        if self.cfg.hc_mult > 1:
            h = ref.hc_head(self.cfg, self.mw.extra["hc_head"], h)
        x = ref.rms_norm(h, self.mw.final_norm, self.cfg.rms_eps)
        return int((x @ self.mw.lm_head.dequant().t()).argmax(-1))


def serve_stage(st: Stage, listener: socket.socket, next_addr: Optional[Tuple[str, int]] = None,
                rtt_ms: float = 0.0) -> None:
    """Stage s > 0: answer one driver connection until it sends "stop"."""
    ow = rtt_ms / 2000.0
    conn, _ = listener.accept()
    conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    nxt = None
    if next_addr is not None:
        nxt = socket.create_connection(next_addr)
        nxt.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    try:
        while True:
            hdr, ts = recv_frame(conn)
            if hdr.get("op") == "stop":
                if nxt is not None:
                    send_frame(nxt, {"op": "stop"}, None, ow)
                return
            if hdr.get("op") == "reset":
                st.reset()
                if nxt is not None:
                    send_frame(nxt, hdr, None, ow)
                    recv_frame(nxt)
                send_frame(conn, {"op": "ok"}, None, ow)
                continue
            t0 = time.perf_counter()
            h = st.run(ts["h"], torch.tensor(hdr["positions"]))
            if st.dev.type == "cuda":
                torch.cuda.synchronize(st.dev)
            own_ms = (time.perf_counter() - t0) * 1e3
            if nxt is not None:
                send_frame(nxt, hdr, {"h": h}, ow)
                reply, _ = recv_frame(nxt)
            else:
                t1 = time.perf_counter()
                reply = {"token": st.head(h), "compute_ms": []}
                own_ms += (time.perf_counter() - t1) * 1e3
            reply["compute_ms"] = [own_ms] + list(reply.get("compute_ms", []))
            send_frame(conn, reply, None, ow)
    finally:
        conn.close()
        if nxt is not None:
            nxt.close()


class Driver:
    """Stage 0: embeds, runs its layers, ships the hidden state down the chain."""

    def __init__(self, st: Stage, peer: Tuple[str, int], rtt_ms: float = 0.0):
        self.st, self.ow = st, rtt_ms / 2000.0
        self.sock = socket.create_connection(peer)
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self.bytes_sent = 0

    def _step(self, ids: List[int], start: int) -> Tuple[int, List[float], float]:
        t0 = time.perf_counter()
        pos = torch.arange(start, start + len(ids))
        h = self.st.run(torch.tensor(ids), pos)
        if self.st.dev.type == "cuda":
            torch.cuda.synchronize(self.st.dev)
        own_ms = (time.perf_counter() - t0) * 1e3
        self.bytes_sent += send_frame(self.sock, {"op": "fwd", "positions": pos.tolist()}, {"h": h}, self.ow)
        reply, _ = recv_frame(self.sock)
        total_ms = (time.perf_counter() - t0) * 1e3
        return int(reply["token"]), [own_ms] + reply["compute_ms"], total_ms

    def generate(self, prompt: List[int], new_tokens: int) -> dict:
        """Greedy: one prefill round trip, then one round trip per token."""
        self.st.reset()
        send_frame(self.sock, {"op": "reset"}, None, self.ow)
        recv_frame(self.sock)
        tok, comp, total = self._step(prompt, 0)
        out, per_tok = [tok], []
        prefill = {"total_ms": total, "compute_ms": sum(comp)}
        for i in range(new_tokens - 1):
            tok, comp, total = self._step([tok], len(prompt) + i)
            out.append(tok)
            per_tok.append((total, sum(comp)))
        n = max(1, len(per_tok))
        tot = sum(t for t, _ in per_tok) / n
        cmp_ = sum(c for _, c in per_tok) / n
        return {"tokens": out, "prefill": prefill, "per_token_ms": tot, "stage_compute_ms": cmp_,
                "link_ms": tot - cmp_, "tok_s": 1000.0 / tot if per_tok else 0.0,
                "hidden_bytes_per_token": self.st.cfg.hidden * 2}

    def close(self):
        try:
            send_frame(self.sock, {"op": "stop"}, None, 0.0)
        finally:
            self.sock.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description="inter-host pipeline-parallel prototype")
    ap.add_argument("--stage", type=int, required=True)
    ap.add_argument("--stages", type=int, default=2)
    ap.add_argument("--model", default="tiny-moe")
    ap.add_argument("--num-layers", type=int, default=None)
    ap.add_argument("--hc-mult", type=int, default=None, help="hyper-connection streams (model default)")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--port", type=int, default=29777, help="stage > 0: port to listen on")
    ap.add_argument("--next", default=None, help="stage > 0, not last: host:port of the next stage")
    ap.add_argument("--peer", default="127.0.0.1:29777", help="stage 0: host:port of stage 1")
    ap.add_argument("--rtt-ms", type=float, default=0.0)
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--new-tokens", type=int, default=16)
    ap.add_argument("--trellis-pack", default=None, help="serve the routed experts from these trellis packs")
    args = ap.parse_args(argv)
    cfg = get_preset(args.model)
    if args.num_layers:
        cfg = cfg.replace(num_layers=args.num_layers)
    if args.hc_mult:
        cfg = cfg.replace(hc_mult=args.hc_mult)
    st = Stage(cfg, args.stage, args.stages, args.device, trellis_pack=args.trellis_pack)
    if args.stage > 0:
        ls = socket.create_server(("0.0.0.0", args.port))
        nxt = None
        if args.next:
            host, port = args.next.rsplit(":", 1)
            nxt = (host, int(port))
        serve_stage(st, ls, nxt, args.rtt_ms)
        ls.close()
        return
    host, port = args.peer.rsplit(":", 1)
    d = Driver(st, (host, int(port)), args.rtt_ms)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(3, cfg.vocab, (args.prompt_len,), generator=g).tolist()
    try:
        res = d.generate(prompt, args.new_tokens)
    finally:
        d.close()
    print(json.dumps({k: v for k, v in res.items() if k != "tokens"}))


if __name__ == "__main__":
    main()

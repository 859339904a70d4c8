"""CPU / reference executor with exactly the native runner's step semantics
(MTP k-draft verify, greedy acceptance, chained MTP drafts), built on the
fp32 reference model and per-sequence KV lists.  Used for the CPU engine
path and as the oracle of the GPU engine."""
from __future__ import annotations

from typing import Optional

import torch

from ..models import reference as ref
from ..models.weights import ModelWeights
from ..spec.logits_process import process_logits


class TorchRunner:
    def __init__(self, mw: ModelWeights, k: int, max_len: int, device="cpu", tp_group=None, sp_group=None,
                 dcp_group=None, dcp_interleave: int = 1, ep_group=None, dspark: Optional[dict] = None,
                 prefix_block: int = 0, prefix_entries: int = 64):
        self.mw = mw
        self.k = k if (mw.mtp is not None or mw.extra.get("eagle3") is not None) and dspark is None else 0
        self.dspark = None              # DSpark block drafting instead of MTP: {drafter, tau, budget_frac}
        if dspark is not None:
            from ..spec.dspark import DSparkDrafter
            torch.manual_seed(dspark.get("seed", 0))
            from ..spec.dspark_policy import DSparkPolicy
            block = dspark.get("block", 4)
            # drafter: "context" (the DSpark draft model over the target's aux hidden states,
            # default), "simple" (a context-free block head), or an object given as "drafter"
            drafter = dspark.get("drafter")
            if drafter is None and dspark.get("model", "context") == "simple":
                drafter = DSparkDrafter(mw.cfg.hidden, mw.cfg.vocab, block=block)
            self.dspark = dict(drafter=drafter, tau=dspark.get("tau", 0.5),
                               budget_frac=dspark.get("budget_frac", 0.5))
            # hardware-aware verify length: a cost table T(R, L) given, or profiled here
            pol = DSparkPolicy(block, self.dspark["tau"], self.dspark["budget_frac"])
            self.dspark["policy"] = pol
        self.dev = torch.device(device)
        self.cs = ref.rope_cos_sin(mw.cfg, max_len + 64, self.dev)
        self.rows = {}
        self.last_logits = {}           # row -> logits rows that predicted the tokens emitted by the last call
        self.prompt_logits = {}         # row -> logits of the prompt positions (prompt_logprobs)
        self.partial = {}               # row -> state of a prefill in progress (chunked prefill)
        # automatic prefix caching: block-aligned prompt prefix -> its main K/V, MTP K/V (one
        # position shorter: the MTP entry of the prefix's last position needs the next token),
        # last hidden state and logits
        from collections import OrderedDict
        self.prefix_block, self.prefix_entries = prefix_block, prefix_entries
        self.prefix_cache: "OrderedDict" = OrderedDict()
        self.prefix_stats = {"hits": 0, "hit_tokens": 0, "lookups": 0}
        self.tp_group = tp_group        # tensor-parallel CPU ranks (gloo): sharded weights, all-reduced partials
        self.sp_group = sp_group        # sequence-parallel prefill ranks: prompt chunks, gathered MLA latents
        self.dcp_group = dcp_group      # decode-context-parallel ranks: KV interleaved by position, LSE merge
        self.dcp_interleave = dcp_interleave
        self.moe_impl = None            # routed-expert function replacing the MoE block (e.g. the trellis tier)
        self.ep_group = ep_group        # expert parallelism over data-parallel ranks (all-to-all MoE)
        if dspark is not None:
            if self.dspark["drafter"] is None:
                from ..models.dspark_model import DSparkModelDrafter, random_dspark_weights
                dw = random_dspark_weights(mw, num_layers=dspark.get("layers", 2), window=dspark.get("window", 128),
                                           seed=dspark.get("seed", 0))
                self.dspark["drafter"] = DSparkModelDrafter(mw, dw, block, self.cs, markov=dspark.get("markov", True))
            if dspark.get("cost_table") is not None:
                pol.set_cost_table(*dspark["cost_table"])
            elif dspark.get("profile"):
                pol.set_cost_table(dspark.get("r_grid", [1, 2, 4]),
                                   self.profile_dspark(dspark.get("r_grid", [1, 2, 4]), block))

    def _row(self, r):
        return self.rows[r]

    def _ctx(self):
        import contextlib
        if self.moe_impl is not None:        # an alternative routed-expert tier (one rank)
            return ref.moe_context(self.moe_impl)
        if self.ep_group is not None:
            from ..parallel.ep import ep_moe_block
            g = self.ep_group
            return ref.moe_context(lambda cfg, lw, h: ep_moe_block(cfg, lw, h, g))
        if self.dcp_group is not None:
            from ..parallel.context import dcp_attention_fn
            return ref.attention_context(dcp_attention_fn(self.dcp_group))
        return ref.tp_context(self.tp_group) if self.tp_group is not None else contextlib.nullcontext()

    def _kv(self, n_layers: int):
        if self.dcp_group is None:
            return ref.RefKV(n_layers)
        import torch.distributed as dist
        from ..parallel.context import ShardKV
        return ShardKV(n_layers, dist.get_world_size(self.dcp_group), dist.get_rank(self.dcp_group),
                       self.dcp_interleave)

    @torch.no_grad()
    def prefill(self, prompts, rows, params=None):
        """params[i] (SamplingParams or None): temperature > 0 samples (per-row seeded
        generator); the verify steps then use speculative rejection sampling."""
        with self._ctx():
            return self._prefill(prompts, rows, params or [None] * len(prompts))

    def _sample_state(self, sp):
        if sp is None or sp.temperature <= 0:
            return None
        g = torch.Generator(device=self.dev)
        if sp.seed is not None:
            g.manual_seed(sp.seed)
        else:   # one draw shared by the TP ranks (they must sample the same tokens)
            from .sampling_params import shared_seeds
            g.manual_seed(shared_seeds(1, self.tp_group, self.dev)[0])
        return dict(sp=sp, gen=g)

    def _prefill(self, prompts, rows, params):
        firsts = []
        for prompt, r, sp in zip(prompts, rows, params):
            if self.sp_group is not None:
                firsts.append(self._prefill_sp(prompt, r, sp))
                continue
            self._start(prompt, r, sp)
            firsts.append(self._chunk(r, len(prompt)))
        return firsts

    # ------------------------------------------------------------------ chunked prefill
    @torch.no_grad()
    def start_prefill(self, prompt, r, sp=None):
        """Begin a prefill that `prefill_chunk` advances a token budget at a time."""
        self._start(prompt, r, sp)
        return self.partial[r]["done"]

    @torch.no_grad()
    def prefill_chunk(self, r, budget: int):
        """Run up to `budget` more prompt tokens of row r -> the first generated token when
        the prompt is complete, else None."""
        with self._ctx():
            return self._chunk(r, budget)

    def _start(self, prompt, r, sp):
        m, ent = self._prefix_lookup(prompt)
        if ent is not None:             # cached prefix: only the suffix runs
            main, mtp = self._kv_copy(ent["main"]), self._kv_copy(ent["mtp"])
            logits, hprev = [ent["logits"]], ent["hid"]
        else:
            main, mtp = self._kv(len(self.mw.layers)), self._kv(1)
            logits, hprev = [], None
        # invariant: main K/V covers [0, done), MTP K/V covers [0, done - 1) (the MTP entry of
        # position p needs token p + 1); hprev is the hidden state at done - 1
        self.partial[r] = dict(prompt=list(prompt), sp=sp, smp=self._sample_state(sp), main=main, mtp=mtp, done=m,
                               hprev=hprev, logits=logits, bound={}, chunks=0, dsnap={})
        if ent is not None and ent.get("dctx") is not None:      # the DSpark context of the prefix
            self.partial[r]["dctx"] = self._dctx_copy(ent["dctx"])

    def _chunk(self, r, budget):
        st = self.partial[r]
        prompt, main, mtp = st["prompt"], st["main"], st["mtp"]
        n, s = len(prompt), st["done"]
        e = min(n, s + max(1, budget))
        cd = self._context_drafter()
        aux = cd.aux_request() if cd is not None else None
        ls, hs = ref.forward(self.mw, torch.tensor(prompt[s:e], device=self.dev),
                             torch.arange(s, e, device=self.dev), self.cs, main, aux=aux)
        if cd is not None:
            # extend the drafter's context, snapshotting it at every block boundary for the
            # prefix cache (its window ends there)
            st.setdefault("dctx", cd.new_context())
            b, at = self.prefix_block, s
            cuts = [m for m in range(-(-(s + 1) // b) * b, min(e, n - 1) + 1, b)] if b else []
            for m in cuts + [e]:
                if m > at:
                    cd.extend(st["dctx"], {li: a[at - s:m - s] for li, a in aux.items()}, at, m - at)
                    at = m
                if m in cuts:
                    st["dsnap"][m] = self._dctx_copy(st["dctx"])
        st["logits"].append(ls)
        st["chunks"] += 1
        b = self.prefix_block
        if b and self.dcp_group is None:
            for m in range(-(-(s + 1) // b) * b, min(e, n - 1) + 1, b):      # prefixes ending in this chunk
                st["bound"][m] = hs[m - 1 - s]
        # MTP rows from position max(s - 1, 0): the hidden state of s - 1 came from the last chunk
        hid = hs if s == 0 else torch.cat([st["hprev"][None], hs])
        p0 = max(s - 1, 0)
        st["done"], st["hprev"] = e, hs[-1]
        if e < n:
            if self.k and e - 1 > p0:
                ref.mtp_forward(self.mw, hid[:-1], torch.tensor(prompt[p0 + 1:e], device=self.dev),
                                torch.arange(p0, e - 1, device=self.dev), self.cs, mtp)
            return None
        logits = torch.cat(st["logits"])
        last, smp = logits[-1], st["smp"]
        self.prompt_logits[r] = logits[:-1]          # rows that predicted prompt tokens 1..n-1
        self.last_logits[r] = last[None]
        tgt = self._first_token(process_logits(last[None], st["sp"], prompt, [])[0], smp, st["sp"])
        drafts = []
        if self.k:
            nxt = torch.tensor(prompt[p0 + 1:] + [tgt], device=self.dev)
            ml, mh = ref.mtp_forward(self.mw, hid, nxt, torch.arange(p0, n, device=self.dev), self.cs, mtp)
            drafts = self._chain_drafts(ml, mh, n, mtp)
        for m, h in st["bound"].items():
            self._prefix_put(prompt[:m], main, mtp, h, logits[:m], st["dsnap"].get(m))
        self.rows[r] = dict(main=main, mtp=mtp, tokens=[tgt] + drafts, pos=n, sample=smp, hid=hid[-1],
                            sp=st["sp"], prompt=prompt, out=[tgt], dctx=st.get("dctx"))
        del self.partial[r]
        return tgt

    def _first_token(self, last, smp, sp=None):
        if smp is None:
            return int(last.argmax())
        from ..spec.rejection import filter_probs
        p = filter_probs(last[None], smp["sp"].temperature, smp["sp"].top_k, smp["sp"].top_p, smp["sp"].min_p)
        return int(torch.multinomial(p[0], 1, generator=smp["gen"]))

    def _chain_drafts(self, ml, mh, n, mtp):
        d = int(ml[-1].argmax())
        drafts, h = [d], mh[-1:]
        for j in range(1, self.k):
            ml, h = ref.mtp_forward(self.mw, h, torch.tensor([d], device=self.dev),
                                    torch.tensor([n + j - 1], device=self.dev), self.cs, mtp)
            d = int(ml[-1].argmax()); drafts.append(d)
        return drafts

    def _prefill_sp(self, prompt, r, sp):
        """Sequence-parallel prefill: the prompt's chunks on the SP ranks, gathered latents."""
        from ..parallel.context import sp_prefill_forward
        smp = self._sample_state(sp)
        n = len(prompt)
        main, mtp = self._kv(len(self.mw.layers)), self._kv(1)
        last, hid = sp_prefill_forward(self.mw, torch.tensor(prompt, device=self.dev), self.cs, self.sp_group, main)
        self.last_logits[r] = last[None]
        tgt = self._first_token(last, smp)
        drafts = []
        if self.k:
            nxt = torch.tensor(prompt[1:] + [tgt], device=self.dev)
            ml, mh = ref.mtp_forward(self.mw, hid, nxt, torch.arange(n, device=self.dev), self.cs, mtp)
            drafts = self._chain_drafts(ml, mh, n, mtp)
        self.rows[r] = dict(main=main, mtp=mtp, tokens=[tgt] + drafts, pos=n, sample=smp, hid=hid[-1])
        return tgt

    # ------------------------------------------------------------------ prefix cache
    @staticmethod
    def _kv_copy(kv):
        c = ref.RefKV(len(kv.k))
        c.k, c.v = list(kv.k), list(kv.v)        # later appends concatenate into new tensors
        return c

    def _context_drafter(self):
        d = self.dspark["drafter"] if self.dspark is not None else None
        return d if hasattr(d, "extend") else None

    def _prefix_lookup(self, prompt):
        """-> (m, entry) of the longest cached block-aligned prefix shorter than the prompt
        (with a context drafter, only entries that hold its context)."""
        if not self.prefix_block or self.sp_group is not None or self.dcp_group is not None:
            return 0, None
        need_ctx = self._context_drafter() is not None
        self.prefix_stats["lookups"] += 1
        b = self.prefix_block
        for m in range((len(prompt) - 1) // b * b, 0, -b):
            ent = self.prefix_cache.get(tuple(prompt[:m]))
            if ent is not None and (not need_ctx or ent.get("dctx") is not None):
                self.prefix_cache.move_to_end(tuple(prompt[:m]))
                self.prefix_stats["hits"] += 1
                self.prefix_stats["hit_tokens"] += m
                return m, ent
        return 0, None

    @staticmethod
    def _dctx_copy(c):
        from ..models.dspark_model import DSparkContext
        return DSparkContext(list(c.k), list(c.v), c.end)

    def _prefix_put(self, key, main, mtp, hid, logits, dctx=None):
        """Cache one block-aligned prefix (`hid`: the hidden state at its last position;
        `dctx`: the DSpark context at its end)."""
        key, m = tuple(key), len(key)
        if key in self.prefix_cache:
            self.prefix_cache.move_to_end(key)
            return
        pm, pq = self._kv_copy(main), self._kv_copy(mtp)
        pm.truncate(m)
        pq.truncate(m - 1)
        self.prefix_cache[key] = dict(main=pm, mtp=pq, hid=hid, logits=logits, dctx=dctx)
        while len(self.prefix_cache) > self.prefix_entries:
            self.prefix_cache.popitem(last=False)

    def step(self, rows):
        """-> {row: (emitted tokens list, n_accepted)}"""
        with self._ctx():
            return self._step(rows)

    def _dspark_step(self, rows):
        """DSpark: the policy picks the batch-uniform verify length L (tokens / s from the
        cost table, calibrated survival and the engine overhead); one parallel block
        proposal per live row; per-row widths inside L (`allocate_widths`); each row
        verifies [pending token] + drafts[:width] in one target pass and emits the
        accepted prefix + the correction; the outcome feeds survival calibration."""
        ds = self.dspark
        drafter, pol = ds["drafter"], ds["policy"]
        L = pol.begin_step(len(rows))
        cd = self._context_drafter()
        if cd is not None:
            props = [cd.propose_one(self.rows[r]["dctx"], self.rows[r]["tokens"][0], self.rows[r]["pos"])
                     for r in rows]
            drafts, surv = torch.stack([d for d, _, _ in props]), torch.stack([c for _, _, c in props])
        else:
            h = torch.stack([self.rows[r]["hid"].float() for r in rows])
            last = torch.tensor([self.rows[r]["tokens"][0] for r in rows], device=self.dev)
            drafts, _, surv = drafter.propose(h, last)
        widths = pol.allocate(surv, len(rows), L) if L > 0 else torch.zeros(len(rows), dtype=torch.int32)
        out, acc = {}, []
        for i, r in enumerate(rows):
            st = self.rows[r]
            p, w = st["pos"], int(widths[i])
            st["main"].truncate(p)
            toks = torch.tensor([st["tokens"][0]] + drafts[i, :w].tolist(), device=self.dev)
            aux = cd.aux_request() if cd is not None else None
            logits, hid = ref.forward(self.mw, toks, torch.arange(p, p + w + 1, device=self.dev), self.cs,
                                      st["main"], aux=aux)
            tg = logits.argmax(-1).tolist()
            a = 0
            while a < w and int(drafts[i, a]) == tg[a]:
                a += 1
            if cd is not None:                         # the verified positions p .. p + a join the context
                cd.extend(st["dctx"], aux, p, a + 1)
            self.last_logits[r] = logits[: a + 1]
            st["tokens"], st["pos"], st["hid"] = [tg[a]], p + a + 1, hid[a]
            out[r] = (tg[: a + 1], a)
            acc.append(a)
        pol.observe(surv, widths, torch.tensor(acc), L)
        return out

    @torch.no_grad()
    def profile_dspark(self, r_grid, gamma: int, context: int = 16):
        """The DSpark cost table of this engine: seconds of one verify step of R rows at
        width 1 + L (a row verifies in one target pass of 1 + L tokens after `context`)."""
        from ..spec.dspark_policy import profile_cost_table
        H = self.mw.cfg.hidden
        caches = {}

        def step(R, L):
            for i in range(R):
                kv = caches.get(i)
                if kv is None:
                    kv = caches[i] = ref.RefKV(len(self.mw.layers))
                    ref.forward(self.mw, torch.arange(3, 3 + context, device=self.dev),
                                torch.arange(context, device=self.dev), self.cs, kv)
                kv.truncate(context)
                ref.forward(self.mw, torch.full((L + 1,), 5, device=self.dev),
                            torch.arange(context, context + L + 1, device=self.dev), self.cs, kv)
            cd = self._context_drafter()
            if cd is not None:
                for i in range(R):
                    c = cd.new_context()
                    cd.extend(c, {li: torch.zeros(context, H, device=self.dev) for li in cd.dw.target_layers},
                              0, context)
                    cd.propose_one(c, 5, context)
            else:
                self.dspark["drafter"].propose(torch.zeros(R, H, device=self.dev),
                                               torch.zeros(R, dtype=torch.long, device=self.dev))
        with self._ctx():
            return profile_cost_table(step, r_grid, gamma, repeats=3)

    def _step(self, rows):
        if self.dspark is not None:
            return self._dspark_step(rows)
        out = {}
        k = self.k
        for r in rows:
            st = self.rows[r]
            p = st["pos"]
            st["main"].truncate(p)
            toks = torch.tensor(st["tokens"], device=self.dev)
            pos = torch.arange(p, p + k + 1, device=self.dev)
            logits, hid = ref.forward(self.mw, toks, pos, self.cs, st["main"])
            smp, sp = st.get("sample"), st.get("sp")
            scores = logits if sp is None or not sp.processes_logits else \
                process_logits(logits, sp, st["prompt"], st["out"], st["tokens"][1:])
            if smp is None:
                tg = scores.argmax(-1).tolist()
                a = 0
                while a < k and st["tokens"][a + 1] == tg[a]:
                    a += 1
            else:       # speculative sampling: the MTP drafts are greedy, so q is one-hot
                from ..spec.rejection import filter_probs, rejection_sample
                sp = smp["sp"]
                probs = filter_probs(scores, sp.temperature, sp.top_k, sp.top_p, sp.min_p)     # [k+1, V]
                d = toks[1:].long()
                q = torch.nn.functional.one_hot(d, probs.shape[-1]).float()
                n_acc, em = rejection_sample(probs[None], q[None], d[None], generator=smp["gen"])
                a = int(n_acc[0])
                tg = em[0, : a + 1].tolist() + [int(em[0, a])] * (k - a)   # MTP input: accepted + sampled
            emitted = tg[: a + 1]
            self.last_logits[r] = logits[: a + 1]
            drafts = []
            if k:
                st["mtp"].truncate(p)
                ml, mh = ref.mtp_forward(self.mw, hid, torch.tensor(tg, device=self.dev), pos, self.cs, st["mtp"])
                d = int(ml[a].argmax()); drafts.append(d)
                h = mh[a:a + 1]
                st["mtp"].truncate(p + a + 1)
                for j in range(1, k):
                    ml, h = ref.mtp_forward(self.mw, h, torch.tensor([d], device=self.dev),
                                            torch.tensor([p + a + j], device=self.dev), self.cs, st["mtp"])
                    d = int(ml[-1].argmax()); drafts.append(d)
            st["tokens"] = [tg[a]] + drafts
            st["pos"] = p + a + 1
            if "out" in st:
                st["out"] += emitted
            out[r] = (emitted, a)
        return out

    @torch.no_grad()
    def dummy_rows(self, n: int):
        """EP: the MoE collectives of n rows with no tokens (see parallel.ep.ep_dummy_row)."""
        from ..parallel.ep import ep_dummy_row
        for _ in range(max(0, n)):
            ep_dummy_row(self.mw, self.k, self.ep_group)

    def release(self, r):
        self.rows.pop(r, None)
        self.partial.pop(r, None)
        self.last_logits.pop(r, None)
        self.prompt_logits.pop(r, None)

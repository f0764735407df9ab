"""Serving engine: requests, paged latent cache, prefill and decode steps, greedy sampling, CUDA-graph decode.

Public API (what a user of the reference's engine calls — ``prepare_model`` / ``forward_model`` of the slot ABI,
``king_v10/bundle_v9/slots.py:274-289``, wrap exactly this):

    eng = Engine(model_cfg, device="cuda", source=WeightSource(cfg, seed=0))
    out = eng.generate(prompts, max_new_tokens=16)          # greedy
    logits = eng.prefill(reqs); logits = eng.decode(reqs)    # step level

Decode steps are captured as CUDA graphs per batch bucket (the reference's decode / target-verify graph buckets,
``dec/gemm_tables.py:51``); a step replays the graph of the smallest bucket ≥ batch after copying the step's
metadata into the graph's static input buffers.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from ..config import ModelConfig
from ..models.deepseek import DeepseekModel, ForwardBatch
from ..models.weights import WeightSource
from .kv_cache import PagedLatentCache


@dataclass
class Request:
    rid: int
    prompt: List[int]
    out: List[int] = field(default_factory=list)
    pages: List[int] = field(default_factory=list)
    n_cached: int = 0            # tokens whose KV is in the cache
    done: bool = False
    late_from: int = 0           # first position that exists at the late layers (bounded late-layer replay)
    home: int = -1               # DP owner-only KV: the rank that caches this request's KV and runs its rows
    n_pages: int = 0             # DP owner-only KV: pages its home rank holds (known on every rank)

    @property
    def seq_len(self) -> int:
        return len(self.prompt) + len(self.out)


def _meta_ext():
    from ..ops._ext import available, ext

    return ext() if available() else None


class PinnedStager:
    """Reusable pinned host buffers for the per-step host -> device copies (token ids, positions, slots), so those
    copies are asynchronous DMA from page-locked memory.  Each key alternates between two buffers; a buffer is
    refilled only after the event recorded behind its last copy has completed.  CPU engines pass tensors through."""

    def __init__(self, device):
        self.device = device
        self.bufs: Dict[str, list] = {}
        self.turn: Dict[str, int] = {}

    def to_device(self, key: str, t: torch.Tensor) -> torch.Tensor:
        if self.device.type != "cuda":
            return t
        slots = self.bufs.setdefault(key, [None, None])
        i = self.turn.get(key, 0)
        self.turn[key] = i ^ 1
        n = t.numel()
        cur = slots[i]
        if cur is not None:
            cur[1].synchronize()                 # the copy that last read this buffer has finished
        if cur is None or cur[0].numel() < n or cur[0].dtype != t.dtype:
            cur = [torch.empty(max(n, 4096), dtype=t.dtype, pin_memory=True), None]
            slots[i] = cur
        view = cur[0][:n].view(t.shape)
        view.copy_(t)
        out = view.to(self.device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        cur[1] = ev
        return out


def decode_metadata(page_tables, seq_lens, page_size, pad_to, min_lmax=1):
    e = _meta_ext()
    if e is not None:
        return e.decode_metadata(page_tables, seq_lens, page_size, pad_to, min_lmax)
    B, Bp = len(seq_lens), max(len(seq_lens), pad_to)
    Lmax = max([min_lmax, 1] + list(seq_lens))
    out_loc = torch.zeros(Bp, dtype=torch.int32)
    ks = torch.full((Bp, Lmax), -1, dtype=torch.int32)
    nk = torch.ones(Bp, dtype=torch.int32)
    pos = torch.zeros(Bp, dtype=torch.int32)
    for b in range(B):
        L = seq_lens[b]
        for p in range(L):
            ks[b, p] = page_tables[b][p // page_size] * page_size + p % page_size
        out_loc[b] = ks[b, L - 1]
        nk[b] = L
        pos[b] = L - 1
    for b in range(B, Bp):
        ks[b, 0] = 0
    return [out_loc, ks, nk, pos]


def prefill_metadata(page_tables, starts, lens, page_size):
    e = _meta_ext()
    if e is not None:
        return e.prefill_metadata(page_tables, starts, lens, page_size)
    ol, ps = [], []
    for b, (s, n) in enumerate(zip(starts, lens)):
        for p in range(s, s + n):
            ol.append(page_tables[b][p // page_size] * page_size + p % page_size)
            ps.append(p)
    return [torch.tensor(ol, dtype=torch.int32), torch.tensor(ps, dtype=torch.int32)]


def _unpermute(rows: torch.Tensor, order: Sequence[int]) -> torch.Tensor:
    """rows[j] belongs to original item order[j]; returns them in original order."""
    inv = [0] * len(order)
    for j, i in enumerate(order):
        inv[i] = j
    return rows[torch.tensor(inv, dtype=torch.long, device=rows.device)]


class Engine:
    def __init__(self, cfg: ModelConfig, device="cpu", source: Optional[WeightSource] = None, num_pages: int = 256,
                 page_size: int = 64, model: Optional[DeepseekModel] = None, cuda_graphs: bool = False,
                 graph_buckets: Sequence[int] = (1, 2, 4, 8, 16, 32, 64, 128, 256), pctx=None, fp8: bool = True,
                 prefix_cache: bool = False, record_expert_load: bool = False, balance_dp: bool = False,
                 dp_owner_kv: bool = False, owner_kv: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.model = model if model is not None else DeepseekModel(cfg, source or WeightSource(cfg), device,
                                                                   fp8=fp8, pctx=pctx)
        dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.cache = PagedLatentCache(cfg, cfg.n_layers, num_pages, page_size, self.device, dtype)
        # page 0 is a scratch page for padded rows of graph buckets
        self._scratch = self.cache.alloc.alloc(1)
        self.page_size = page_size
        self._next_id = 0
        self._live: Dict[int, Request] = {}          # requests added and not yet released
        self.cuda_graphs = cuda_graphs and self.device.type == "cuda"
        self.graph_buckets = sorted(graph_buckets)
        self._graphs: Dict[int, "_DecodeGraph"] = {}
        self.stats = {"prefill_tokens": 0, "decode_tokens": 0}
        from ..utils.metrics import Metrics

        self.metrics = Metrics()       # device-timed steps: summary(), json_line(), prometheus()
        self.stager = PinnedStager(self.device)
        # DP attention: place prefill sequences and decode rows on ranks by a FLOP cost model instead of by count
        self.balance_dp = balance_dp
        # Owner-only KV: every request has a home rank (chosen by the cost-model planner at its prefill) that alone
        # allocates and writes its KV pages; its prefill and decode rows always run there, and decode pads each
        # rank's rows to the busiest rank's count (fixed per-rank blocks for the decode graphs).  Each rank then
        # holds only its own requests' KV.  DP attention reads the cache on the home rank by construction; TP
        # attention does too, because its cache-reading core runs token-parallel after the heads -> tokens
        # exchange (the prefill core of MLA works on the gathered new rows, not on the cache).
        # (`dp_owner_kv` is the older name of the same switch.)
        pc = self.model.pctx
        want = dp_owner_kv or owner_kv
        self.owner_kv = bool(want and pc.world > 1 and (pc.attn_dp or hasattr(pc, "heads_to_tokens")))
        if want and not self.owner_kv:
            raise ValueError("owner-only KV needs several ranks (DP attention, or TP attention with a heads -> "
                             "tokens exchange)")
        if self.owner_kv and prefix_cache:
            raise ValueError("owner-only KV does not combine with the prefix cache (pages are per home rank)")
        self.model.owner_kv = self.owner_kv
        if record_expert_load and cfg.n_routed_experts:
            from ..parallel.placement import ExpertLoad

            self.model.expert_load = ExpertLoad(cfg.n_routed_experts)
        # prefix reuse of full prompt pages (off with bounded late-layer replay: the late layers hold KV only for
        # each prompt's own replayed tail)
        self.prefix = None
        if prefix_cache and cfg.late_layer_start < 0:
            from .prefix_cache import PrefixCache

            self.prefix = PrefixCache(self.cache.alloc, page_size)

    # -- request lifecycle -------------------------------------------------------------------------------------------
    def add_request(self, prompt: Sequence[int]) -> Request:
        r = Request(self._next_id, list(int(t) for t in prompt))
        self._next_id += 1
        self._live[r.rid] = r
        if self.prefix is not None:
            r.pages = self.prefix.match(r.prompt)          # shared pages of the longest cached prefix
            r.n_cached = len(r.pages) * self.page_size
        return r

    def pages_for(self, r: Request, n_tokens: int) -> int:
        """New KV pages request ``r`` needs to hold ``n_tokens`` tokens (on its home rank, with owner-only KV)."""
        held = r.n_pages if self.owner_kv else len(r.pages)
        return max(0, (n_tokens + self.page_size - 1) // self.page_size - held)

    def pages_available(self, home: Optional[int] = None) -> int:
        """Pages an allocation can get now: free pages plus cached prefix pages that only the prefix cache holds.
        With owner-only KV, the free pages of rank ``home``, counted from the page counts of the requests it owns
        (the same number on every rank, so every rank takes the same scheduling decisions)."""
        if self.owner_kv:
            held = sum(r.n_pages for r in self._live.values() if r.home == home)
            return self.cache.alloc.num_pages() - 1 - held
        a = self.cache.alloc
        n = a.num_free()
        if self.prefix is not None:
            n += sum(1 for p in self.prefix.entries.values() if a.refcount(p) == 1)
        return n

    def _mine(self, r: Request) -> bool:
        return not self.owner_kv or r.home == self.model.pctx.rank

    def _table(self, r: Request, n_tokens: int) -> List[int]:
        """Page table used for ``r``'s metadata on this rank: its pages, or (owner-only KV, another rank's request)
        the scratch page for every position, so this rank never touches pages it does not own."""
        if self._mine(r):
            return r.pages
        return [self._scratch[0]] * max(1, (n_tokens + self.page_size - 1) // self.page_size)

    def _ensure_pages(self, r: Request, n_tokens: int):
        if self.owner_kv:
            need = self.pages_for(r, n_tokens)
            if need > 0 and self._mine(r):
                r.pages += list(self.cache.alloc.alloc(need))
            r.n_pages += need
            return
        need = self.pages_for(r, n_tokens)
        if need > 0:
            while self.prefix is not None and self.cache.alloc.num_free() < need and self.prefix.entries:
                self.prefix.evict(1)             # least recently used prefixes first (shared ones free nothing)
            r.pages += list(self.cache.alloc.alloc(need))

    def check_device(self) -> None:
        """Raise if a cross-rank kernel recorded an error (a bounded wait that ran out, a capacity overflow) in the
        parallel context's status word.  Contexts without device-side exchanges have nothing to check."""
        chk = getattr(self.model.pctx, "check", None)
        code = chk() if chk is not None else 0
        if code:
            what = {1: "producer data never arrived", 2: "a pipeline stage was never released",
                    3: "accumulator hand-off timed out", 4: "a peer rank's flag never arrived",
                    5: "bad argument"}.get(code, "unknown")
            raise RuntimeError(f"cross-rank kernel status {code}: {what}")

    def rebalance_experts(self):
        """Expert placement from the routing recorded while serving (``record_expert_load=True``): every MoE layer's
        experts are relabelled and moved so each EP rank carries a similar load.  Captured decode graphs are dropped
        (they hold the old weight tensors) and recaptured on the next decode.  All ranks call it together."""
        from ..parallel import placement

        if self.model.expert_load is None:
            raise RuntimeError("construct the engine with record_expert_load=True")
        out = placement.rebalance(self.model, self.model.expert_load)
        self._graphs.clear()
        return out

    def _register_prefix(self, reqs: List[Request]) -> None:
        if self.prefix is not None:
            for r in reqs:
                if r.n_cached >= len(r.prompt):
                    self.prefix.insert(r.prompt, r.pages)

    def release(self, r: Request):
        if r.pages:
            self.cache.alloc.free(r.pages)
            r.pages = []
        r.n_pages = 0
        self._live.pop(r.rid, None)

    # -- steps ---------------------------------------------------------------------------------------------------------
    def _dp_balanced(self) -> bool:
        pc = self.model.pctx
        return self.balance_dp and pc.world > 1 and pc.attn_dp

    def prefill(self, reqs: List[Request]) -> torch.Tensor:
        """Run every request's uncached prompt tokens; returns logits [B, V] of each request's last token.  Requests
        with a cached prefix (chunked prefill, prefix reuse) continue through per-row attention over the cache."""
        if any(r.n_cached > 0 for r in reqs):
            return self._prefill_rows(reqs, [r.seq_len - r.n_cached for r in reqs])
        if self.owner_kv or (self._dp_balanced() and len(reqs) > 1):
            from ..parallel.balance import plan_prefill

            world = self.model.pctx.world
            if self.owner_kv and all(r.home >= 0 for r in reqs):      # homes chosen by the caller (scheduler)
                order = sorted(range(len(reqs)), key=lambda i: (reqs[i].home, i))
                bounds = [0]
                for h in range(world):
                    bounds.append(bounds[-1] + sum(r.seq_len for r in reqs if r.home == h))
                return _unpermute(self._prefill_full([reqs[i] for i in order], bounds), order)
            order, bounds, _ = plan_prefill(self.cfg, [r.seq_len for r in reqs], world)
            if self.owner_kv:                # the planned rank becomes each request's home
                start = 0
                for i in order:
                    reqs[i].home = max(k for k in range(len(bounds) - 1) if bounds[k] <= start)
                    start += reqs[i].seq_len
            return _unpermute(self._prefill_full([reqs[i] for i in order], bounds), order)
        return self._prefill_full(reqs, None)

    def _prefill_full(self, reqs: List[Request], bounds: Optional[List[int]]) -> torch.Tensor:
        dev = self.device
        ids, starts, lens = [], [], []
        for r in reqs:
            toks = (r.prompt + r.out)[r.n_cached:]
            self._ensure_pages(r, r.seq_len)
            ids += toks
            starts.append(r.n_cached)
            lens.append(len(toks))
        if self.cfg.late_layer_start >= 0:
            for r, n in zip(reqs, lens):
                r.late_from = max(0, n - self.cfg.late_replay)
        out_loc, pos = prefill_metadata([self._table(r, r.seq_len) for r in reqs], starts, lens, self.page_size)
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        rows = torch.tensor([c - 1 for c in cu[1:]], dtype=torch.int32)
        st = self.stager
        fb = ForwardBatch(ids=st.to_device("ids", torch.tensor(ids, dtype=torch.int32)),
                          pos=st.to_device("pos", pos), out_loc=st.to_device("loc", out_loc),
                          is_prefill=True, cu_seqlens=cu, logits_rows=st.to_device("rows", rows),
                          bounds=bounds if bounds is not None else self._bounds(lens))
        with self.metrics.step("prefill", sum(lens), len(reqs)):
            logits = self.model.forward(fb, self.cache)
        for r, n in zip(reqs, lens):
            r.n_cached += n
        self.stats["prefill_tokens"] += sum(lens)
        self._register_prefix(reqs)
        return logits

    def prefill_chunked(self, reqs: List[Request], chunk: int) -> torch.Tensor:
        """Chunked prefill: each step runs at most ``chunk`` uncached prompt tokens per request, every token attending
        to its request's cached keys (the reference bounds a prefill step at 131,072 tokens, 32,768 per rank).
        Returns logits [B, V] of each request's last prompt token.  Every row of a step carries its own key-slot
        list, so a step's metadata is chunk x context int32 (e.g. 8,192 rows over a 32k context: 1 GB); size
        ``chunk`` to the context length."""
        if self.cfg.late_layer_start >= 0:
            for r in reqs:                      # the replayed tail is fixed by the whole prompt
                r.late_from = max(0, r.seq_len - self.cfg.late_replay)
        out = [None] * len(reqs)
        while True:
            todo = [(b, r) for b, r in enumerate(reqs) if r.n_cached < r.seq_len]
            if not todo:
                break
            n = [min(chunk, r.seq_len - r.n_cached) for _, r in todo]
            lg = self._prefill_rows([r for _, r in todo], n)
            for (b, r), row in zip(todo, lg):
                if r.n_cached == r.seq_len:
                    out[b] = row
        return torch.stack(out)

    def _row_layout(self, reqs: List[Request], rows: List[List[tuple]]):
        """Batch layout of per-row work (prefill chunks, verify rows): ``rows[b]`` holds request b's rows as
        (page table, keys, token, late_from).  Rows are concatenated, or, with owner-only KV, grouped by home rank
        with each rank's block padded to the busiest rank's count (pad rows on the scratch page).  Returns the
        flat (tables, lengths, ids, late) lists and the position of each request's first row."""
        tables, lens, ids, late, first = [], [], [], [], [0] * len(reqs)
        if self.owner_kv:
            world = self.model.pctx.world
            groups = [[b for b, r in enumerate(reqs) if r.home == h] for h in range(world)]
            width = max(sum(len(rows[b]) for b in g) for g in groups)
        else:
            groups, width = [list(range(len(reqs)))], 0
        for g in groups:
            k0 = len(ids)
            for b in g:
                first[b] = len(ids)
                for tb, n, tok, lf in rows[b]:
                    tables.append(tb)
                    lens.append(n)
                    ids.append(tok)
                    late.append(lf)
            pad = max(0, width - (len(ids) - k0))
            tables += [[self._scratch[0]]] * pad
            lens += [1] * pad
            ids += [0] * pad
            late += [0] * pad
        return tables, lens, ids, late, first

    def _prefill_rows(self, reqs: List[Request], counts: List[int]) -> torch.Tensor:
        """Run the next ``counts[b]`` uncached tokens of each request as per-row attention over the paged cache
        (keys: the request's cached tokens and the rows before it).  Returns logits [B, V] of each request's last
        row of this step.  With owner-only KV the rows are grouped by home rank (requests without one get it from
        the cost-model plan) and each rank's block is padded to the busiest rank's row count."""
        if self.owner_kv:
            fresh = [b for b, r in enumerate(reqs) if r.home < 0]
            if fresh:                               # first chunk: the cost-model plan picks the home rank
                from ..parallel.balance import plan_prefill

                world = self.model.pctx.world
                order, bounds, _ = plan_prefill(self.cfg, [counts[b] for b in fresh], world,
                                                [reqs[b].n_cached for b in fresh])
                start = 0
                for i in order:
                    reqs[fresh[i]].home = max(k for k in range(world) if bounds[k] <= start)
                    start += counts[fresh[i]]
        rows = []
        for r, n in zip(reqs, counts):
            toks = (r.prompt + r.out)[r.n_cached:r.n_cached + n]
            self._ensure_pages(r, r.n_cached + n)
            table = self._table(r, r.n_cached + n)
            rows.append([(table, r.n_cached + j + 1, int(tok), r.late_from) for j, tok in enumerate(toks)])
        rows_pt, rows_len, ids, late, first = self._row_layout(reqs, rows)
        last = [f + n - 1 for f, n in zip(first, counts)]
        m = len(ids)
        out_loc, key_slots, n_keys, pos = decode_metadata(rows_pt, rows_len, self.page_size, m)
        dev = self.device
        fb = ForwardBatch(ids=torch.tensor(ids, dtype=torch.int32).to(dev), pos=pos.to(dev), out_loc=out_loc.to(dev),
                          is_prefill=False, key_slots=key_slots.to(dev), n_keys=n_keys.to(dev),
                          bounds=self._bounds([1] * m), late_from=torch.tensor(late, dtype=torch.int32).to(dev))
        with self.metrics.step("prefill", sum(counts), len(reqs)):
            logits = self.model.forward(fb, self.cache)
        for r, n in zip(reqs, counts):
            r.n_cached += n
        self.stats["prefill_tokens"] += sum(counts)
        self._register_prefix(reqs)
        return logits[torch.tensor(last, dtype=torch.long, device=logits.device)]

    def decode(self, reqs: List[Request], next_tokens: Sequence[int]) -> torch.Tensor:
        """Append one token per request and run it; returns logits [B, V]."""
        if self.owner_kv:
            return self._decode_owner(reqs, next_tokens)
        if self._dp_balanced() and len(reqs) > 1:
            from ..parallel.balance import plan_rows, seq_cost

            n = self._bucket(len(reqs)) if self.cuda_graphs else len(reqs)
            n = n if n is not None else len(reqs)
            perm = plan_rows([seq_cost(self.cfg, 1, r.seq_len) for r in reqs], self._bounds([1] * n))
            return _unpermute(self._decode([reqs[i] for i in perm], [next_tokens[i] for i in perm]), perm)
        return self._decode(reqs, next_tokens)

    def _decode_owner(self, reqs: List[Request], next_tokens: Sequence[int]) -> torch.Tensor:
        """Owner-only KV decode: rank r's block of the batch holds the requests whose home is r, padded to the
        largest per-rank count (pad rows read and write the scratch page), so the even split of the step's rows
        puts every request on its home rank."""
        pc = self.model.pctx
        groups: List[List[int]] = [[] for _ in range(pc.world)]
        for j, r in enumerate(reqs):
            if not 0 <= r.home < pc.world:
                raise RuntimeError(f"request {r.rid} has no home rank (prefill it on this engine first)")
            groups[r.home].append(j)
        m = max(len(g) for g in groups)
        mb = (self._bucket(m) or m) if self.cuda_graphs else m
        order: List[Optional[int]] = []
        for g in groups:
            order += g + [None] * (mb - len(g))
        for r, t in zip(reqs, next_tokens):
            r.out.append(int(t))
            self._ensure_pages(r, r.seq_len)
        total = len(order)
        tables = [self._table(reqs[j], reqs[j].seq_len) if j is not None else [self._scratch[0]] for j in order]
        lens = [reqs[j].seq_len if j is not None else 1 for j in order]
        out_loc, key_slots, n_keys, pos = decode_metadata(tables, lens, self.page_size, total)
        ids = torch.tensor([reqs[j].out[-1] if j is not None else 0 for j in order], dtype=torch.int32)
        late = torch.tensor([reqs[j].late_from if j is not None else 0 for j in order], dtype=torch.int32)
        st = self.stager
        ids, pos, out_loc = st.to_device("d_ids", ids), st.to_device("d_pos", pos), st.to_device("d_loc", out_loc)
        key_slots, n_keys = st.to_device("d_keys", key_slots), st.to_device("d_nk", n_keys)
        late = st.to_device("d_late", late)
        B = len(reqs)
        with self.metrics.step("decode", B, B):
            if self.cuda_graphs and self._bucket(m) is not None:
                logits = self._graph(total, key_slots.shape[1]).run(ids, pos, out_loc, key_slots, n_keys, late)
            else:
                fb = ForwardBatch(ids=ids, pos=pos, out_loc=out_loc, is_prefill=False, key_slots=key_slots,
                                  n_keys=n_keys, bounds=self._bounds([1] * total), late_from=late)
                logits = self.model.forward(fb, self.cache)
        where = [0] * B
        for k, j in enumerate(order):
            if j is not None:
                where[j] = k
        for r in reqs:
            r.n_cached = r.seq_len
        self.stats["decode_tokens"] += B
        return logits[torch.tensor(where, dtype=torch.long, device=logits.device)]

    def _decode(self, reqs: List[Request], next_tokens: Sequence[int]) -> torch.Tensor:
        B = len(reqs)
        for r, t in zip(reqs, next_tokens):
            r.out.append(int(t))
            self._ensure_pages(r, r.seq_len)
        bucket = self._bucket(B) if self.cuda_graphs else B
        out_loc, key_slots, n_keys, pos = decode_metadata([r.pages for r in reqs], [r.seq_len for r in reqs],
                                                          self.page_size, bucket)
        ids = torch.zeros(bucket, dtype=torch.int32)
        ids[:B] = torch.tensor([r.out[-1] for r in reqs], dtype=torch.int32)
        late = torch.zeros(bucket, dtype=torch.int32)
        late[:B] = torch.tensor([r.late_from for r in reqs], dtype=torch.int32)
        st = self.stager
        ids, pos, out_loc = st.to_device("d_ids", ids), st.to_device("d_pos", pos), st.to_device("d_loc", out_loc)
        key_slots, n_keys = st.to_device("d_keys", key_slots), st.to_device("d_nk", n_keys)
        late = st.to_device("d_late", late)
        with self.metrics.step("decode", B, B):
            if self.cuda_graphs and bucket is not None:
                g = self._graph(bucket, key_slots.shape[1])
                logits = g.run(ids, pos, out_loc, key_slots, n_keys, late)[:B]
            else:
                fb = ForwardBatch(ids=ids, pos=pos, out_loc=out_loc, is_prefill=False, key_slots=key_slots,
                                  n_keys=n_keys, bounds=self._bounds([1] * bucket), late_from=late)
                logits = self.model.forward(fb, self.cache)[:B]
        for r in reqs:
            r.n_cached = r.seq_len
        self.stats["decode_tokens"] += B
        return logits

    def verify(self, reqs: List[Request], last_tokens: Sequence[int], drafts: List[List[int]]):
        """Target verification of speculative drafts (the reference's DSpark 6-row verify, ``dec/gemm_tables.py:51``).

        Each request appends ``last_token`` followed by its draft tokens; all rows run in ONE forward, every row
        attending to the cache plus the rows before it. Greedy acceptance keeps the longest draft prefix the target
        agrees with and adds the target's next token. Returns the accepted new tokens per request (>= 1 each).
        KV rows of rejected drafts are simply overwritten later (positions are slot-addressed)."""
        rows = []
        for r, t, d in zip(reqs, last_tokens, drafts):
            if self.owner_kv and not 0 <= r.home < self.model.pctx.world:
                raise RuntimeError(f"request {r.rid} has no home rank (prefill it on this engine first)")
            base = r.seq_len
            seq = [int(t)] + [int(x) for x in d]
            self._ensure_pages(r, base + len(seq))
            table = self._table(r, base + len(seq))
            rows.append([(table, base + j + 1, tok, r.late_from) for j, tok in enumerate(seq)])
        rows_pt, rows_len, ids, late, first = self._row_layout(reqs, rows)
        n = len(ids)
        # verify rows are decode rows (one token each, its own key list): a captured decode graph of a large enough
        # bucket serves them (the reference captures verify buckets of 6-row multiples).  Owner-only KV runs them
        # eagerly: its per-rank padded blocks need the exact row count.
        bucket = self._bucket(n) if self.cuda_graphs and not self.owner_kv else None
        out_loc, key_slots, n_keys, pos = decode_metadata(rows_pt, rows_len, self.page_size, bucket or n)
        dev = self.device
        with self.metrics.step("verify", n, len(reqs)):
            if bucket is not None:
                ids_t = torch.zeros(bucket, dtype=torch.int32)
                ids_t[:n] = torch.tensor(ids, dtype=torch.int32)
                late_t = torch.zeros(bucket, dtype=torch.int32)
                late_t[:n] = torch.tensor(late, dtype=torch.int32)
                logits = self._graph(bucket, key_slots.shape[1]).run(ids_t, pos, out_loc, key_slots, n_keys,
                                                                     late_t)[:n]
            else:
                fb = ForwardBatch(ids=torch.tensor(ids, dtype=torch.int32).to(dev), pos=pos.to(dev),
                                  out_loc=out_loc.to(dev), is_prefill=False, key_slots=key_slots.to(dev),
                                  n_keys=n_keys.to(dev), bounds=self._bounds([1] * n),
                                  late_from=torch.tensor(late, dtype=torch.int32).to(dev))
                logits = self.model.forward(fb, self.cache)
        pred = torch.argmax(logits.float(), dim=-1).tolist()
        accepted = []
        for r, t, d, i in zip(reqs, last_tokens, drafts, first):
            k = len(d) + 1
            p = pred[i:i + k]
            a = 0
            while a < len(d) and p[a] == d[a]:
                a += 1
            new = [int(x) for x in d[:a]] + [p[a]]
            r.out += [int(t)] + [int(x) for x in d[:a]]      # tokens whose KV is now valid in the cache
            r.n_cached = r.seq_len
            accepted.append(new)
        self.stats["decode_tokens"] += sum(len(x) for x in rows)
        return accepted

    def generate_speculative(self, prompts: List[Sequence[int]], max_new_tokens: int, drafter=None, n_draft: int = 5):
        """Greedy generation with draft-and-verify steps (``n_draft`` drafts + 1 row per request per step)."""
        from .spec import NgramDrafter

        drafter = drafter or NgramDrafter()
        reqs = [self.add_request(p) for p in prompts]
        logits = self.prefill(reqs)
        pending = torch.argmax(logits.float(), dim=-1).tolist()       # next token of each request, not yet cached
        produced = [[t] for t in pending]
        self.stats.setdefault("verify_steps", 0)
        while min(len(x) for x in produced) < max_new_tokens:
            drafts = [drafter.propose(r.prompt + r.out + [t], n_draft) for r, t in zip(reqs, pending)]
            acc = self.verify(reqs, pending, drafts)
            self.stats["verify_steps"] += 1
            for b, a in enumerate(acc):
                produced[b] += a
                pending[b] = a[-1]
        outs = [p[:max_new_tokens] for p in produced]
        for r in reqs:
            self.release(r)
        return outs

    def _bounds(self, lengths):
        """Per-rank token bounds (whole sequences per rank) when the model runs on several ranks."""
        pc = self.model.pctx
        if pc.world == 1:
            return None
        from ..parallel.dist import split_bounds

        return split_bounds(list(lengths), pc.world)

    def _bucket(self, B: int) -> Optional[int]:
        for b in self.graph_buckets:
            if b >= B:
                return b
        return None

    def _graph(self, bucket: int, lmax: int) -> "_DecodeGraph":
        g = self._graphs.get(bucket)
        if g is None or g.lmax < lmax:
            # context grows: recapture with headroom (power-of-two rounding of the key width)
            cap = max(lmax, 1 << math.ceil(math.log2(max(lmax, 2))))
            g = _DecodeGraph(self, bucket, cap)
            self._graphs[bucket] = g
        return g

    # -- convenience ---------------------------------------------------------------------------------------------------
    def generate(self, prompts: List[Sequence[int]], max_new_tokens: int, return_logits: bool = False):
        reqs = [self.add_request(p) for p in prompts]
        logits = self.prefill(reqs)
        history = [logits.float().cpu()] if return_logits else None
        nxt = torch.argmax(logits.float(), dim=-1).tolist()
        for _ in range(max_new_tokens - 1):
            logits = self.decode(reqs, nxt)
            if return_logits:
                history.append(logits.float().cpu())
            nxt = torch.argmax(logits.float(), dim=-1).tolist()
        for r, t in zip(reqs, nxt):
            r.out.append(int(t))
        outs = [r.out for r in reqs]
        for r in reqs:
            self.release(r)
        return (outs, history) if return_logits else outs


class _DecodeGraph:
    """One captured decode step for a fixed (bucket, key width). Inputs are static device buffers."""

    def __init__(self, eng: Engine, bucket: int, lmax: int):
        dev = eng.device
        self.lmax = lmax
        self.ids = torch.zeros(bucket, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(bucket, dtype=torch.int32, device=dev)
        self.out_loc = torch.zeros(bucket, dtype=torch.int32, device=dev)
        self.key_slots = torch.full((bucket, lmax), -1, dtype=torch.int32, device=dev)
        self.key_slots[:, 0] = 0
        self.n_keys = torch.ones(bucket, dtype=torch.int32, device=dev)
        self.late_from = torch.zeros(bucket, dtype=torch.int32, device=dev)
        fb = ForwardBatch(ids=self.ids, pos=self.pos, out_loc=self.out_loc, is_prefill=False,
                          key_slots=self.key_slots, n_keys=self.n_keys, bounds=eng._bounds([1] * bucket),
                          late_from=self.late_from)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up: lazy kernel attributes, allocator pools
                eng.model.forward(fb, eng.cache)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = eng.model.forward(fb, eng.cache)

    def run(self, ids, pos, out_loc, key_slots, n_keys, late_from=None) -> torch.Tensor:
        self.ids.copy_(ids, non_blocking=True)
        if late_from is not None:
            self.late_from.copy_(late_from, non_blocking=True)
        self.pos.copy_(pos, non_blocking=True)
        self.out_loc.copy_(out_loc, non_blocking=True)
        L = key_slots.shape[1]
        self.key_slots[:, :L].copy_(key_slots, non_blocking=True)
        if L < self.lmax:
            self.key_slots[:, L:].fill_(-1)
        self.n_keys.copy_(n_keys, non_blocking=True)
        self.graph.replay()
        return self.logits

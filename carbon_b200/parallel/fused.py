"""Multi-rank execution over NVLink peer memory (the product path; ``dist.DistCtx`` is the NCCL baseline).

Same sharding as ``DistCtx`` (sequence-sharded residual, TP attention, EP MoE, vocab-parallel embedding / head),
but every data movement is one of this repo's kernels on the symmetric heap:

* ``gather_rows``      — P2P stores of this rank's rows into every peer's gathered buffer (csrc/p2p.cu),
* ``reduce_scatter_rows`` — P2P stores of the o_proj partial rows into their owner's per-source slot, then a local
  fp32 sum of the slots,
* ``moe``              — count -> owner layout -> dispatch fused with the fp8 quantisation (rows and UE8M0 scales
  land in the owner's SF-tile layout) -> the owner's grouped tcgen05 GEMMs read them in place -> combine by P2P
  loads fused with the weighted top-k sum and the shared-expert add,
* ``embed``            — rows read straight from the owner's vocabulary shard in peer HBM.

Ordering between ranks uses one device-epoch barrier kernel (release/acquire at system scope, bounded wait; graph
capturable).  Gathered buffers are double-buffered per call site, which together with the barriers guarantees a
rank never overwrites data a slower peer is still reading.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch

from ..ops._ext import ext
from ..ops.gemm import fp8_gemm, fp8_gemm_swiglu
from ..ops.quant import sf_words
from .dist import DistCtx
from .symm import SymmHeap


class FusedCtx(DistCtx):
    def __init__(self, rank: int, world: int, group=None, heap_bytes: int = 4 << 30, max_tokens: int = 8192,
                 max_seq: int = 4096, moe_capacity: float = 1.6, barrier_timeout_s: float = 20.0,
                 attn_dp: bool = False, oproj_a2a: bool = True):
        super().__init__(rank, world, group, attn_dp=attn_dp, oproj_a2a=oproj_a2a)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.heap = SymmHeap(heap_bytes, rank, world, group, self.device)
        self.max_tokens = max_tokens
        self.max_local = min(max_tokens, (max_tokens + world - 1) // world + max_seq)
        self.moe_capacity = moe_capacity
        self.flags = self.heap.alloc((world,), torch.int32)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.limit_ns = int(barrier_timeout_s * 1e9)
        self._gather: Dict[str, list] = {}
        self._parity: Dict[str, int] = {}
        self._rs = None
        self._moe = None
        self._embed = None
        self._bounds_dev = None
        self._bounds_key = None

    # -- primitives ------------------------------------------------------------------------------------------------
    def barrier(self):
        ext().p2p_barrier(self.flags.peers, self.rank, self.epoch, self.flags.local, self.status, self.limit_ns)

    def check(self) -> int:
        """Device status word (0 = ok; otherwise a timeout / capacity error code recorded by a kernel)."""
        return int(self.status.item())

    def _gbuf(self, key: str, row_shape, dtype, rows: int):
        """Double-buffered gather slot for one call site; grows (power of two rows) when a call needs more rows.
        Every rank sees the same sequence of shapes, so the heap layout stays symmetric."""
        cur = self._gather.get(key)
        if cur is None or cur[0].shape[0] < rows:
            cap = 1 << max(4, (rows - 1).bit_length())
            self._gather[key] = [self.heap.alloc((cap,) + tuple(row_shape), dtype) for _ in range(2)]
            self._parity[key] = 0
        bufs = self._gather[key]
        p = self._parity[key]
        self._parity[key] = p ^ 1
        return bufs[p]

    def gather_rows(self, x: torch.Tensor, key: str = "rows") -> torch.Tensor:
        return self._gather_counts(x, self.counts(), key)

    def gather_var(self, x: torch.Tensor, counts: List[int], key: str = "var") -> torch.Tensor:
        return self._gather_counts(x, counts, key)

    def _gather_counts(self, x: torch.Tensor, cnt: List[int], key: str) -> torch.Tensor:
        T = sum(cnt)
        row0 = sum(cnt[: self.rank])
        b = self._gbuf(key + ":" + str(x.dtype) + str(tuple(x.shape[1:])), x.shape[1:], x.dtype, T)
        if x.shape[0] > 0:
            ext().p2p_gather_rows(x.contiguous(), b.peers, row0)
        self.barrier()
        return b.local[:T]

    def _bounds_tensor(self):
        key = tuple(self.bounds)
        if self._bounds_key != key:
            self._bounds_dev = torch.tensor(self.bounds, dtype=torch.int32, device=self.device)
            self._bounds_key = key
        return self._bounds_dev

    def heads_to_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """[T, Hl, W] (all tokens, this rank's heads) -> [n_r, world * Hl, W]: P2P stores of each owner's token rows
        into column block `rank` of its buffer, one barrier."""
        T, Hl, W = x.shape
        cnt = self.counts()
        buf = self._gbuf(f"h2t:{x.dtype}:{Hl}x{W}", (self.world * Hl, W), x.dtype, max(cnt))
        ext().p2p_a2a_heads(x.contiguous(), self._bounds_tensor(), self.rank, buf.peers, Hl * W * x.element_size(), 0,
                            max(cnt))
        self.barrier()
        return buf.local[: cnt[self.rank]]

    def tokens_to_heads(self, y: torch.Tensor) -> torch.Tensor:
        """Inverse of ``heads_to_tokens``: [n_r, world * Hl, W] -> [T, Hl, W]."""
        n, HW, W = y.shape
        Hl = HW // self.world
        T = self.bounds[-1] - self.bounds[0]
        buf = self._gbuf(f"t2h:{y.dtype}:{Hl}x{W}", (Hl, W), y.dtype, T)
        ext().p2p_a2a_heads(y.contiguous(), self._bounds_tensor(), self.rank, buf.peers, Hl * W * y.element_size(), 1,
                            n)
        self.barrier()
        return buf.local[:T]

    def reduce_scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        T, D = x.shape
        buf = self._rs_buf(D)
        n = self.counts()[self.rank]
        if max(self.counts()) > self.max_local:
            raise RuntimeError("reduce-scatter shard larger than the slot buffer")
        ext().p2p_scatter_partials(x.to(torch.bfloat16).contiguous(), self._bounds_tensor(), self.rank, buf.peers,
                                   self.max_local)
        self.barrier()
        out = torch.empty(n, D, dtype=torch.bfloat16, device=x.device)
        ext().reduce_slots(buf.local, self.world, self.max_local, n, out)
        return out

    def _rs_buf(self, D: int):
        if self._rs is None or self._rs[0].shape[2] != D:
            self._rs = [self.heap.alloc((self.world, self.max_local, D), torch.bfloat16) for _ in range(2)]
            self._rs_parity = 0
        buf = self._rs[self._rs_parity]
        self._rs_parity ^= 1
        return buf

    def row_parallel_out(self, lin, x):
        """o_proj GEMM fused with the reduce-scatter: the GEMM epilogue stores each output row into its owner's slot
        over NVLink; after one barrier the owner sums the world slots."""
        if getattr(lin, "kind", None) != "fp8":
            return self.reduce_scatter_rows(lin(x))
        from ..ops.quant import quant_act

        D = lin.out_features
        buf = self._rs_buf(D)
        if max(self.counts()) > self.max_local:
            raise RuntimeError("reduce-scatter shard larger than the slot buffer")
        q, sf = quant_act(x)
        ext().gemm_fp8_scatter(q, sf, lin.fw.q, lin.fw.sf, buf.peers, self._bounds_tensor(), self.rank,
                               self.max_local, self.status)
        self.barrier()
        n = self.counts()[self.rank]
        out = torch.empty(n, D, dtype=torch.bfloat16, device=x.device)
        ext().reduce_slots(buf.local, self.world, self.max_local, n, out)
        return out

    # -- model hooks -----------------------------------------------------------------------------------------------
    def adopt_embedding(self, model):
        """Move this rank's vocabulary shard into the heap so peers can read it."""
        if self._embed is not None:
            return
        V, D = model.embed.shape
        per = (model.cfg.vocab_size + self.world - 1) // self.world
        b = self.heap.alloc((per, D), torch.bfloat16)
        b.local[:V].copy_(model.embed)
        model.embed = b.local[:V]
        self._embed = (b, per)
        self.barrier()          # every shard is in place before any rank reads a peer's

    def embed(self, model, ids_all: torch.Tensor):
        self.adopt_embedding(model)
        cfg = model.cfg
        lo, hi = self.local
        ids = ids_all[lo:hi].to(torch.int32).contiguous()
        X = torch.empty(hi - lo, cfg.hc_streams, cfg.hidden_size, dtype=torch.bfloat16, device=ids.device)
        sumsq = torch.empty(hi - lo, device=ids.device)
        b, per = self._embed
        ext().embed_peer(b.peers, per, ids, X, sumsq)
        return X, sumsq

    def _moe_bufs(self, model, chunk: int, align: int, total_rows: int = 0):
        """Heap buffers of one MoE chunk for one segment alignment: set 0 holds a whole call (max_local tokens), set
        1 the second half of a two-chunk call.  256-aligned calls (prefill-sized) push the expert outputs to the
        tokens' home ranks (`slots`); 128-aligned calls (decode-sized: fewer than 384 routed rows per expert over
        all ranks) keep them in `y` for the homes to pull."""
        cfg = model.cfg
        D, El, k, E = cfg.hidden_size, model.E_local, cfg.n_activated_experts, cfg.n_routed_experts
        tokens = self.max_local if chunk == 0 else (self.max_local + 1) // 2
        rows = int(tokens * k * self.moe_capacity)
        if align == 128:
            # an owner receives at most the call's routed rows over all ranks (below 384 per expert at this
            # alignment): size classes of powers of two, so decode-sized calls get small buffers
            rows = min(rows, 1 << max(10, (max(total_rows, 1) - 1).bit_length()))
        cap = (rows + El * align + 255) // 256 * 256
        key = (chunk, align, cap)
        if self._moe is None:
            self._moe = {}
        if key not in self._moe:
            h = self.heap
            push = align == 256
            self._moe[key] = {
                "cnt": h.alloc((self.world, E), torch.int32),
                "off": torch.empty(E, dtype=torch.int32, device=self.device),
                "recv": h.alloc((cap, D), torch.float8_e4m3fn),
                "sf": h.alloc((sf_words(cap, D),), torch.int32),
                "rinfo": h.alloc((cap,), torch.int32),
                "slots": h.alloc((tokens * k, D), torch.bfloat16) if push else None,
                "y": None if push else h.alloc((cap, D), torch.bfloat16),
                "cap": cap,
                "mbe": torch.empty(cap // 128, dtype=torch.int32, device=self.device),
                "nb": torch.empty(1, dtype=torch.int32, device=self.device),
                "align": align,
                "push": push,
            }
        return self._moe[key]

    # a call is split in two pipelined chunks once the whole batch has at least this many tokens per rank
    CHUNK_MIN_TOKENS_PER_RANK = 2048

    def moe(self, model, L, h, w, ids, shared, hq=None):
        """EP MoE over NVLink.  Per chunk: counts to every rank -> barrier -> local layout + quantise and P2P row
        stores into the owners' expert-sorted buffers -> barrier -> owner's grouped GEMMs, whose down-projection
        epilogue stores each output row straight into its token's home-rank slot (prefill-sized calls) -> barrier ->
        local weighted top-k sum.  Decode-sized calls keep the outputs on the owner and the homes pull them after
        the third barrier (three barriers per call either way).
        Prefill-sized calls run as two token chunks on a communication stream and the compute stream: chunk 1's
        dispatch overlaps chunk 0's expert GEMMs, chunk 0's combine overlaps chunk 1's.  Every cross-rank barrier
        is issued on the communication stream, in the same order on every rank."""
        cfg = model.cfg
        T, k = ids.shape
        ids = ids.to(torch.int32).contiguous()
        wf = w.float().contiguous()
        from ..models.deepseek import resolve
        from ..ops.core import moe_align
        from ..utils.trace import region

        total = self.bounds[-1] - self.bounds[0] if self.bounds is not None else T
        # segment alignment from the call's routed rows over all ranks (the same number on every rank)
        align = moe_align(total * k, cfg.n_routed_experts)
        gmode = 1 if align == 256 else (2 if total * k <= 32 * cfg.n_routed_experts else 0)
        chunked = total >= self.CHUNK_MIN_TOKENS_PER_RANK * self.world and self.device.type == "cuda"
        out = torch.empty(T, cfg.hidden_size, dtype=torch.bfloat16, device=h.device)
        if not chunked:
            m = self._moe_bufs(model, 0, align, total * k)
            with region("moe.dispatch"):
                pos = self._moe_dispatch(model, m, h, ids)
            self._moe_gemms(model, L, m, gmode)
            with region("moe.combine"):
                self._moe_combine(model, m, ids, pos, wf, resolve(shared), out)
            return out
        main = torch.cuda.current_stream()
        if getattr(self, "_comm", None) is None:
            self._comm = torch.cuda.Stream(device=self.device)
        cs = self._comm
        half = (T + 1) // 2
        spans = [(0, half), (half, T)]
        bufs = [self._moe_bufs(model, c, align, total * k) for c in range(2)]
        ev_disp = [torch.cuda.Event() for _ in range(2)]
        ev_gemm = [torch.cuda.Event() for _ in range(2)]
        poss = [None, None]
        for t_ in (h, ids, wf, out):
            t_.record_stream(cs)
        cs.wait_stream(main)
        with torch.cuda.stream(cs), region("moe.dispatch"):
            for c, (a, b) in enumerate(spans):
                poss[c] = self._moe_dispatch(model, bufs[c], h[a:b], ids[a:b])
                ev_disp[c].record(cs)
        for c in range(2):
            main.wait_event(ev_disp[c])
            self._moe_gemms(model, L, bufs[c], gmode)
            ev_gemm[c].record(main)
        with torch.cuda.stream(cs), region("moe.combine"):
            sh = resolve(shared)
            for c, (a, b) in enumerate(spans):
                cs.wait_event(ev_gemm[c])
                self._moe_combine(model, bufs[c], ids[a:b], poss[c], wf[a:b], sh[a:b] if sh is not None else None,
                                  out[a:b])
        main.wait_stream(cs)
        return out

    def _moe_dispatch(self, model, m, h, ids):
        """Counts -> barrier -> layout -> quantise + P2P row stores (and the rows' way back) -> barrier."""
        e = ext()
        cfg = model.cfg
        T, k = ids.shape
        El, E = model.E_local, cfg.n_routed_experts
        # rows no source fills this call stay -1: the GEMM epilogues skip them.  Peers write rinfo only after the
        # next barrier, and this rank's last read of it (its previous call's GEMMs) precedes this point.
        m["rinfo"].local.fill_(-1)
        pair_rank = torch.empty(max(T * k, 1), dtype=torch.int32, device=self.device)
        e.moe_count(ids.reshape(-1), E, self.rank, m["cnt"].peers, pair_rank)
        self.barrier()
        e.moe_layout(m["cnt"].local, self.world, self.rank, m["off"], m["mbe"], m["nb"], m["align"])
        pos = torch.empty(T, k, dtype=torch.int32, device=self.device)
        if T > 0:
            e.moe_dispatch(h.contiguous(), ids, El, self.rank, pair_rank, m["recv"].peers, m["sf"].peers, m["off"],
                           m["rinfo"].peers, m["cap"], pos, self.status)
        self.barrier()
        return pos

    def _moe_gemms(self, model, L, m, gmode: int):
        """Owner side: grouped GEMMs over the expert-sorted received rows, in place in the heap.  Push mode: the
        down projection's epilogue stores every row into its home rank's combine slot over NVLink."""
        from ..utils.trace import region

        cfg = model.cfg
        I2 = 2 * cfg.moe_intermediate
        rv = m["rinfo"].local
        with region("moe.gemm_up"):
            act, act_sf = fp8_gemm_swiglu(m["recv"].local, m["sf"].local, L.e_w13, cfg.swiglu_limit, m["mbe"],
                                          m["nb"], I2, pair=gmode, row_valid=rv if gmode == 2 else None)
        with region("moe.gemm_down"):
            if m["push"]:
                ext().gemm_fp8_push(act, act_sf, L.e_w2.q, L.e_w2.sf, m["mbe"], m["nb"], cfg.hidden_size, rv,
                                    m["slots"].peers, self.status)
            else:
                fp8_gemm(act, act_sf, L.e_w2, out=m["y"].local, m_block_expert=m["mbe"], num_m_blocks=m["nb"],
                         n_per_group=cfg.hidden_size, pair=gmode, row_valid=rv if gmode == 2 else None)

    def _moe_combine(self, model, m, ids, pos, wf, shared, out):
        """Home side.  Push mode: one barrier (every owner's stores into this rank's slots are done), then a local
        weighted sum.  Pull mode: barrier, then P2P loads of the outputs from the owners.  No barrier follows the
        pull: an owner overwrites `y` only in the grouped GEMMs of its next call on these buffers, after that call's
        second barrier, which every home reaches only after its first barrier and so after this pull (stream
        order); the count matrix and the receive rows are likewise written by peers only past barriers this rank
        reaches after its last read of them."""
        self.barrier()
        if m["push"]:
            ext().moe_combine_slots(m["slots"].local, pos, wf, shared, out)
            return
        if ids.shape[0] > 0:
            ext().moe_combine_pull(m["y"].peers, ids, pos, wf, model.E_local, shared, out)

    def lm_head(self, model, y: torch.Tensor) -> torch.Tensor:
        part = model.head_w(y, out_dtype=torch.float32)                     # [n, V/world]
        per = (model.cfg.vocab_size + self.world - 1) // self.world
        n = part.shape[0]
        pad = torch.zeros(1, n * per, dtype=torch.float32, device=part.device)
        pad.view(n, per)[:, : part.shape[1]] = part
        g = self._gather_counts(pad, [1] * self.world, "logits%d" % n)        # [world, n*per]
        return g.view(self.world, n, per).permute(1, 0, 2).reshape(n, self.world * per)[:, : model.cfg.vocab_size]

"""Multi-rank execution: TP attention + EP MoE with a sequence-sharded residual, over ``torch.distributed``.

Layout (one process per GPU, all ranks run the same engine steps in the same order — SPMD):

* Every batch's tokens are split into contiguous per-rank shards at **sequence boundaries** (``ForwardBatch.bounds``).
  A rank owns the mHC residual streams, the boundaries, the q/kv down-projections, the DSA indexer and the MoE
  routing of its own tokens.
* The small outputs of the down-projections (q_lat, the MLA latent, the indexer key) and the DSA selection are
  **all-gathered** (``gather_rows``): attention is **tensor-parallel over heads** on all tokens, and every rank keeps
  the full latent cache (MLA's latent is shared by all heads).
* The row-parallel o_proj partial sums are **reduce-scattered** back to the token shards (``reduce_scatter_rows``).
* MoE is **expert-parallel**: ``moe`` sends each (token, expert) row to the expert's owner, runs the owner's
  grouped GEMMs and returns the rows for the weighted combine.
* Embedding and LM head are **vocab-parallel** (each rank holds V/world rows).

This module holds the collective-library implementation (NCCL on GPUs, gloo on CPU) — the baseline the fused
NVLink kernels in ``carbon_b200.parallel.fused`` are measured against. Reference: DP-attention 4 / EP4 with
MegaMoE's in-kernel dispatch and combine (``king_v10/bundle_v9/moe_route.py:190-213``), TP wo_b all-reduce
(``slots.py:63``), all-to-all Engram column exchange (``col_exchange.py:117``).
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .context import ParallelCtx


def split_bounds(lengths: List[int], world: int) -> List[int]:
    """Token bounds [world+1] assigning whole sequences (in order) to ranks, balancing token counts."""
    total = sum(lengths)
    bounds = [0]
    acc = 0
    target_i = 1
    for n in lengths:
        acc += n
        while target_i < world and acc >= total * target_i / world:
            bounds.append(acc)
            target_i += 1
    while len(bounds) < world + 1:
        bounds.append(total)
    bounds[-1] = total
    for i in range(1, len(bounds)):
        bounds[i] = max(bounds[i], bounds[i - 1])
    return bounds


class DistCtx(ParallelCtx):
    def __init__(self, rank: int, world: int, group=None, attn_dp: bool = False, oproj_a2a: bool = False):
        """attn_dp: data-parallel attention (each rank attends over its own sequences with all heads) instead of
        tensor-parallel attention over heads; MoE is expert-parallel either way.  oproj_a2a (TP attention): the
        per-head outputs go to each token's owner by an all-to-all and the owner runs the whole output projection,
        instead of a row-parallel projection whose [T, hidden] partial sums are reduce-scattered (the NCCL baseline
        keeps the reduce-scatter by default)."""
        super().__init__(rank=rank, world=world, tp=1 if attn_dp else world, ep=world,
                         tp_rank=0 if attn_dp else rank, ep_rank=rank, vocab_parallel=True, attn_dp=attn_dp,
                         oproj_a2a=oproj_a2a and not attn_dp and world > 1, group=group)
        self.bounds: Optional[List[int]] = None

    # -- shard bookkeeping ----------------------------------------------------------------------------------------
    def set_bounds(self, bounds: List[int]) -> None:
        assert len(bounds) == self.world + 1
        self.bounds = bounds

    @property
    def local(self):
        return self.bounds[self.rank], self.bounds[self.rank + 1]

    def counts(self) -> List[int]:
        return [self.bounds[i + 1] - self.bounds[i] for i in range(self.world)]

    # -- collectives ----------------------------------------------------------------------------------------------
    def gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        """Local rows [n_r, ...] -> all rows [T, ...] in global token order (uneven shards)."""
        cnt = self.counts()
        mx = max(cnt)
        pad = x.new_zeros((mx,) + tuple(x.shape[1:]))
        pad[: x.shape[0]] = x
        out = x.new_empty((self.world * mx,) + tuple(x.shape[1:]))
        dist.all_gather_into_tensor(out, pad.contiguous(), group=self.group)
        return torch.cat([out[r * mx: r * mx + cnt[r]] for r in range(self.world)], dim=0)

    def reduce_scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        """All-rows partial sums [T, ...] -> this rank's rows of the sum [n_r, ...]."""
        cnt = self.counts()
        mx = max(cnt)
        pad = x.new_zeros((self.world * mx,) + tuple(x.shape[1:]))
        for r in range(self.world):
            pad[r * mx: r * mx + cnt[r]] = x[self.bounds[r]: self.bounds[r + 1]]
        out = x.new_empty((mx,) + tuple(x.shape[1:]))
        if x.dtype == torch.bfloat16 and x.is_cuda:
            # sum in fp32 on the wire-independent side: NCCL reduces bf16 in bf16; keep that (baseline semantics)
            dist.reduce_scatter_tensor(out, pad, group=self.group)
        else:
            dist.reduce_scatter_tensor(out, pad, group=self.group)
        return out[: cnt[self.rank]]

    def all_to_all_rows(self, x: torch.Tensor, send_counts: List[int], recv_counts: List[int]) -> torch.Tensor:
        out = x.new_empty((sum(recv_counts),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=self.group)
        return out

    def heads_to_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """Tensor-parallel head shard of every token [T, Hl, W] -> every head of this rank's tokens
        [n_r, world * Hl, W] (head blocks in rank order)."""
        T, Hl, W = x.shape
        cnt = self.counts()
        n = cnt[self.rank]
        out = x.new_empty((self.world * n, Hl, W))
        dist.all_to_all_single(out, x.contiguous(), [n] * self.world, cnt, group=self.group)
        return out.view(self.world, n, Hl, W).permute(1, 0, 2, 3).reshape(n, self.world * Hl, W)

    def tokens_to_heads(self, y: torch.Tensor) -> torch.Tensor:
        """Inverse of ``heads_to_tokens``: [n_r, world * Hl, W] -> [T, Hl, W]."""
        n, HW, W = y.shape
        Hl = HW // self.world
        cnt = self.counts()
        send = y.view(n, self.world, Hl, W).permute(1, 0, 2, 3).reshape(self.world * n, Hl, W)
        out = y.new_empty((sum(cnt), Hl, W))
        dist.all_to_all_single(out, send.contiguous(), cnt, [n] * self.world, group=self.group)
        return out

    def exchange_counts(self, send_counts: torch.Tensor) -> List[int]:
        """send_counts [world] int64 (this rank -> r) -> recv_counts (r -> this rank)."""
        recv = torch.empty_like(send_counts)
        dist.all_to_all_single(recv, send_counts.contiguous(), group=self.group)
        return recv.tolist()

    # -- model hooks ----------------------------------------------------------------------------------------------
    def gather_var(self, x: torch.Tensor, counts: List[int]) -> torch.Tensor:
        """Like gather_rows with explicit per-rank row counts."""
        mx = max(max(counts), 1)
        pad = x.new_zeros((mx,) + tuple(x.shape[1:]))
        pad[: x.shape[0]] = x
        out = x.new_empty((self.world * mx,) + tuple(x.shape[1:]))
        dist.all_gather_into_tensor(out, pad.contiguous(), group=self.group)
        return torch.cat([out[r * mx: r * mx + counts[r]] for r in range(self.world)], dim=0)

    def embed(self, model, ids_all: torch.Tensor):
        """Vocab-parallel lookup: every rank sends the rows its vocabulary shard holds for the others' tokens."""
        cfg = model.cfg
        vs = model.v_hi - model.v_lo
        per = (cfg.vocab_size + self.world - 1) // self.world
        owner = (ids_all.long() // per).clamp(max=self.world - 1)
        b = self.bounds
        # rows I serve: for each destination rank r, the tokens of r whose id is in my shard (in token order)
        send_rows, send_counts = [], []
        for r in range(self.world):
            toks = torch.arange(b[r], b[r + 1], device=ids_all.device)
            mine = toks[owner[b[r]:b[r + 1]] == self.rank]
            send_rows.append(model.embed[(ids_all[mine].long() - model.v_lo).clamp(0, vs - 1)])
            send_counts.append(int(mine.numel()))
        send = torch.cat(send_rows, 0)
        recv_counts = [int(((owner[b[self.rank]:b[self.rank + 1]]) == s).sum()) for s in range(self.world)]
        recv = self.all_to_all_rows(send, send_counts, recv_counts)
        # place received rows back in local token order
        lo, hi = self.local
        own = owner[lo:hi]
        rows = torch.empty(hi - lo, cfg.hidden_size, dtype=model.embed.dtype, device=ids_all.device)
        off = 0
        for s in range(self.world):
            sel = torch.nonzero(own == s, as_tuple=True)[0]
            rows[sel] = recv[off: off + sel.numel()]
            off += sel.numel()
        X = rows[:, None, :].expand(hi - lo, cfg.hc_streams, cfg.hidden_size).contiguous()
        sumsq = X.float().pow(2).sum((1, 2)) if model.on_gpu else None
        return X, sumsq

    def moe(self, model, L, h, w, ids, shared, hq=None):
        """Expert parallel: route rows to their experts' owners (all-to-all), grouped GEMMs there, rows back."""
        El = model.E_local
        T, k = ids.shape
        flat_e = ids.reshape(-1).long()
        dest = flat_e // El
        order = torch.sort(dest, stable=True).indices
        send_counts_t = torch.bincount(dest, minlength=self.world)
        send_counts = send_counts_t.tolist()
        recv_counts = self.exchange_counts(send_counts_t)
        send_x = h[order // k]
        send_e = (flat_e[order] % El).to(torch.int32)
        recv_x = self.all_to_all_rows(send_x, send_counts, recv_counts)
        recv_e = self.all_to_all_rows(send_e, send_counts, recv_counts)
        n_recv = recv_x.shape[0]
        if n_recv > 0:
            ones = torch.ones(n_recv, 1, dtype=torch.float32, device=h.device)
            y = model.moe_local(L, recv_x, ones, recv_e.view(-1, 1), None)
        else:
            y = recv_x
        back = self.all_to_all_rows(y.to(h.dtype), recv_counts, send_counts)     # rows in `order`
        contrib = torch.zeros(T * k, h.shape[1], dtype=torch.float32, device=h.device)
        contrib[order] = back.float()
        out = (contrib.view(T, k, h.shape[1]) * w.float()[..., None]).sum(1)
        if shared is not None:
            from ..models.deepseek import resolve

            out = out + resolve(shared).float()
        return out.to(h.dtype)

    def lm_head(self, model, y: torch.Tensor) -> torch.Tensor:
        """y: final normalized rows [n, D] of ALL logits rows (gathered by the caller) -> logits [n, V]."""
        part = model.head_w(y, out_dtype=torch.float32)                     # [n, V/world]
        per = (model.cfg.vocab_size + self.world - 1) // self.world
        pad = part.new_zeros(part.shape[0], per)
        pad[:, : part.shape[1]] = part
        n = part.shape[0]
        out = part.new_empty(self.world * n, per)
        dist.all_gather_into_tensor(out, pad.contiguous(), group=self.group)
        return out.view(self.world, n, per).permute(1, 0, 2).reshape(n, self.world * per)[:, : model.cfg.vocab_size]

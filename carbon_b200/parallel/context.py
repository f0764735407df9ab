"""Parallel context: where the model's collectives plug in.

The model calls four hooks; this module provides the single-rank versions and the NCCL baseline versions.  The
fused NVLink kernels (``carbon_b200.parallel.fused``) replace the NCCL ones when enabled.

* ``embed(model, ids)``      — vocab-parallel embedding lookup (rows of other ranks come from their HBM).
* ``attn_out(x)``            — TP attention output reduction (all-reduce of the row-parallel o_proj partials).
* ``moe(model, L, h, w, ids, shared)`` — expert-parallel MoE: dispatch rows to expert owners, grouped GEMMs, combine.
* ``lm_head(model, y)``      — vocab-parallel LM head (logits of all ranks' vocabulary shards).

Reference equivalents: MegaMoE's in-kernel dispatch/combine over a symmetric buffer (``cuda_moe_prefill.py:
4343-4660,5542-5681``), the TP wo_b all-reduce (``slots.py:63``), Engram/embedding peer reads
(``cuda_peer_read.py:64``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class ParallelCtx:
    rank: int = 0
    world: int = 1
    tp: int = 1
    ep: int = 1
    tp_rank: int = 0
    ep_rank: int = 0
    vocab_parallel: bool = False
    # DP attention: every rank runs attention for its own sequences with all heads (tp = 1 for attention weights,
    # no attention collectives); MoE stays expert-parallel over all ranks
    attn_dp: bool = False
    # TP attention output: heads -> tokens all-to-all of the per-head outputs, then the whole output projection on each
    # token's owner (wo replicated), instead of the row-parallel projection + reduce-scatter of [T, hidden] partials
    oproj_a2a: bool = False
    group: Optional[object] = None   # torch.distributed process group (NCCL) when world > 1
    bounds: Optional[list] = None    # token shard bounds of the current batch ([0, T] on one rank)

    @staticmethod
    def single() -> "ParallelCtx":
        return ParallelCtx()

    def set_bounds(self, bounds) -> None:
        self.bounds = bounds

    @property
    def local(self):
        return self.bounds[self.rank], self.bounds[self.rank + 1]

    def gather_rows(self, x):
        return x

    def gather_var(self, x, counts):
        return x

    def reduce_scatter_rows(self, x):
        return x

    def row_parallel_out(self, lin, x):
        """Row-parallel projection (o_proj) of all tokens, reduced onto each token's owner rank."""
        return self.reduce_scatter_rows(lin(x))

    # -- hooks (single rank) -----------------------------------------------------------------------------------------
    def embed(self, model, ids: torch.Tensor):
        """ids: all tokens of the batch (one rank: all tokens are local)."""
        from ..ops._ext import ext

        cfg = model.cfg
        T = ids.shape[0]
        X = torch.empty(T, cfg.hc_streams, cfg.hidden_size, dtype=torch.bfloat16, device=ids.device)
        sumsq = torch.empty(T, device=ids.device)
        ext().embed_hc(model.embed, model.v_lo, ids.to(torch.int32).contiguous(), X, sumsq)
        return X, sumsq

    def attn_out(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def moe(self, model, L, h, w, ids, shared, hq=None):
        return model.moe_local(L, h, w, ids, shared, hq=hq)

    def lm_head(self, model, y: torch.Tensor) -> torch.Tensor:
        return model.head_w(y, out_dtype=torch.float32)

"""Cost-model balancing of data-parallel attention ranks (prefill sequences, decode rows).

With DP attention each rank runs its own requests' rows through attention, the indexer, mHC and the dense / shared
projections; only the routed experts are spread by routing.  Splitting a batch by token count therefore leaves the
rank that holds the long prompt (quadratic attention and indexer work) or the long contexts (decode indexer scans and
attention keys) behind the others, and every MoE exchange waits for it.  The reference plans moves of token rows from
heavy DP ranks to light ones with a per-row cost model: REHOME in prefill (``rehome_plan.py:347-387``, ns-per-row
constants ``:17-24``) and ROW_BALANCE in decode (``dec/row_balance.py:124-146``).

Here the cost of a sequence is counted in FLOPs from the model config (row-local projections per token, attention
query-key pairs per layer with the DSA top-k / window caps, indexer pairs on indexer layers), and requests are
placed whole: LPT (longest-processing-time first) over ranks for prefill, where the per-rank token bounds follow the
plan; and, for decode, a capacity-constrained LPT that keeps the per-rank row counts (so captured decode graphs keep
their shapes) and only chooses which rows each rank runs.  By default decode KV is in every DP rank's cache (new
rows are all-gathered), so a request can move between ranks from one step to the next at no transfer cost; with
owner-only KV (``Engine(owner_kv=True)``) the prefill plan fixes each request's home rank instead.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

from ..config import ModelConfig


def _capped_pairs(p0: int, n: int, cap: int) -> int:
    """Σ_{p=p0}^{p0+n-1} min(p + 1, cap): keys seen by the causal queries at positions p0..p0+n-1 with at most
    ``cap`` keys each (cap <= 0: no cap)."""
    def f(P: int) -> int:                           # Σ_{p<P} min(p + 1, cap)
        if cap <= 0 or P <= cap:
            return P * (P + 1) // 2
        return cap * (cap + 1) // 2 + (P - cap) * cap
    return f(p0 + n) - f(p0)


def _token_flops(cfg: ModelConfig, layer: int) -> float:
    """FLOPs per token of one layer's row-local projections (everything but the routed experts and the attention
    core): q / kv down and up projections, output projection, dense or shared-expert FFN, indexer projections."""
    h, H = cfg.hidden_size, cfg.n_heads
    dq = cfg.qk_head_dim
    ql = cfg.q_lora_rank or h
    p = 0
    p += h * ((cfg.q_lora_rank or 0) + cfg.latent_dim)                   # q_a + kv_a
    p += ql * H * dq                                                     # q_b
    if cfg.attn_kind != "latent_mqa":
        p += cfg.kv_lora_rank * H * (cfg.qk_nope_head_dim + cfg.v_head_dim)   # kv_b (prefill MHA form)
    if cfg.o_groups:
        p += H * cfg.head_out_dim * cfg.o_lora_rank + cfg.o_groups * cfg.o_lora_rank * h
    else:
        p += H * cfg.head_out_dim * h
    if cfg.is_moe_layer(layer):
        p += 3 * h * cfg.moe_intermediate * cfg.n_shared_experts + h * cfg.n_routed_experts
    else:
        p += 3 * h * cfg.dense_intermediate
    if cfg.has_indexer(layer):
        p += ql * cfg.index_n_heads * cfg.index_head_dim + h * (cfg.index_head_dim + cfg.index_n_heads)
    return 2.0 * p


def seq_cost(cfg: ModelConfig, n_new: int, n_ctx: int = 0) -> float:
    """Rank-local FLOPs to run ``n_new`` tokens of one sequence whose first ``n_ctx`` tokens are already cached."""
    if n_new <= 0:
        return 0.0
    H = cfg.n_heads
    if cfg.attn_kind == "latent_mqa":
        pair = 2.0 * H * (cfg.kv_lora_rank + cfg.kv_lora_rank)
    else:
        pair = 2.0 * H * (cfg.qk_head_dim + cfg.v_head_dim)
    idx_pair = 2.0 * cfg.index_n_heads * cfg.index_head_dim
    total = 0.0
    for layer in range(cfg.n_layers):
        n, p0 = n_new, n_ctx
        if cfg.is_late_layer(layer) and n_ctx == 0:             # bounded replay: late layers run the tail only
            keep = min(n, cfg.late_replay)
            p0, n = p0 + n - keep, keep
        total += n * _token_flops(cfg, layer)
        src = cfg.index_source(layer)
        if src is not None:
            cap = cfg.index_topk + (cfg.swa_window if cfg.attn_kind == "latent_mqa" else 0)
        elif cfg.attn_kind == "latent_mqa" and cfg.swa_window > 0:
            cap = cfg.swa_window
        else:
            cap = 0
        total += pair * _capped_pairs(p0, n, cap)
        if cfg.has_indexer(layer):
            total += idx_pair * _capped_pairs(p0, n, 0)
    return total


def plan_prefill(cfg: ModelConfig, lengths: Sequence[int], world: int,
                 cached: Sequence[int] = None) -> Tuple[List[int], List[int], List[float]]:
    """Place whole sequences on ``world`` DP ranks balancing ``seq_cost``.  Returns (order, bounds, rank_costs):
    the batch reordered so that rank r's sequences are contiguous (original indices, original order within a rank),
    the per-rank token bounds [world + 1] of that order, and each rank's planned cost."""
    cached = list(cached) if cached is not None else [0] * len(lengths)
    costs = [seq_cost(cfg, n, c) for n, c in zip(lengths, cached)]
    load = [0.0] * world
    owner = [0] * len(lengths)
    for i in sorted(range(len(lengths)), key=lambda i: (-costs[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += costs[i]
    order = [i for r in range(world) for i in range(len(lengths)) if owner[i] == r]
    bounds, acc = [0], 0
    for r in range(world):
        acc += sum(lengths[i] for i in range(len(lengths)) if owner[i] == r)
        bounds.append(acc)
    return order, bounds, load


def plan_rows(costs: Sequence[float], bounds: Sequence[int]) -> List[int]:
    """Decode rows: batch positions are split over the ranks by the fixed ``bounds`` [world + 1] the decode step
    runs with (the split its graphs are captured with; padding positions follow the ``len(costs)`` real rows).
    Returns perm with perm[position] = original row for the real positions, chosen so the per-rank cost sums are as
    even as those block capacities allow (capacity-constrained LPT)."""
    n = len(costs)
    world = len(bounds) - 1
    cap = [max(0, min(bounds[r + 1], n) - bounds[r]) for r in range(world)]
    load = [0.0] * world
    rows: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(n), key=lambda i: (-costs[i], i)):
        r = min((r for r in range(world) if len(rows[r]) < cap[r]), key=lambda r: (load[r], r))
        rows[r].append(i)
        load[r] += costs[i]
    return [i for r in range(world) for i in sorted(rows[r])]


def imbalance(rank_costs: Sequence[float]) -> float:
    """max / mean of per-rank costs (1.0 = perfectly even)."""
    m = sum(rank_costs) / max(1, len(rank_costs))
    return max(rank_costs) / m if m > 0 else 1.0


def split_costs(cfg: ModelConfig, lengths: Sequence[int], bounds: Sequence[int]) -> List[float]:
    """Per-rank costs of the in-order whole-sequence split given by token ``bounds`` (the unbalanced baseline)."""
    out = [0.0] * (len(bounds) - 1)
    start = 0
    for n in lengths:
        r = max(k for k in range(len(bounds) - 1) if bounds[k] <= start) if start < bounds[-1] else len(bounds) - 2
        out[r] += seq_cost(cfg, n)
        start += n
    return out

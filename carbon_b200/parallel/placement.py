"""Expert placement: relabel experts so that every EP rank carries a similar routed load.

The reference fits a per-layer table offline and moves expert tensors with one NCCL all-to-all
(``king_v10/bundle_v9/placement.py:47-128``, ``placement_table.py``).  Here:

* ``ExpertLoad`` accumulates per-layer expert hit counts from the router output (host-side, cheap: one bincount
  per MoE layer while enabled);
* ``plan(load, ep)`` is a greedy longest-processing-time assignment: experts in decreasing load go to the rank
  with the least load that still has a free slot.  It returns ``perm`` with ``perm[new_id] = old_id``; rank r
  then owns new ids ``[r*El, (r+1)*El)``;
* ``apply(model, layer, perm)`` permutes that layer's router rows, router bias and stacked expert weights in place,
  so routing picks the new ids directly and the model computes exactly the same function.

On several ranks the relabelled weights of a rank come from other ranks; ``redistribute`` moves them with one
all-to-all per weight tensor (same mechanism as the reference).
"""
from __future__ import annotations

from typing import Dict, List

import torch


class ExpertLoad:
    def __init__(self, n_experts: int):
        self.E = n_experts
        self.counts: Dict[int, torch.Tensor] = {}
        self.dev_counts: Dict[int, torch.Tensor] = {}

    def record(self, layer: int, ids: torch.Tensor) -> None:
        c = torch.bincount(ids.reshape(-1).long().cpu(), minlength=self.E)
        self.counts[layer] = self.counts.get(layer, torch.zeros(self.E, dtype=torch.long)) + c

    def record_device(self, layer: int, ids: torch.Tensor) -> None:
        """Accumulate on the router's device with a scatter-add: no host synchronisation, so it also runs inside
        captured decode graphs (the counter exists from the first eager step on)."""
        c = self.dev_counts.get(layer)
        if c is None:
            c = torch.zeros(self.E, dtype=torch.int64, device=ids.device)
            self.dev_counts[layer] = c
        flat = ids.reshape(-1).long()
        c.index_add_(0, flat, torch.ones_like(flat))

    def take(self, layer: int) -> torch.Tensor:
        """This rank's counts of one layer since the last take (host and device records), then reset."""
        out = self.counts.pop(layer, torch.zeros(self.E, dtype=torch.long)).clone()
        c = self.dev_counts.get(layer)
        if c is not None:
            out += c.cpu()
            c.zero_()
        return out


def plan(load: torch.Tensor, ep: int) -> torch.Tensor:
    """load [E] -> perm [E] (perm[new] = old) balancing the summed load of each rank's E/ep experts."""
    E = load.numel()
    El = E // ep
    order = torch.argsort(load.float(), descending=True, stable=True).tolist()
    rank_load = [0.0] * ep
    slots: List[List[int]] = [[] for _ in range(ep)]
    for e in order:
        r = min((r for r in range(ep) if len(slots[r]) < El), key=lambda r: (rank_load[r], r))
        slots[r].append(e)
        rank_load[r] += float(load[e])
    return torch.tensor([e for r in range(ep) for e in sorted(slots[r])], dtype=torch.long)


def imbalance(load: torch.Tensor, ep: int, perm: torch.Tensor = None) -> float:
    """max rank load / mean rank load for a placement (identity when perm is None)."""
    l = load.float() if perm is None else load.float()[perm]
    per = l.view(ep, -1).sum(1)
    return float(per.max() / per.mean().clamp(min=1e-9))


def apply(model, layer: int, perm: torch.Tensor) -> None:
    """Relabel the experts of one MoE layer of a single-rank model (EP = 1) in place."""
    L = model.layers[layer]
    assert L.moe and model.pctx.ep == 1, "apply() relabels a single-rank model; use redistribute() across ranks"
    p = perm.to(L.gate_b.device)
    if L.gate.kind == "f32" or L.gate.kind == "bf16":
        L.gate.w[: p.numel()] = L.gate.w[: p.numel()][p.to(L.gate.w.device)]
    L.gate_b.copy_(L.gate_b[p])
    if model.on_gpu:
        from ..ops.quant import Fp8Weight, pack_sf

        for name in ("e_w13", "e_w2"):
            W = getattr(L, name)
            E = p.numel()
            rows = W.q.shape[0] // E
            pq = p.to(W.q.device)
            q = W.q.view(E, rows, -1)[pq].reshape(E * rows, -1).contiguous()
            scale = W.scale.view(E, rows // 128, -1)[pq].reshape(E * rows // 128, -1).contiguous()
            setattr(L, name, Fp8Weight(q, pack_sf(scale.repeat_interleave(128, dim=0)), scale))
    else:
        L.e_w1 = L.e_w1[p].contiguous()
        L.e_w3 = L.e_w3[p].contiguous()
        L.e_w2 = L.e_w2[p].contiguous()


def _exchange_experts(t: torch.Tensor, perm: torch.Tensor, E: int, ep: int, rank: int, group) -> torch.Tensor:
    """t: this rank's experts stacked on dim 0 ([El * rows, ...], old labels).  Returns the rows of the experts this
    rank owns under ``perm`` (new labels [rank*El, (rank+1)*El), in order), fetched with one all-to-all."""
    import torch.distributed as dist

    El = E // ep
    rows = t.shape[0] // El
    p = perm.tolist()
    send_idx, send_counts = [], []
    for d in range(ep):                      # experts destination d needs from this rank, in new-id order
        mine = [p[n] - rank * El for n in range(d * El, (d + 1) * El) if p[n] // El == rank]
        send_idx += mine
        send_counts.append(len(mine) * rows)
    recv_src = [p[n] // El for n in range(rank * El, (rank + 1) * El)]
    recv_counts = [sum(1 for s in recv_src if s == r) * rows for r in range(ep)]
    tv = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t      # NCCL moves fp8 as bytes
    tv = tv.view(El, rows, *tv.shape[1:])
    send = tv[torch.tensor(send_idx, dtype=torch.long, device=t.device)].reshape(-1, *tv.shape[2:]).contiguous() \
        if send_idx else tv.new_empty((0,) + tuple(tv.shape[2:]))
    recv = tv.new_empty((sum(recv_counts),) + tuple(tv.shape[2:]))
    dist.all_to_all_single(recv, send, recv_counts, send_counts, group=group)
    # received blocks arrive grouped by source rank, each group in new-id order
    starts, off = [], 0
    for r in range(ep):
        starts.append(off)
        off += recv_counts[r]
    seen = [0] * ep
    parts = []
    for s in recv_src:
        parts.append(recv[starts[s] + seen[s] * rows: starts[s] + (seen[s] + 1) * rows])
        seen[s] += 1
    out = torch.cat(parts) if parts else recv
    return out.view(torch.float8_e4m3fn) if t.dtype == torch.float8_e4m3fn else out


def redistribute(model, layer: int, perm: torch.Tensor) -> None:
    """Relabel the experts of one MoE layer across the EP ranks (``perm[new] = old``): every rank permutes its
    replicated router rows and bias, and the stacked expert weights move to their new owners with one all-to-all
    per tensor (the reference moves per-expert tensors with one NCCL all_to_all, ``placement.py:89-128``).  All
    ranks call it with the same perm, in the same order."""
    L = model.layers[layer]
    pc = model.pctx
    E, ep = perm.numel(), pc.ep
    if ep == 1:
        return apply(model, layer, perm)
    assert L.moe
    group = getattr(pc, "group", None)
    p = perm.to(L.gate_b.device)
    if L.gate.kind == "f32" or L.gate.kind == "bf16":
        L.gate.w[:E] = L.gate.w[:E][p.to(L.gate.w.device)]
    L.gate_b.copy_(L.gate_b[p])
    if getattr(L, "gate_b_img", None) is not None:
        L.gate_b_img.copy_(L.gate_b_img[p.to(L.gate_b_img.device)])
    rank = pc.ep_rank
    if model.on_gpu:
        from ..ops.quant import Fp8Weight, pack_sf

        for name in ("e_w13", "e_w2"):
            W = getattr(L, name)
            q = _exchange_experts(W.q, perm, E, ep, rank, group)
            scale = _exchange_experts(W.scale.contiguous(), perm, E, ep, rank, group)
            setattr(L, name, Fp8Weight(q.contiguous(), pack_sf(scale.repeat_interleave(128, dim=0)[: q.shape[0]]),
                                       scale))
    else:
        L.e_w1 = _exchange_experts(L.e_w1.contiguous(), perm, E, ep, rank, group)
        L.e_w3 = _exchange_experts(L.e_w3.contiguous(), perm, E, ep, rank, group)
        L.e_w2 = _exchange_experts(L.e_w2.contiguous(), perm, E, ep, rank, group)


def rebalance(model, load: "ExpertLoad") -> Dict[int, tuple]:
    """Plan and apply a balanced placement for every MoE layer from the routing recorded since the last call.  The
    counts are summed over the EP ranks first, so every rank plans the same permutation; weights then move with
    ``redistribute`` (``apply`` on one rank).  Returns {layer: (imbalance before, after)}."""
    import torch.distributed as dist

    pc = model.pctx
    if model.n_weight_sets < model.cfg.n_layers:
        raise RuntimeError("rebalance needs untied layers: tied layers share one expert set")
    out = {}
    for layer in range(model.cfg.n_layers):
        if not model.layers[layer].moe:
            continue
        c = load.take(layer)
        if pc.world > 1:
            dev = model.device if dist.get_backend(getattr(pc, "group", None)) == "nccl" else torch.device("cpu")
            t = c.to(dev)
            dist.all_reduce(t, group=getattr(pc, "group", None))
            c = t.cpu()
        perm = plan(c, pc.ep)
        out[layer] = (imbalance(c, pc.ep), imbalance(c, pc.ep, perm))
        redistribute(model, layer, perm)
    return out

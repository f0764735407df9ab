"""Attention-side ops: MLA prefill (dense causal, optional DSA key mask), absorbed-MLA sparse attention over the
latent cache, and the DSA lightning indexer with top-k.

Semantics (oracle: ``ref.ops.causal_attention`` / ``indexer_logits`` / ``topk_mask``):

* prefill: q [T,H,dqk], k [T,H,dqk], v [T,H,dv] per sequence (``cu_seqlens``), causal, softmax scale; when
  ``key_mask`` is given (bool [T, Lmax] per sequence, True = allowed) keys outside the mask are dropped.  This is the
  DSA "top-k keys per query" rule evaluated inside a dense causal kernel, which for contexts up to a few top-k widths
  costs fewer FLOPs than the absorbed sparse form.
* absorbed sparse: q [T,H,dl+dr] against latent rows kv [S, dl+dr] selected by idx [T,K] (-1 = none);
  o_lat [T,H,dl] = softmax(q·kvᵀ·scale) · kv[:, :dl].  This is the decode / long-context path
  (reference: ``king_v10/bundle_v9/dec/cuda_decode_attn.py:20-116``, ``cuda_prefill_attn.py:1449``).
* indexer: logits[t,s] = Σ_h w[t,h]·relu(q[t,h]·k[s]) over each query's causal keys, top-k selection
  (reference: ``dec/cuda_paged_logits.py:115``, ``cuda_exact_topk.py:559``).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from ..ref import ops as R
from ._ext import ext


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: List[int], scale: float,
                      key_masks=None, version: int = 0, trace: Optional[torch.Tensor] = None,
                      sink: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reference-layout entry: q [T,H,dqk], k [T,H,dqk], v [T,H,dv]; sink [H]: per-head attention-sink logit."""
    T, H, dv = q.shape[0], q.shape[1], v.shape[2]
    if q.is_cuda and q.shape[2] == 192 and dv == 128:
        dn = 128
        kvb = torch.cat([k[..., :dn], v], dim=-1).contiguous()
        kpe = k[:, 0, dn:].contiguous()
        return mla_prefill(q, kvb, kpe, cu_seqlens, scale, key_masks, version, trace, sink)
    out = torch.empty(T, H, dv, dtype=torch.float32, device=q.device)
    if isinstance(key_masks, torch.Tensor):
        key_masks = unpack_key_mask(key_masks, cu_seqlens)
    for b in range(len(cu_seqlens) - 1):
        s, t = cu_seqlens[b], cu_seqlens[b + 1]
        pos = torch.arange(t - s, device=q.device)
        m = key_masks[b] if key_masks is not None else None
        out[s:t] = R.causal_attention(q[s:t], k[s:t], v[s:t], scale, pos, pos, m, sink=sink)
    return out


def mla_prefill(q: torch.Tensor, kvb: torch.Tensor, kpe: torch.Tensor, cu_seqlens: List[int], scale: float,
                key_masks=None, version: int = 0, trace: Optional[torch.Tensor] = None,
                sink: Optional[torch.Tensor] = None) -> torch.Tensor:
    """MLA prefill in the projection's own layout: q [T,H,192], kvb [T,H,256] = (k_nope | v) straight from the
    wkv_b GEMM, kpe [T,64] the shared RoPE key (k = [k_nope, kpe] per head). Returns o [T,H,128].
    version 1: one 128-row Q tile per CTA; 2: two Q tiles per CTA sharing each 128-key K/V tile; 3: two Q tiles,
    64-key steps with double-buffered S.  0 (default) picks by measurement on B200: 3 for DSA-masked calls (its
    shorter steps keep the masked softmax off the tensor pipe's critical path), 2 for dense causal ones."""
    T, H = q.shape[0], q.shape[1]
    if not q.is_cuda:
        dn = q.shape[2] - kpe.shape[-1]
        k = torch.cat([kvb[..., :dn], kpe.view(T, 1, kpe.shape[-1]).expand(T, H, kpe.shape[-1])], dim=-1)
        return prefill_attention(q, k, kvb[..., dn:], cu_seqlens, scale, key_masks, sink=sink)
    mask = None
    if isinstance(key_masks, torch.Tensor):
        mask = key_masks
    elif key_masks is not None and any(m is not None for m in key_masks):
        mask = pack_key_mask(key_masks, cu_seqlens, q.device)
    if version == 0:
        version = 3 if mask is not None else 2
    out = torch.empty(T, H, 128, dtype=torch.bfloat16, device=q.device)
    tiles = _device_tiles(cu_seqlens, 256 if version >= 2 else 128, q.device)
    ext().attn_prefill(q.contiguous(), kvb.contiguous(), kpe.contiguous(), tiles, mask, float(scale), out, None,
                       version, trace, sink.float().contiguous() if sink is not None else None)
    return out


_TILES = {}


def _device_tiles(cu_seqlens: List[int], bm: int, device) -> torch.Tensor:
    """``prefill_tiles`` on the device, cached by batch layout: every layer of a forward reuses one copy, and the
    first copy goes through pinned memory, so no layer waits on the host for a pageable transfer."""
    key = (tuple(cu_seqlens), bm, str(device))
    t = _TILES.get(key)
    if t is None:
        if len(_TILES) > 64:
            _TILES.clear()
        host = prefill_tiles(cu_seqlens, bm)
        if torch.cuda.is_available():
            host = host.pin_memory()
        t = host.to(device, non_blocking=True)
        _TILES[key] = t
    return t


def prefill_tiles(cu_seqlens: List[int], bm: int = 128) -> torch.Tensor:
    """(seq_start, seq_len, q0, 0) for every bm-query tile, longest causal work first (load balance)."""
    tiles = []
    for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:]):
        for q0 in range(0, b - a, bm):
            tiles.append((a, b - a, q0, 0))
    tiles.sort(key=lambda t: -t[2])
    return torch.tensor(tiles, dtype=torch.int32).view(-1, 4)


def pack_key_mask(key_masks, cu_seqlens, device, W: Optional[int] = None) -> torch.Tensor:
    """Per-sequence bool masks -> one uint32 bit matrix [T, W] (bit j of word w = key 32w+j)."""
    T = cu_seqlens[-1]
    Lmax = max([b - a for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:])] + [1])
    W = (Lmax + 31) // 32 if W is None else W
    bits = torch.zeros(T, W * 32, dtype=torch.bool, device=device)
    for b, m in enumerate(key_masks):
        s, t = cu_seqlens[b], cu_seqlens[b + 1]
        if m is None:
            bits[s:t, : t - s] = True
        else:
            bits[s:t, : t - s] = m
    w = bits.view(T, W, 32).to(torch.int64)
    shifts = torch.arange(32, device=device, dtype=torch.int64)
    words = (w << shifts).sum(-1)
    return words.to(torch.int64).bitwise_and(0xFFFFFFFF).to(torch.int32).contiguous()


def unpack_key_mask(words: torch.Tensor, cu_seqlens: List[int]) -> List[torch.Tensor]:
    shifts = torch.arange(32, device=words.device, dtype=torch.int64)
    bits = ((words.to(torch.int64)[..., None] >> shifts) & 1).bool().reshape(words.shape[0], words.shape[1] * 32)
    return [bits[a:b, : b - a] for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:])]


def indexer_prefill_mask(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, cu_seqlens: List[int],
                         topk: int, lmax: Optional[int] = None, fp8: bool = False) -> Optional[torch.Tensor]:
    """DSA selection for a prefill batch: per sequence, logits of every (query, causal key) pair and exact top-k.
    q [T, Hi, Di], k [T, Di], w [T, Hi]. Returns packed bits [T, ceil(Lmax/32)] (None when no sequence exceeds
    top-k, i.e. attention stays dense causal).  fp8: q and k are quantised to e4m3 (1x128 UE8M0 per row) and the
    logits run as block-scaled fp8 MMAs."""
    lens = [b - a for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:])]
    lmax = max(lens) if lmax is None else lmax
    if lmax <= topk:
        return None
    T, W = cu_seqlens[-1], (lmax + 31) // 32
    if q.is_cuda:
        if q.shape[1] % 16:
            raise ValueError("the indexer kernel needs a multiple of 16 indexer heads")
        e = ext()
        mask = torch.empty(T, W, dtype=torch.int32, device=q.device)
        for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:]):
            n = b - a
            ldo = (n + 3) // 4 * 4
            logits = torch.empty(n, ldo, dtype=torch.float32, device=q.device)
            if n > topk and fp8:
                from .quant import quant_act

                kq, ksf = quant_act(k[a:b].contiguous())
                qq, qsf = quant_act(q[a:b].reshape(n * q.shape[1], q.shape[2]).contiguous())
                e.indexer_logits_fp8(kq, ksf, qq, qsf, q.shape[1], w[a:b].float().contiguous(), logits, True)
            elif n > topk:
                e.indexer_logits(k[a:b].contiguous(), q[a:b].contiguous(), w[a:b].float().contiguous(), logits, True)
            e.topk_mask(logits, n, topk, mask, a)
        return mask
    masks = []
    if fp8:
        q, k = R.fake_quant_fp8_rows(q), R.fake_quant_fp8_rows(k)
    for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:]):
        n = b - a
        pos = torch.arange(n)
        lg = R.indexer_logits(q[a:b], k[a:b], w[a:b])
        masks.append(R.topk_mask(lg, pos, pos, topk))
    return pack_key_mask(masks, cu_seqlens, q.device, W)


def mla_splits(T: int, K: int, device) -> int:
    """Key splits so that T x 2 (value halves) x splits CTAs fill the SMs; each split keeps >= 128 keys."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    s = max(1, sms // max(1, 2 * T))
    return max(1, min(s, (K + 127) // 128))


def sparse_mla(q: torch.Tensor, kv: torch.Tensor, idx: torch.Tensor, scale: float, d_latent: int,
               sink: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Absorbed MQA over latent rows: q [T,H,D], kv [S,D] (or the fp8 cache rows, uint8 [S, row_bytes]), idx [T,K]
    int32 (-1 pad) -> o_lat [T,H,d_latent].  sink [H]: per-head attention-sink logit (an extra softmax denominator
    term).  fp8 rows run the kernel's fp16 path (q is rounded to fp16)."""
    T, H, D = q.shape
    f8 = kv.dtype == torch.uint8
    if q.is_cuda:
        e = ext()
        if D in (576, 512) and d_latent == 512 and H <= 128:
            out = torch.empty(T, H, d_latent, dtype=torch.bfloat16, device=q.device)
            splits = mla_splits(T, idx.shape[1], q.device)
            work = torch.empty(T * splits * H * 514, dtype=torch.float32, device=q.device) if splits > 1 else None
            qk = q.to(torch.float16 if f8 else torch.bfloat16).contiguous()
            e.sparse_mla(qk, kv, idx, float(scale), splits, work, out,
                         sink.float().contiguous() if sink is not None else None)
            return out
        raise RuntimeError("sparse_mla: the tcgen05 kernel needs D=576 (512 latent + 64 RoPE key) or D=512 (latent "
                           "MQA), d_latent=512, H<=128")
    mla = D > d_latent
    out = torch.zeros(T, H, d_latent)
    for t in range(T):
        sel = idx[t][idx[t] >= 0].long()
        if sel.numel() == 0:
            continue
        keys = R.dequant_latent_fp8(kv[sel], d_latent, D - d_latent if mla else 0, mla) if f8 else kv[sel].float()
        s = (q[t].float() @ keys.t()) * scale
        if sink is not None:
            s = torch.cat([s, sink.float()[:, None]], dim=-1)
            p = torch.softmax(s, dim=-1)[:, :-1]
        else:
            p = torch.softmax(s, dim=-1)
        out[t] = p @ keys[:, :d_latent]
    return out


def indexer_prefill_slots(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, cu_seqlens: List[int], topk: int,
                          slots: torch.Tensor, fp8: bool = False) -> torch.Tensor:
    """DSA selection of a prefill batch as cache slots (the sparse-prefill form of ``indexer_prefill_mask``): for
    every query, the slots of its top-k causal keys, in key order, -1 padded; all causal keys when a query has at
    most topk.  q [T, Hi, Di], k [T, Di], w [T, Hi]; slots [T] the cache slot of every token of the batch (the
    sequences are contiguous runs of it).  Returns [T, topk] int32."""
    T = cu_seqlens[-1]
    out = torch.full((T, topk), -1, dtype=torch.int32, device=q.device)
    if q.is_cuda:
        if q.shape[1] % 16:
            raise ValueError("the indexer kernel needs a multiple of 16 indexer heads")
        e = ext()
        for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:]):
            n = b - a
            if n == 0:
                continue
            ldo = (n + 3) // 4 * 4
            logits = torch.empty(n, ldo, dtype=torch.float32, device=q.device)
            if n > topk and fp8:
                from .quant import quant_act

                kq, ksf = quant_act(k[a:b].contiguous())
                qq, qsf = quant_act(q[a:b].reshape(n * q.shape[1], q.shape[2]).contiguous())
                e.indexer_logits_fp8(kq, ksf, qq, qsf, q.shape[1], w[a:b].float().contiguous(), logits, True)
            elif n > topk:
                e.indexer_logits(k[a:b].contiguous(), q[a:b].contiguous(), w[a:b].float().contiguous(), logits, True)
            e.topk_causal_slots(logits, slots[a:b].to(torch.int32).contiguous(), 0, out[a:b])
        return out
    if fp8:
        q, k = R.fake_quant_fp8_rows(q), R.fake_quant_fp8_rows(k)
    for a, b in zip(cu_seqlens[:-1], cu_seqlens[1:]):
        n = b - a
        if n == 0:
            continue
        pos = torch.arange(n)
        m = R.topk_mask(R.indexer_logits(q[a:b], k[a:b], w[a:b]), pos, pos, topk)     # [n, n] bool
        for i in range(n):
            sel = torch.nonzero(m[i], as_tuple=False).flatten()
            out[a + i, : sel.numel()] = slots[a:b][sel].to(torch.int32)
    return out


def indexer_topk(q: torch.Tensor, w: torch.Tensor, kcache: torch.Tensor, key_slots: torch.Tensor,
                 n_keys: torch.Tensor, topk: int) -> torch.Tensor:
    """For each query t: keys are ``key_slots[t, :n_keys[t]]`` (slots of ``kcache``), in causal order.
    Returns the selected slots [T, topk] (-1 pad), ordered by descending logit (ties -> lower key index)."""
    T = q.shape[0]
    if q.is_cuda:
        e = ext()
        if hasattr(e, "indexer_topk"):
            out = torch.empty(T, topk, dtype=torch.int32, device=q.device)
            e.indexer_topk(q, w, kcache, key_slots, n_keys, out)
            return out
        # temporary batched path until the fused indexer kernel is registered (no host sync: graph-capturable)
        kk = min(topk, key_slots.shape[1])
        keys = kcache[key_slots.clamp(min=0).long()].float()                       # [T, L, Di]
        s = torch.einsum("thd,tld->thl", q.float(), keys).clamp_(min=0)
        logits = torch.einsum("thl,th->tl", s, w.float())
        valid = torch.arange(key_slots.shape[1], device=q.device)[None, :] < n_keys[:, None]
        logits = logits.masked_fill(~valid, float("-inf"))
        top = torch.topk(logits, kk, dim=-1)
        sel = torch.gather(key_slots, 1, top.indices).masked_fill(torch.isinf(top.values), -1)
        out = torch.full((T, topk), -1, dtype=torch.int32, device=q.device)
        out[:, :kk] = sel
        return out
    out = torch.full((T, topk), -1, dtype=torch.int32, device=q.device)
    for t in range(T):
        n = int(n_keys[t])
        slots = key_slots[t, :n].long()
        k = kcache[slots].float()
        logits = R.indexer_logits(q[t:t + 1].float(), k, w[t:t + 1].float())[0]
        kk = min(topk, n)
        order = torch.sort(-logits, stable=True).indices[:kk]
        out[t, :kk] = slots[order].to(torch.int32)
    return out

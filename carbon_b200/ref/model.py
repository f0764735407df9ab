"""CPU fp32 oracle of the whole model (the tiny CPU model's reference and the source of truth for every GPU path).

The model is a DeepSeek-V3/V4-style decoder:

* **mHC residual**: the residual is ``hc`` parallel streams ``X [T, hc, D]``.  Each sublayer reads
  ``y = Σ pre_i X_i`` (then RMSNorm) and writes ``X'_o = post_o·F(y) + Σ_i comb[i][o] X_i`` with (pre, post, comb)
  computed from ``X`` itself (``ref.ops.mhc_coeffs``).  This is the computation behind the reference's mHC boundary
  kernels (``king_v10/bundle_v9/cuda_mhc_packed.py:40-170``, ``cuda_sinkhorn.py:150-190``).
* **MLA attention** (q_lora → q, kv_lora latent + shared RoPE key), optionally **DSA sparse**: a lightning indexer
  scores keys and each query attends only to its top-k keys (``dec/cuda_paged_logits.py:35-37``,
  ``exact_topk.py:14``).
* **MoE**: biased top-k router + routed SwiGLU experts + shared expert (``moe_route.py:166-216``).

This module is deliberately naive: full-sequence recompute, no cache, fp32 everywhere.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Dict, List, Tuple

import torch

from ..config import ModelConfig
from . import ops


# ----------------------------------------------------------------------------------------------------------------------
# parameter declaration (this order is the random-init order; names are the checkpoint format)
# ----------------------------------------------------------------------------------------------------------------------
def param_shapes(cfg: ModelConfig) -> "OrderedDict[str, Tuple[Tuple[int, ...], str]]":
    """name -> (shape, init) with init in {"normal", "ones", "zeros"}."""
    D, H, hc = cfg.hidden_size, cfg.n_heads, cfg.hc_streams
    p: "OrderedDict[str, Tuple[Tuple[int, ...], str]]" = OrderedDict()
    p["embed.weight"] = ((cfg.vocab_size, D), "normal")
    for i in range(cfg.n_layers):
        L = f"layers.{i}."
        for sub in (() if cfg.plain_residual else ("attn_hc", "ffn_hc")):
            p[L + sub + ".fn"] = ((cfg.hc_mix_dim, hc * D), "normal")
            p[L + sub + ".base"] = ((cfg.hc_mix_dim,), "normal")
            p[L + sub + ".scale"] = ((3,), "ones")
        p[L + "attn_norm.weight"] = ((D,), "ones")
        if i in cfg.engram_layers:
            p[L + "engram.table"] = ((cfg.engram_table_rows, cfg.engram_dim), "normal")
            p[L + "engram.wkv.weight"] = (((hc + 1) * D, cfg.engram_cols * cfg.engram_dim), "normal")
            p[L + "engram.q_weight"] = ((D,), "ones")
            p[L + "engram.k_weight"] = ((D,), "ones")
        if cfg.q_lora_rank > 0:
            p[L + "attn.wq_a.weight"] = ((cfg.q_lora_rank, D), "normal")
            p[L + "attn.q_norm.weight"] = ((cfg.q_lora_rank,), "ones")
            p[L + "attn.wq_b.weight"] = ((H * cfg.qk_head_dim, cfg.q_lora_rank), "normal")
        else:
            p[L + "attn.wq.weight"] = ((H * cfg.qk_head_dim, D), "normal")
        p[L + "attn.wkv_a.weight"] = ((cfg.latent_dim, D), "normal")
        p[L + "attn.kv_norm.weight"] = ((cfg.kv_lora_rank,), "ones")
        if cfg.attn_kind == "mla":
            p[L + "attn.wkv_b.weight"] = ((H * (cfg.qk_nope_head_dim + cfg.v_head_dim), cfg.kv_lora_rank), "normal")
        if cfg.o_groups:
            G = cfg.o_groups
            p[L + "attn.wo_a.weight"] = ((G, cfg.o_lora_rank, H // G * cfg.head_out_dim), "normal")
            p[L + "attn.wo_b.weight"] = ((D, G * cfg.o_lora_rank), "normal")
        else:
            p[L + "attn.wo.weight"] = ((D, H * cfg.head_out_dim), "normal")
        if cfg.attn_sink:
            p[L + "attn.sink"] = ((H,), "normal")
        if cfg.has_indexer(i):
            qin = cfg.q_lora_rank if cfg.q_lora_rank > 0 else D
            p[L + "attn.indexer.wq.weight"] = ((cfg.index_n_heads * cfg.index_head_dim, qin), "normal")
            p[L + "attn.indexer.wk.weight"] = ((cfg.index_head_dim, D), "normal")
            p[L + "attn.indexer.k_norm.weight"] = ((cfg.index_head_dim,), "ones")
            p[L + "attn.indexer.k_norm.bias"] = ((cfg.index_head_dim,), "zeros")
            p[L + "attn.indexer.weights_proj.weight"] = ((cfg.index_n_heads, D), "normal")
        p[L + "ffn_norm.weight"] = ((D,), "ones")
        if cfg.is_moe_layer(i):
            E, I = cfg.n_routed_experts, cfg.moe_intermediate
            p[L + "ffn.gate.weight"] = ((E, D), "normal")
            p[L + "ffn.gate.bias"] = ((E,), "normal")
            if cfg.image_token_id >= 0:
                p[L + "ffn.gate.bias_img"] = ((E,), "normal")
            p[L + "ffn.experts.w1"] = ((E, I, D), "normal")
            p[L + "ffn.experts.w3"] = ((E, I, D), "normal")
            p[L + "ffn.experts.w2"] = ((E, D, I), "normal")
            if cfg.n_shared_experts > 0:
                Is = I * cfg.n_shared_experts
                p[L + "ffn.shared.w1"] = ((Is, D), "normal")
                p[L + "ffn.shared.w3"] = ((Is, D), "normal")
                p[L + "ffn.shared.w2"] = ((D, Is), "normal")
        else:
            I = cfg.dense_intermediate
            p[L + "ffn.w1"] = ((I, D), "normal")
            p[L + "ffn.w3"] = ((I, D), "normal")
            p[L + "ffn.w2"] = ((D, I), "normal")
    if not cfg.plain_residual:
        p["head_hc.fn"] = ((hc, hc * D), "normal")
        p["head_hc.base"] = ((hc,), "normal")
        p["head_hc.scale"] = ((1,), "ones")
    p["norm.weight"] = ((D,), "ones")
    p["head.weight"] = ((cfg.vocab_size, D), "normal")
    return p


def init_weights(cfg: ModelConfig, seed: int = 0, device="cpu", dtype=torch.float32) -> Dict[str, torch.Tensor]:
    """Seeded random init: every "normal" tensor ~ N(0, init_std²), drawn in declaration order from one generator."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out: Dict[str, torch.Tensor] = {}
    for name, (shape, kind) in param_shapes(cfg).items():
        if kind == "normal":
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * cfg.init_std
        elif kind == "ones":
            t = torch.ones(shape, device=device, dtype=torch.float32)
        else:
            t = torch.zeros(shape, device=device, dtype=torch.float32)
        out[name] = t.to(dtype)
    return out


# ----------------------------------------------------------------------------------------------------------------------
# forward
# ----------------------------------------------------------------------------------------------------------------------
class RefModel:
    """Naive full-sequence fp32 model. ``forward(ids)`` for one sequence returns logits [S, V]."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, torch.Tensor]):
        self.cfg = cfg
        self.w = {k: v.float() for k, v in weights.items()}
        self.forced_routing = None   # {layer: ids [T, k]}: use these expert choices instead of the router's top-k
        self.forced_dsa = None       # {layer: positions [T, topk] (-1 pad)}: use this DSA selection instead
        self._dsa = {}               # DSA selection of each index-source layer in the current forward

    # -- sublayers -------------------------------------------------------------------------------------------------
    def attention(self, i: int, h: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        L = f"layers.{i}.attn."
        T, H = h.shape[0], cfg.n_heads
        dr, r, dq = cfg.qk_rope_head_dim, cfg.kv_lora_rank, cfg.qk_head_dim
        if cfg.q_lora_rank > 0:
            q_lat = ops.rms_norm(h @ w[L + "wq_a.weight"].t(), w[L + "q_norm.weight"], cfg.rms_eps)
            q = (q_lat @ w[L + "wq_b.weight"].t()).view(T, H, dq)
        else:
            q_lat = h
            q = (h @ w[L + "wq.weight"].t()).view(T, H, dq)
        dn = dq - dr                                  # non-RoPE part of q
        qf = torch.cat([q[..., :dn], ops.apply_rope(q[..., dn:], pos, cfg.rope)], dim=-1)
        kv = h @ w[L + "wkv_a.weight"].t()
        if cfg.attn_kind == "latent_mqa":
            # one shared head: the normalised latent, RoPE on its last dr dims; value = the same row
            kv_c = ops.rms_norm(kv, w[L + "kv_norm.weight"], cfg.rms_eps)
            k = torch.cat([kv_c[:, :r - dr], ops.apply_rope(kv_c[:, None, r - dr:], pos, cfg.rope)[:, 0]],
                          dim=-1)[:, None, :]                                   # [T,1,r]
            v = k
        else:
            dv = cfg.v_head_dim
            kv_c = ops.rms_norm(kv[:, :r], w[L + "kv_norm.weight"], cfg.rms_eps)
            k_pe = ops.apply_rope(kv[:, None, r:], pos, cfg.rope)         # [T,1,dr]
            kvb = (kv_c @ w[L + "wkv_b.weight"].t()).view(T, H, dn + dv)
            k = torch.cat([kvb[..., :dn], k_pe.expand(T, H, dr)], dim=-1)
            v = kvb[..., dn:]
        W = cfg.swa_window
        window = None
        if W > 0:
            window = (pos[None, :] > pos[:, None] - W) & (pos[None, :] <= pos[:, None])
        allowed = None
        src = cfg.index_source(i)
        if src == i:
            logits = self.indexer_logits(i, h, q_lat, pos)
            if window is not None:                      # top-k over the keys older than the window
                logits = logits.masked_fill(window, float("-inf"))
            allowed = ops.topk_mask(logits, pos, pos, cfg.index_topk)
            if self.forced_dsa is not None and i in self.forced_dsa:
                sel = self.forced_dsa[i].long()
                allowed = torch.zeros(T, T + 1, dtype=torch.bool)          # column T collects the -1 pads
                allowed.scatter_(1, torch.where(sel >= 0, sel, T), True)
                allowed = allowed[:, :T]
            if window is not None:
                allowed = allowed & ~window
            self._dsa[i] = allowed
        elif src is not None:
            allowed = self._dsa[src]           # shared selection of the source layer
        if window is not None:
            allowed = window if allowed is None else (allowed | window)
        sink = w[L + "sink"] if cfg.attn_sink else None
        o = ops.causal_attention(qf, k, v, cfg.softmax_scale, pos, pos, allowed, sink=sink)   # [T,H,dvh]
        if cfg.attn_kind == "latent_mqa":
            # the value's RoPE dims carry each key's rotation: rotate the output back by the query position
            o = torch.cat([o[..., :r - dr], ops.apply_rope(o[..., r - dr:], pos, cfg.rope, inverse=True)],
                          dim=-1)
        return self.out_proj(i, o)

    def out_proj(self, i: int, o: torch.Tensor) -> torch.Tensor:
        """o [T, H, dvh] -> [T, D]: one dense wo, or the grouped low-rank wo_a (per group of heads) then wo_b."""
        cfg, w = self.cfg, self.w
        L = f"layers.{i}.attn."
        T, H = o.shape[0], o.shape[1]
        if not cfg.o_groups:
            return o.reshape(T, o.shape[1] * o.shape[2]) @ w[L + "wo.weight"].t()
        G = cfg.o_groups
        og = o.reshape(T, G, -1)                                                # [T, G, (H/G)*dvh]
        z = torch.einsum("tgk,gnk->tgn", og, w[L + "wo_a.weight"])              # [T, G, o_lora]
        return z.reshape(T, z.shape[1] * z.shape[2]) @ w[L + "wo_b.weight"].t()

    def indexer_logits(self, i: int, h: torch.Tensor, q_lat: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        q, k, wt = self.indexer_qkw(i, h, q_lat, pos)
        return ops.indexer_logits(q, k, wt)

    def indexer_qkw(self, i, h, q_lat, pos):
        cfg, w = self.cfg, self.w
        L = f"layers.{i}.attn.indexer."
        T, Hi, Di, dr = h.shape[0], cfg.index_n_heads, cfg.index_head_dim, cfg.qk_rope_head_dim
        q = (q_lat @ w[L + "wq.weight"].t()).view(T, Hi, Di)
        q = torch.cat([ops.apply_rope(q[..., :dr], pos, cfg.rope), q[..., dr:]], dim=-1)
        k = ops.layer_norm(h @ w[L + "wk.weight"].t(), w[L + "k_norm.weight"], w[L + "k_norm.bias"], 1e-6)
        k = torch.cat([ops.apply_rope(k[:, None, :dr], pos, cfg.rope)[:, 0], k[:, dr:]], dim=-1)
        wt = (h @ w[L + "weights_proj.weight"].t()) * (Hi ** -0.5) * (Di ** -0.5)
        if cfg.index_fp4:
            q, k = ops.fake_quant_mxfp4(q), ops.fake_quant_mxfp4(k)
        elif cfg.index_fp8:
            q, k = ops.fake_quant_fp8_rows(q), ops.fake_quant_fp8_rows(k)
        return q, k, wt

    def ffn(self, i: int, h: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        L = f"layers.{i}.ffn."
        if not cfg.is_moe_layer(i):
            return ops.swiglu(h @ w[L + "w1"].t(), h @ w[L + "w3"].t(), cfg.swiglu_limit) @ w[L + "w2"].t()
        logits = h @ w[L + "gate.weight"].t()
        bias = w[L + "gate.bias"]
        if cfg.image_token_id >= 0:             # image tokens rank with their own bias
            is_img = (self._ids.long() == cfg.image_token_id)[:, None]
            bias = torch.where(is_img, w[L + "gate.bias_img"][None, :], bias[None, :])
        wts, ids = ops.router_topk(logits, bias, cfg.n_activated_experts, cfg.score_func,
                                   cfg.route_scale, cfg.norm_topk_prob, cfg.n_groups, cfg.topk_groups)
        if self.forced_routing is not None and i in self.forced_routing:
            ids = self.forced_routing[i].to(ids.dtype)
            act = torch.sigmoid(logits) if cfg.score_func == "sigmoid" else (
                torch.sqrt(ops.softplus(logits)) if cfg.score_func == "sqrtsoftplus" else torch.softmax(logits, -1))
            wts = act.gather(1, ids.long())
            if cfg.norm_topk_prob:
                wts = wts / (wts.sum(-1, keepdim=True) + 1e-20)
            wts = wts * cfg.route_scale
        out = torch.zeros_like(h)
        for e in range(cfg.n_routed_experts):
            rows, slot = torch.nonzero(ids == e, as_tuple=True)
            if rows.numel() == 0:
                continue
            x = h[rows]
            y = ops.swiglu(x @ w[L + "experts.w1"][e].t(), x @ w[L + "experts.w3"][e].t(), cfg.swiglu_limit)
            y = y @ w[L + "experts.w2"][e].t()
            out.index_add_(0, rows, y * wts[rows, slot][:, None])
        if cfg.n_shared_experts > 0:
            out = out + ops.swiglu(h @ w[L + "shared.w1"].t(), h @ w[L + "shared.w3"].t(),
                                   cfg.swiglu_limit) @ w[L + "shared.w2"].t()
        return out

    def hc_sublayer(self, X, prefix: str, norm_w: torch.Tensor, fn_apply) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        if cfg.plain_residual:                  # x + f(RMSNorm(x)·w)
            return X + fn_apply(ops.rms_norm(X[:, 0], norm_w, cfg.rms_eps))[:, None]
        pre, post, comb = ops.mhc_coeffs(X, w[prefix + ".fn"], w[prefix + ".base"], w[prefix + ".scale"],
                                         cfg.hc_mult, cfg.sinkhorn_iters, cfg.hc_eps, cfg.rms_eps)
        y = ops.rms_norm(ops.mhc_pre_mix(X, pre), norm_w, cfg.rms_eps)
        return ops.mhc_post_mix(X, fn_apply(y), post, comb)

    # -- whole model -----------------------------------------------------------------------------------------------
    def forward(self, ids: torch.Tensor, pos: torch.Tensor = None, late_from: int = None) -> torch.Tensor:
        """late_from: first position that exists at the late layers (bounded replay; default: the prompt's last
        late_replay tokens).  Returns logits of the tokens that reach the head."""
        cfg, w = self.cfg, self.w
        T = ids.shape[0]
        pos = torch.arange(T) if pos is None else pos
        self._dsa = {}
        self._ids = ids
        X = w["embed.weight"][ids.long()][:, None, :].expand(T, cfg.hc_streams, cfg.hidden_size).clone()
        for i in range(cfg.n_layers):
            if i == cfg.late_layer_start:
                lf = max(0, T - cfg.late_replay) if late_from is None else late_from
                keep = pos >= lf
                X, pos, ids = X[keep], pos[keep], ids[keep]
                self._ids = ids
            L = f"layers.{i}."
            if i in cfg.engram_layers:
                X = self.engram(i, X, ids, pos)
            X = self.hc_sublayer(X, L + "attn_hc", w[L + "attn_norm.weight"], lambda y: self.attention(i, y, pos))
            X = self.hc_sublayer(X, L + "ffn_hc", w[L + "ffn_norm.weight"], lambda y: self.ffn(i, y))
        return self.head(X)

    def engram(self, i: int, X: torch.Tensor, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Hashed n-gram memory on the residual streams (one sequence: ids in position order)."""
        cfg, w = self.cfg, self.w
        L = f"layers.{i}.engram."
        T = ids.shape[0]
        nmax = max(cfg.engram_orders)
        back = torch.arange(nmax)
        src = torch.arange(T)[:, None] - back[None, :]
        window = torch.where(pos[:, None] - back[None, :] >= 0, ids.long()[src.clamp(min=0)], -1)
        rows = ops.engram_hash_ids(window, cfg.engram_orders, cfg.engram_heads, cfg.engram_primes, cfg.vocab_size)
        emb = w[L + "table"][rows].reshape(T, -1)                                  # [T, cols * dim]
        kv = emb @ w[L + "wkv.weight"].t()
        Xn = ops.engram_gate(X, kv, w[L + "q_weight"], w[L + "k_weight"], cfg.rms_eps, cfg.engram_clamp)
        if cfg.image_token_id >= 0:             # image tokens take no n-gram memory update
            Xn = torch.where((ids.long() == cfg.image_token_id)[:, None, None], X, Xn)
        return Xn

    def head(self, X: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        if cfg.plain_residual:
            return ops.rms_norm(X[:, 0], w["norm.weight"], cfg.rms_eps) @ w["head.weight"].t()
        pre = ops.mhc_head_coeffs(X, w["head_hc.fn"], w["head_hc.base"], w["head_hc.scale"], cfg.hc_eps, cfg.rms_eps)
        y = ops.rms_norm(ops.mhc_pre_mix(X, pre), w["norm.weight"], cfg.rms_eps)
        return y @ w["head.weight"].t()

    def greedy(self, prompt: torch.Tensor, n_new: int) -> Tuple[List[int], List[torch.Tensor]]:
        """Recompute-everything greedy decode. Returns (new token ids, last-position logits of every step)."""
        ids = prompt.clone()
        toks, logits = [], []
        late_from = max(0, prompt.shape[0] - self.cfg.late_replay)     # fixed by the prompt (bounded replay)
        for _ in range(n_new + 1):
            lg = self.forward(ids, late_from=late_from)[-1]
            logits.append(lg)
            if len(toks) == n_new:
                break
            nxt = int(torch.argmax(lg))
            toks.append(nxt)
            ids = torch.cat([ids, torch.tensor([nxt], dtype=ids.dtype)])
        return toks, logits

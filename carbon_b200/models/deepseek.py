"""DeepSeek-V3/V4-style model graph (MLA + DSA indexer + MoE + mHC) for the serving engine.

One implementation runs on two kinds of device tensors:

* CPU fp32 — every op resolves to the oracle math in ``carbon_b200.ref``; used to test the engine logic (paged
  latent cache, absorbed decode, batching) against the naive full-recompute oracle (the tiny CPU model).
* CUDA (B200) — bf16 activations, block-scaled fp8 weights (128×128 UE8M0) and the sm_100a kernels in
  ``carbon_b200._C``.

Layer structure (reference engine: ``sglang.srt.models.deepseek_v4`` patched by ``king_v10/bundle_v9/slots.py``):
``X [T, hc, D]`` → mHC boundary (coeffs from X) → RMSNorm → MLA attention (+ indexer top-k) → post-mix →
mHC boundary → RMSNorm → dense SwiGLU FFN or MoE (router top-k, routed experts, shared expert) → post-mix.
Prefill uses the non-absorbed MLA form (k/v from wkv_b); decode uses the absorbed form over the latent cache.

Parallelism: attention heads are split over TP ranks, experts over EP ranks (``carbon_b200.parallel``); with one
rank every collective is the identity.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from ..config import ModelConfig
from ..ops import attention as A
from ..ops import core as C
from ..ops.gemm import bf16_gemm, fp8_gemm, fp8_gemm_swiglu, interleave_gate_up
from ..ops.quant import Fp8Weight, gather_rows_fp8, quant_act, quantize_weight, stack_weights
from ..ref import ops as R
from ..utils.trace import region
from .weights import WeightSource


# ----------------------------------------------------------------------------------------------------------------------
# linear layers
# ----------------------------------------------------------------------------------------------------------------------
class Lin:
    """y = x·Wᵀ. CPU: fp32 weight. CUDA: block-scaled fp8 (default) or bf16."""

    def __init__(self, w: torch.Tensor, device: torch.device, fp8: bool = True):
        self.out_features, self.in_features = w.shape
        if device.type == "cpu":
            self.kind, self.w = "f32", w.float()
        elif fp8 and self.in_features % 128 == 0:
            self.kind, self.fw = "fp8", quantize_weight(w.to(device))
        else:
            # bf16 GEMM tiles need N % 16 == 0: pad the weight rows with zeros and slice the output
            self.kind = "bf16"
            n_pad = (-self.out_features) % 16
            wp = torch.nn.functional.pad(w.float(), (0, 0, 0, n_pad)) if n_pad else w
            self.w = wp.to(device=device, dtype=torch.bfloat16).contiguous()

    def __call__(self, x: torch.Tensor, out_dtype=torch.bfloat16, xq=None) -> torch.Tensor:
        if self.kind == "f32":
            return x.float() @ self.w.t()
        if self.kind == "fp8":
            q, sf = xq if xq is not None else quant_act(x)
            return fp8_gemm(q, sf, self.fw, out_dtype=out_dtype)
        y = bf16_gemm(x, self.w, out_dtype=out_dtype)
        return y if y.shape[1] == self.out_features else y[:, : self.out_features]


class SwigluFFN:
    """down(silu(gate(x)) * up(x)). CUDA: one fp8 GEMM with the SwiGLU+requant epilogue, then the down GEMM."""

    def __init__(self, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, device, limit: float):
        self.limit = limit
        if device.type == "cpu":
            self.kind = "f32"
            self.w1, self.w3, self.w2 = w1.float(), w3.float(), w2.float()
        else:
            self.kind = "fp8"
            self.w13 = quantize_weight(interleave_gate_up(w1.to(device), w3.to(device)))
            self.w2 = quantize_weight(w2.to(device))

    def __call__(self, x: torch.Tensor, xq=None) -> torch.Tensor:
        if self.kind == "f32":
            return R.swiglu(x @ self.w1.t(), x @ self.w3.t(), self.limit) @ self.w2.t()
        q, sf = xq if xq is not None else quant_act(x)
        act, act_sf = fp8_gemm_swiglu(q, sf, self.w13, self.limit)
        return fp8_gemm(act, act_sf, self.w2)


@dataclass
class HCParams:
    fn: torch.Tensor        # CPU: fp32 [nmix, hc*D]; CUDA: bf16 [64, hc*D] = [hi; lo; 0-pad]
    base: torch.Tensor
    scale: torch.Tensor
    nmix: int


def make_hc(fn, base, scale, device) -> HCParams:
    nmix = fn.shape[0]
    if device.type == "cpu":
        return HCParams(fn.float(), base.float(), scale.float(), nmix)
    hl = C.split_hi_lo(fn.to(device))
    rows = ((2 * nmix + 15) // 16) * 16
    pad = torch.zeros(rows, fn.shape[1], dtype=torch.bfloat16, device=device)
    pad[: 2 * nmix] = hl
    return HCParams(pad, base.to(device).float(), scale.to(device).float(), nmix)


# ----------------------------------------------------------------------------------------------------------------------
# forward batch / cache
# ----------------------------------------------------------------------------------------------------------------------
@dataclass
class ForwardBatch:
    ids: torch.Tensor                      # [T] int32
    pos: torch.Tensor                      # [T] int32 position of each token in its sequence
    out_loc: torch.Tensor                  # [T] int32 cache slot each token's KV is written to
    is_prefill: bool
    cu_seqlens: Optional[List[int]] = None  # prefill: host boundaries of the sequences in `ids`
    key_slots: Optional[torch.Tensor] = None  # decode: [B, Lmax] int32 slots of every key (incl. the new token)
    n_keys: Optional[torch.Tensor] = None     # decode: [B] int32
    logits_rows: Optional[torch.Tensor] = None  # rows that need logits (default: all)
    bounds: Optional[List[int]] = None          # per-rank token shard bounds (multi-rank; sequence-aligned)
    late_from: Optional[torch.Tensor] = None    # decode: [B] first position that exists at the late layers


class Layer:
    pass


class Pending:
    """A tensor being produced on a side stream; ``get()`` joins the side stream into the current one."""

    def __init__(self, tensor: torch.Tensor, stream):
        self.tensor, self.stream = tensor, stream

    def get(self) -> torch.Tensor:
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.stream)
        self.tensor.record_stream(cur)
        return self.tensor


def resolve(x):
    return x.get() if isinstance(x, Pending) else x


class DeepseekModel:
    def __init__(self, cfg: ModelConfig, source: WeightSource, device="cpu", fp8: bool = True,
                 pctx=None):
        from ..parallel.context import ParallelCtx

        self.cfg = cfg
        self.device = torch.device(device)
        self.on_gpu = self.device.type == "cuda"
        if cfg.plain_residual and cfg.engram_layers and self.on_gpu:
            raise NotImplementedError("Engram on the GPU gates the mHC streams; plain-residual models (hc_mult=0) "
                                      "with Engram layers run on the CPU engine only")
        self.pctx = pctx if pctx is not None else ParallelCtx.single()
        self.fp8 = fp8
        self.trace = None          # set to a list to record (name, tensor) at sublayer boundaries (debugging)
        self.expert_load = None    # placement.ExpertLoad: per-layer routing counts for expert rebalancing
        self.owner_kv = False      # only a request's home rank caches its KV (no all-gather of the new rows)
        self._side = None          # side stream of the shared expert
        self._dsa = {}
        self._early_sel: Dict[int, Pending] = {}   # decode DSA selections started before the query projections
        cfg.validate()
        if cfg.swa_window and cfg.attn_kind != "latent_mqa":
            raise NotImplementedError("swa_window is served by the latent-MQA attention path only")
        tp, ep = self.pctx.tp, self.pctx.ep
        # TP attention whose output projection runs on each token's owner after a heads -> tokens all-to-all
        self.o_a2a = bool(getattr(self.pctx, "oproj_a2a", False)) and tp > 1
        self.H_local = cfg.n_heads // tp
        self.E_local = cfg.n_routed_experts // ep if cfg.n_routed_experts else 0
        dev = self.device
        get = lambda n, rows=None: source.get(n, dev, rows)
        self.cos_sin = C.rope_table(cfg.max_position, cfg.qk_rope_head_dim, cfg.rope, dev)
        self.act_dtype = torch.bfloat16 if self.on_gpu else torch.float32
        # vocab-parallel embedding/head: each rank keeps rows [v_lo, v_hi)
        V = cfg.vocab_size
        vs = (V + self.pctx.world - 1) // self.pctx.world if self.pctx.vocab_parallel else V
        self.v_lo = self.pctx.rank * vs if self.pctx.vocab_parallel else 0
        self.v_hi = min(V, self.v_lo + vs)
        self.embed = get("embed.weight", slice(self.v_lo, self.v_hi)).to(self.act_dtype).contiguous()
        self.head_w = Lin(get("head.weight", slice(self.v_lo, self.v_hi)), dev, fp8=False)
        self.head_hc = None if cfg.plain_residual else \
            make_hc(get("head_hc.fn"), get("head_hc.base"), get("head_hc.scale"), dev)
        self.norm_w = get("norm.weight")
        # layers whose weights are tied (WeightSource.layer_sets) share one Layer object
        built: Dict[str, Layer] = {}
        self.layers = []
        for i in range(cfg.n_layers):
            key = source.canonical(f"layers.{i}.")
            if key not in built:
                built[key] = self._load_layer(i, get)
            self.layers.append(built[key])
        self.n_weight_sets = len(built)

    # ------------------------------------------------------------------------------------------------------------------
    def _load_engram(self, prefix: str, get):
        """Engram weights: the hashed table (GPU: e4m3 rows + UE8M0 per 32, the gather kernel's format), the wkv
        projection, the gate's q / k norm weights."""
        E = Layer()
        cfg, pc = self.cfg, self.pctx
        table = get(prefix + "table")
        if self.on_gpu and getattr(pc, "heap", None) is not None and pc.world > 1:
            # split by whole hash columns over the ranks, each shard in the symmetric heap: the gather kernel reads a
            # row from its owner's HBM over NVLink (no table replica, no lookup collective)
            cb = [0]
            for pr in cfg.engram_primes:
                cb.append(cb[-1] + pr)
            C, W = cfg.engram_cols, pc.world
            cpr = (C + W - 1) // W
            bounds = [cb[min(C, r * cpr)] for r in range(W)] + [cb[C]]
            rows_max = max(bounds[r + 1] - bounds[r] for r in range(W))
            lo, hi = bounds[pc.rank], bounds[pc.rank + 1]
            q, sf = R.quant_fp8_rows32(table[lo:hi])
            bd = pc.heap.alloc((max(rows_max, 1), cfg.engram_dim), torch.float8_e4m3fn)
            bs = pc.heap.alloc((max(rows_max, 1), cfg.engram_dim // 32), torch.uint8)
            bd.local[:hi - lo].copy_(q)
            bs.local[:hi - lo].copy_(sf)
            E.shards = (bd, bs)
            E.data_ptrs, E.sf_ptrs = bd.peers, bs.peers
            E.bounds = torch.tensor(bounds, dtype=torch.int32, device=self.device)
        elif self.on_gpu:
            q, sf = R.quant_fp8_rows32(table)
            E.data, E.sf = q.contiguous(), sf.contiguous()
            E.data_ptrs = torch.tensor([E.data.data_ptr()], dtype=torch.int64, device=self.device)
            E.sf_ptrs = torch.tensor([E.sf.data_ptr()], dtype=torch.int64, device=self.device)
            E.bounds = torch.tensor([0, table.shape[0]], dtype=torch.int32, device=self.device)
        else:
            E.table = table
        del table
        E.wkv = Lin(get(prefix + "wkv.weight"), self.device, self.fp8)
        E.qw = get(prefix + "q_weight").float().contiguous()
        E.kw = get(prefix + "k_weight").float().contiguous()
        return E

    def engram(self, i: int, X: torch.Tensor, sumsq, fb: ForwardBatch, cache):
        """Hashed n-gram memory on this rank's residual streams X [T_l, hc, D]: hash each token's preceding n-grams
        (prefill: from the batch; decode: the cached token ids of the key slots), gather the table rows, project
        (wkv) and gate every stream.  Returns (X, sumsq) updated."""
        cfg, E, pc = self.cfg, self.layers[i].engram, self.pctx
        lo, hi = pc.local
        nmax = max(cfg.engram_orders)
        dev = X.device
        back = torch.arange(nmax, device=dev)
        p = fb.pos[lo:hi].long()
        if fb.is_prefill:
            src = (torch.arange(lo, hi, device=dev)[:, None] - back[None, :]).clamp(min=0)
            toks = fb.ids[src].long()
        else:
            j = p[:, None] - back[None, :]
            slot = fb.key_slots[lo:hi].gather(1, j.clamp(min=0)).long()
            toks = cache.tok[slot.clamp(min=0)].long()
        window = torch.where(p[:, None] - back[None, :] >= 0, toks, -1)
        rows = R.engram_hash_ids(window, cfg.engram_orders, cfg.engram_heads, cfg.engram_primes, cfg.vocab_size)
        T = X.shape[0]
        img = cfg.image_token_id
        if not self.on_gpu:
            kv = E.wkv(E.table[rows].reshape(T, rows.shape[1] * E.table.shape[1]))
            Xn = R.engram_gate(X, kv, E.qw, E.kw, cfg.rms_eps, cfg.engram_clamp).to(X.dtype)
            if img >= 0:
                Xn = torch.where((self._tok_local.long() == img)[:, None, None], X, Xn)
            return Xn, (None if sumsq is None else Xn.float().pow(2).sum((1, 2)))
        from ..ops._ext import ext

        emb = torch.empty(T, cfg.engram_cols * cfg.engram_dim, dtype=torch.bfloat16, device=dev)
        ext().engram_gather(rows.to(torch.int32).contiguous(), E.data_ptrs, E.sf_ptrs, E.bounds, cfg.engram_dim, emb)
        kv = E.wkv(emb).contiguous()
        X = X.contiguous()
        ss = torch.empty(T, dtype=torch.float32, device=dev)
        ext().engram_gate(X, kv, E.qw, E.kw, cfg.rms_eps, cfg.engram_clamp, ss,
                          self._tok_local.to(torch.int32).contiguous() if img >= 0 else None, img)
        return X, ss

    def _load_layer(self, i: int, get) -> Layer:
        cfg, dev, pc = self.cfg, self.device, self.pctx
        L = Layer()
        p = f"layers.{i}."
        if cfg.plain_residual:
            L.attn_hc = L.ffn_hc = None
        else:
            L.attn_hc = make_hc(get(p + "attn_hc.fn"), get(p + "attn_hc.base"), get(p + "attn_hc.scale"), dev)
            L.ffn_hc = make_hc(get(p + "ffn_hc.fn"), get(p + "ffn_hc.base"), get(p + "ffn_hc.scale"), dev)
        L.attn_norm = get(p + "attn_norm.weight")
        L.ffn_norm = get(p + "ffn_norm.weight")
        H, Hl, dn, dr, dv, r = cfg.n_heads, self.H_local, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, \
            cfg.v_head_dim, cfg.kv_lora_rank
        dq, dvh = cfg.qk_head_dim, cfg.head_out_dim
        h0, h1 = pc.tp_rank * Hl, (pc.tp_rank + 1) * Hl
        a = p + "attn."
        if cfg.q_lora_rank > 0:
            L.wq_a = Lin(get(a + "wq_a.weight"), dev, self.fp8)
            L.q_norm = get(a + "q_norm.weight")
            L.wq_b = Lin(get(a + "wq_b.weight", slice(h0 * dq, h1 * dq)), dev, self.fp8)
        else:
            L.wq = Lin(get(a + "wq.weight", slice(h0 * dq, h1 * dq)), dev, self.fp8)
        L.wkv_a = Lin(get(a + "wkv_a.weight"), dev, self.fp8)
        L.wqkv_a = None
        if self.on_gpu and cfg.q_lora_rank > 0 and L.wq_a.kind == "fp8" and L.wkv_a.kind == "fp8":
            # both down-projections read the same normalised input: one GEMM over the stacked weights (the output
            # columns [0, q_lora) feed the query path, the rest is the KV latent)
            L.wqkv_a = Lin(torch.cat([get(a + "wq_a.weight"), get(a + "wkv_a.weight")]), dev, self.fp8)
            L.wq_a = L.wkv_a = None
        L.kv_norm = get(a + "kv_norm.weight")
        L.wkv_b = None
        if cfg.attn_kind == "mla":
            wkv_b = get(a + "wkv_b.weight", slice(h0 * (dn + dv), h1 * (dn + dv)))  # [Hl*(dn+dv), r]
            L.wkv_b = Lin(wkv_b, dev, self.fp8)
            # absorbed decode uses the same (fp8-rounded) wkv_b as the prefill GEMM
            wkv_b3 = (L.wkv_b.fw.dequant() if L.wkv_b.kind == "fp8" else wkv_b).view(Hl, dn + dv, r)
            L.w_uk = wkv_b3[:, :dn, :].transpose(1, 2).contiguous().to(self.act_dtype)  # [Hl, r, dn]
            L.w_uv = wkv_b3[:, dn:, :].contiguous().to(self.act_dtype)                  # [Hl, dv, r]
            L.w_uv_all = None
            if self.o_a2a:
                # every head's value up-projection: the absorbed decode output stays token-major on its owner
                wall = get(a + "wkv_b.weight")
                if self.on_gpu and self.fp8:
                    wall = Lin(wall, dev, self.fp8).fw.dequant()
                L.w_uv_all = wall.view(H, dn + dv, r)[:, dn:, :].contiguous().to(self.act_dtype)  # [H, dv, r]
                del wall
        L.wo_a = None
        if cfg.o_groups:
            # grouped low-rank output projection: this rank's heads are whole groups
            G, R = cfg.o_groups, cfg.o_lora_rank
            if G % pc.tp:
                raise ValueError(f"o_groups={G} must be a multiple of the attention TP degree {pc.tp}")
            Gl = G if self.o_a2a else G // pc.tp          # the owner of a token projects all of its groups
            g0 = 0 if self.o_a2a else pc.tp_rank * Gl
            L.wo_a = get(a + "wo_a.weight", slice(g0, g0 + Gl)).to(self.act_dtype).contiguous()  # [Gl, R, (H/G)*dvh]
            wo_b = get(a + "wo_b.weight")                                                      # [D, G*R]
            L.wo = Lin(wo_b[:, g0 * R:(g0 + Gl) * R].contiguous(), dev, self.fp8)
        else:
            wo = get(a + "wo.weight")                                              # [D, H*dvh]
            L.wo = Lin(wo if self.o_a2a else wo[:, h0 * dvh:h1 * dvh].contiguous(), dev, self.fp8)
        L.sink = get(a + "sink")[h0:h1].float().contiguous() if cfg.attn_sink else None
        L.sink_all = get(a + "sink").float().contiguous().to(dev) if cfg.attn_sink else None     # every head
        L.engram = None
        if i in cfg.engram_layers:
            L.engram = self._load_engram(p + "engram.", get)
        L.has_indexer = cfg.has_indexer(i)
        if L.has_indexer:
            ix = a + "indexer."
            L.idx_wq = Lin(get(ix + "wq.weight"), dev, fp8=False)
            L.idx_kn_w, L.idx_kn_b = get(ix + "k_norm.weight"), get(ix + "k_norm.bias")
            if dev.type == "cpu":
                L.idx_wk = Lin(get(ix + "wk.weight"), dev, fp8=False)
                L.idx_wp = Lin(get(ix + "weights_proj.weight"), dev, fp8=False)
            else:
                # the key and head-weight projections read the same input: one GEMM, fp32 out, split by columns
                L.idx_wkp = Lin(torch.cat([get(ix + "wk.weight"), get(ix + "weights_proj.weight")]), dev, fp8=False)
        f = p + "ffn."
        L.moe = cfg.is_moe_layer(i)
        if not L.moe:
            L.dense = SwigluFFN(get(f + "w1"), get(f + "w3"), get(f + "w2"), dev, cfg.swiglu_limit)
        else:
            E, El = cfg.n_routed_experts, self.E_local
            e0 = pc.ep_rank * El
            L.gate = Lin(get(f + "gate.weight"), dev, fp8=False)
            L.gate_b = get(f + "gate.bias")
            L.gate_b_img = get(f + "gate.bias_img").float().contiguous() if cfg.image_token_id >= 0 else None
            if dev.type == "cpu":
                L.e_w1 = get(f + "experts.w1", slice(e0, e0 + El))
                L.e_w3 = get(f + "experts.w3", slice(e0, e0 + El))
                L.e_w2 = get(f + "experts.w2", slice(e0, e0 + El))
            else:
                w13s, w2s = [], []
                for e in range(e0, e0 + El):
                    w1 = get(f + "experts.w1", slice(e, e + 1))[0]
                    w3 = get(f + "experts.w3", slice(e, e + 1))[0]
                    w13s.append(quantize_weight(interleave_gate_up(w1, w3)))
                    w2s.append(quantize_weight(get(f + "experts.w2", slice(e, e + 1))[0]))
                    del w1, w3
                L.e_w13 = stack_weights(w13s)
                L.e_w2 = stack_weights(w2s)
                del w13s, w2s
            L.shared = None
            if cfg.n_shared_experts > 0:
                L.shared = SwigluFFN(get(f + "shared.w1"), get(f + "shared.w3"), get(f + "shared.w2"), dev,
                                     cfg.swiglu_limit)
        return L

    # ------------------------------------------------------------------------------------------------------------------
    # mHC
    # ------------------------------------------------------------------------------------------------------------------
    def hc_coeffs(self, X: torch.Tensor, sumsq: Optional[torch.Tensor], hp: HCParams):
        cfg = self.cfg
        T = X.shape[0]
        if not self.on_gpu:
            return R.mhc_coeffs(X, hp.fn, hp.base, hp.scale, cfg.hc_mult, cfg.sinkhorn_iters, cfg.hc_eps, cfg.rms_eps)
        from ..ops._ext import ext

        mix = mhc_mix(X.view(T, X.shape[1] * X.shape[2]), hp.fn)
        pre = torch.empty(T, 4, device=X.device)
        post = torch.empty(T, 4, device=X.device)
        comb = torch.empty(T, 4, 4, device=X.device)
        ext().mhc_coeffs(mix, sumsq, hp.base, hp.scale, X.shape[1] * X.shape[2], cfg.sinkhorn_iters, cfg.hc_eps,
                         cfg.rms_eps, pre, post, comb)
        return pre, post, comb

    def _boundary_fusable(self, X) -> bool:
        """Decode-sized batches on the GPU (at most 64 rows on this rank) with 4 residual streams run each boundary
        as one fused kernel (not while tracing: the trace records the intermediate streams)."""
        D = self.cfg.hidden_size
        return (self.on_gpu and self.trace is None and not self.cfg.plain_residual and X.shape[0] <= 64 and
                X.shape[1] == 4 and D % 1024 == 0 and D <= 8192 and self.cfg.sinkhorn_iters >= 1 and
                getattr(self.layers[0].attn_hc, "fn", None) is not None and self.layers[0].attn_hc.fn.shape[0] == 48)

    def hc_boundary(self, X, pend, hp: HCParams, w):
        """One fused decode boundary: mix the pending sublayer output ``pend = (out, post, comb)`` into X (in place;
        None at the first boundary of a step), then the next sublayer's coefficients and its RMSNorm'd input.
        Returns (h bf16, (fp8 q, sf), post, comb)."""
        from ..ops._ext import ext
        from ..ops.quant import empty_sf

        cfg = self.cfg
        T, _, D = X.shape
        dev = X.device
        y = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        q = torch.empty(T, D, dtype=torch.float8_e4m3fn, device=dev)
        sf = empty_sf(T, D, dev)
        pre = torch.empty(T, 4, device=dev)
        post = torch.empty(T, 4, device=dev)
        comb = torch.empty(T, 4, 4, device=dev)
        out, p_in, c_in = pend if pend is not None else (None, None, None)
        ext().mhc_boundary_small(X, out.contiguous() if out is not None else None, p_in, c_in, hp.fn, hp.base,
                                 hp.scale, cfg.sinkhorn_iters, cfg.hc_eps, cfg.rms_eps, w, y, q, sf, pre, post, comb)
        return y, (q, sf), post, comb

    def _flush(self, X, sumsq, pend):
        """Apply a pending fused-boundary post-mix (X, its Σx² and no pending output afterwards)."""
        if pend is None:
            return X, sumsq, None
        with region("mhc.post_mix"):
            X, sumsq = self.post_mix(X, *pend)
        return X, sumsq, None

    def pre_norm(self, X, pre, w, want_fp8: bool):
        """RMSNorm(Σ pre_i X_i)·w -> (bf16 h, (fp8 q, sf) or None)."""
        if not self.on_gpu:
            return R.rms_norm(R.mhc_pre_mix(X, pre), w, self.cfg.rms_eps), None
        from ..ops._ext import ext
        from ..ops.quant import empty_sf

        T, _, D = X.shape
        y = torch.empty(T, D, dtype=torch.bfloat16, device=X.device)
        q = sf = None
        if want_fp8:
            q = torch.empty(T, D, dtype=torch.float8_e4m3fn, device=X.device)
            sf = empty_sf(T, D, X.device)
        ext().mhc_pre_norm(X, pre, w, self.cfg.rms_eps, y, q, sf, None)
        return y, ((q, sf) if want_fp8 else None)

    def plain_norm(self, X, w, want_fp8: bool):
        """Plain pre-norm residual: RMSNorm(x)·w of the single stream -> (h, (fp8 q, sf) or None)."""
        x = X[:, 0]
        if not self.on_gpu:
            return R.rms_norm(x, w, self.cfg.rms_eps), None
        if want_fp8:
            return C.rms_norm(x, w, self.cfg.rms_eps, want_bf16=True, want_fp8=True)
        return C.rms_norm(x, w, self.cfg.rms_eps), None

    def plain_add(self, X, out):
        """x + f(x): the sublayer output joins the single residual stream."""
        return X + out.to(X.dtype).reshape(X.shape[0], 1, X.shape[2])

    def post_mix(self, X, out, post, comb):
        if not self.on_gpu:
            return R.mhc_post_mix(X, out, post, comb), None
        from ..ops._ext import ext

        sumsq = torch.empty(X.shape[0], device=X.device)
        ext().mhc_post_mix(X, out.contiguous(), post, comb.view(-1, 16), X, sumsq)   # in place
        return X, sumsq

    # ------------------------------------------------------------------------------------------------------------------
    # attention
    # ------------------------------------------------------------------------------------------------------------------
    def attention(self, i: int, h: torch.Tensor, hq, fb: ForwardBatch, cache) -> torch.Tensor:
        """h: this rank's tokens [T_l, D]. Returns this rank's rows of the attention output [T_l, D]."""
        cfg, L, pc = self.cfg, self.layers[i], self.pctx
        Hl = self.H_local
        dn, dr, dv, r = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
        lo, hi = pc.local
        pos_l = fb.pos[lo:hi]
        dp = pc.attn_dp and pc.world > 1         # attention over this rank's own sequences, all heads
        qkv = None
        q_lat_q = None                           # fp8 rows of q_lat_l when the q-norm emitted them
        if L.wqkv_a is not None:
            with region("attn.q_proj"):
                qkv = L.wqkv_a(h, xq=hq)                                        # [T_l, q_lora + latent_dim]
        with region("attn.q_proj"):
            if cfg.q_lora_rank > 0:
                q_lat_raw = qkv[:, :cfg.q_lora_rank] if qkv is not None else L.wq_a(h, xq=hq)
                if self.on_gpu:
                    # the q-norm also emits the fp8 rows (1x128 UE8M0) that wq_b and the indexer's wq read
                    q_lat_l, q_lat_q = C.rms_norm(q_lat_raw, L.q_norm, cfg.rms_eps, want_bf16=True, want_fp8=True)
                else:
                    q_lat_l = R.rms_norm(q_lat_raw, L.q_norm, cfg.rms_eps)
            else:
                q_lat_l = h
        with region("attn.kv_proj"):
            kv = qkv[:, cfg.q_lora_rank:] if qkv is not None else L.wkv_a(h, xq=hq)   # [T_l, latent_dim]
            if cfg.attn_kind == "latent_mqa":
                # the shared KV head: the normalised latent with RoPE on its last dr dims
                kv_c = C.rms_norm(kv.contiguous(), L.kv_norm, cfg.rms_eps) if self.on_gpu else \
                    R.rms_norm(kv, L.kv_norm, cfg.rms_eps)
                latent_l = kv_c.to(self.act_dtype).contiguous()
                C.rope_(latent_l.view(-1, 1, r), r - dr, dr, self.cos_sin, pos_l)
            elif self.on_gpu:
                # the projection output becomes the latent row in place: RMSNorm of the first r columns, RoPE of the
                # last dr (no copies, no concatenation)
                latent_l = kv
                C.rms_norm_(latent_l[:, :r], L.kv_norm, cfg.rms_eps)
                C.rope_(latent_l.view(-1, 1, r + dr), r, dr, self.cos_sin, pos_l)
            else:
                kv_c = R.rms_norm(kv[:, :r], L.kv_norm, cfg.rms_eps)
                k_pe = kv[:, r:].contiguous().view(-1, 1, dr)
                C.rope_(k_pe, 0, dr, self.cos_sin, pos_l)
                latent_l = torch.cat([kv_c.to(self.act_dtype), k_pe.view(-1, dr).to(self.act_dtype)], dim=-1)
        idx_l = None
        if L.has_indexer:
            with region("attn.indexer_qk"):
                idx_l = self.indexer_qkw(i, h, q_lat_l, pos_l, q_lat_q)
        q_lat_a = q_lat_l.to(self.act_dtype) if self.on_gpu else q_lat_l
        out_loc = fb.out_loc
        if dp and self.owner_kv:
            # each request's rows always run on its home rank: this rank caches only its own rows
            q_lat, latent, latent_c = q_lat_a, latent_l, latent_l
            idx_k = idx_l[1] if idx_l is not None else None
            out_loc = fb.out_loc[lo:hi]
        elif self.owner_kv:
            # TP attention, owner-only KV: the cache-reading core runs token-parallel on each token's home rank, so
            # only the home rank writes the token's rows; the other ranks need the new latent rows only for the MLA
            # prefill core (k / v of every token from wkv_b)
            with region("tp.gather"):
                q_lat = pc.gather_rows(q_lat_a)
                dense_prefill = fb.is_prefill and cfg.attn_kind == "mla" and not self._sparse_prefill(i, fb)
                latent = pc.gather_rows(latent_l) if dense_prefill else None
            latent_c = latent_l
            idx_k = idx_l[1] if idx_l is not None else None
            out_loc = fb.out_loc[lo:hi]
        elif dp:
            q_lat, latent = q_lat_a, latent_l
            # every rank's cache receives every token's rows (one all-gather of the new rows): a later step may
            # give a request to another rank (prefill shards by tokens, decode by rows)
            with region("dp.kv_gather"):
                latent_c = pc.gather_rows(latent_l)
                idx_k = pc.gather_rows(idx_l[1]) if idx_l is not None else None
        else:
            with region("tp.gather"):
                q_lat = pc.gather_rows(q_lat_a)
                latent = pc.gather_rows(latent_l)
                idx_k = pc.gather_rows(idx_l[1]) if idx_l is not None else None
            latent_c = latent
        with region("attn.kv_proj"):
            cache.write_latent(i, out_loc, latent_c)
            if idx_k is not None:
                cache.write_index_k(i, out_loc, idx_k)
        if idx_l is not None and self._selection_early(i, fb, dp):
            self._early_sel[i] = self._start_selection(i, fb, cache, idx_l)
        T = q_lat.shape[0]
        dq = cfg.qk_head_dim
        with region("attn.q_proj"):
            if cfg.q_lora_rank > 0:
                # the norm's fp8 rows serve when q_lat is this rank's own (not gathered) rows
                q = L.wq_b(q_lat, xq=q_lat_q if q_lat is q_lat_a and q_lat_a is q_lat_l else None).view(T, Hl, dq)
            else:
                q = L.wq(q_lat).view(T, Hl, dq)
            if not self.on_gpu:
                q = q.clone()
            C.rope_(q, dq - dr, dr, self.cos_sin, pos_l if dp else fb.pos)
        tok_major = False        # o holds this rank's tokens with every head (else: every token, this rank's heads)
        if cfg.attn_kind == "latent_mqa":
            o, tok_major = self._attn_latent(i, q, fb, cache, idx_l, dp)
        elif fb.is_prefill and self._sparse_prefill(i, fb):
            o, tok_major = self._attn_prefill_sparse(i, q, fb, cache, idx_l, dp)
        elif fb.is_prefill:
            o = self._attn_prefill(i, q, latent, fb, idx_l, cache, dp)
        else:
            o, tok_major = self._attn_decode(i, q, fb, cache, idx_l, dp)
        with region("attn.o_proj"):
            if self.o_a2a:
                if not tok_major:
                    o = pc.heads_to_tokens(o.to(self.act_dtype).contiguous())          # [T_l, H, dvh]
                return L.wo(self._out_heads(L, o, o.shape[0]))
            o2 = self._out_heads(L, o, T)
            return L.wo(o2) if dp else pc.row_parallel_out(L.wo, o2)

    def _out_heads(self, L, o: torch.Tensor, T: int) -> torch.Tensor:
        """Per-head outputs [T, Hl, dvh] -> the output projection's input: the head concatenation, or (grouped
        low-rank projection) wo_a of each local group of heads, [T, Gl * o_lora]."""
        if L.wo_a is None:
            return o.reshape(T, o.shape[1] * o.shape[2]).to(self.act_dtype).contiguous()
        Gl = L.wo_a.shape[0]
        z = head_bmm(o.reshape(T, Gl, L.wo_a.shape[2]).to(self.act_dtype), L.wo_a)                # [T, Gl, o_lora]
        return z.reshape(T, z.shape[1] * z.shape[2]).to(self.act_dtype).contiguous()

    def indexer_qkw(self, i, h, q_lat, pos, q_lat_q=None):
        cfg, L = self.cfg, self.layers[i]
        T, Hi, Di, dr = h.shape[0], cfg.index_n_heads, cfg.index_head_dim, cfg.qk_rope_head_dim
        if self.on_gpu:
            from ..ops._ext import ext

            # decode-size batches: the query projection (from q_lat) runs on the side stream while the key /
            # head-weight projection (from h) runs here, joined before returning (prefill GEMMs fill the GPU alone)
            cur = torch.cuda.current_stream()
            side = self._index_stream() if T <= 1024 else cur
            if side is not cur:
                side.wait_stream(cur)
                for t_ in (q_lat, pos) + (tuple(q_lat_q) if q_lat_q is not None else ()):
                    t_.record_stream(side)
            with torch.cuda.stream(side):
                q = L.idx_wq(q_lat, xq=q_lat_q).view(T, Hi, Di)
                C.rope_(q, 0, dr, self.cos_sin, pos)
            if side is not cur:
                q.record_stream(cur)
            kw = L.idx_wkp(h, out_dtype=torch.float32)                               # [T, Di + Hi]
            k = torch.empty(T, Di, dtype=torch.bfloat16, device=h.device)
            w = torch.empty(T, Hi, dtype=torch.float32, device=h.device)
            # LayerNorm + RoPE of the key and the scaled head weights in one launch
            ext().indexer_kw_post(kw, Di, L.idx_kn_w.float().contiguous(), L.idx_kn_b.float().contiguous(), 1e-6,
                                  self.cos_sin, pos.to(torch.int32).contiguous(), dr, (Hi ** -0.5) * (Di ** -0.5),
                                  k, w)
            k = k.view(T, 1, Di)
            if side is not cur:
                cur.wait_stream(side)
        else:
            q = L.idx_wq(q_lat, xq=q_lat_q).view(T, Hi, Di).clone()
            C.rope_(q, 0, dr, self.cos_sin, pos)
            k = F.layer_norm(L.idx_wk(h).float(), (Di,), L.idx_kn_w, L.idx_kn_b, 1e-6).to(self.act_dtype)
            w = (L.idx_wp(h, out_dtype=torch.float32) * (Hi ** -0.5) * (Di ** -0.5)).float()
            k = k.view(T, 1, Di)
            C.rope_(k, 0, dr, self.cos_sin, pos)
        if cfg.index_fp4:               # fp4 values are exact in bf16: the bf16 logits kernels compute fp4 products
            q = R.fake_quant_mxfp4(q)
            k = R.fake_quant_mxfp4(k)
        elif cfg.index_fp8:             # likewise e4m3 values (prefill re-quantises them exactly for fp8 MMAs)
            q = R.fake_quant_fp8_rows(q)
            k = R.fake_quant_fp8_rows(k)
        return q, k.view(T, Di), w

    def _prefill_key_masks(self, idx_l, fb: ForwardBatch, gather: bool = True):
        """DSA selection of this rank's sequences, gathered to all ranks (rows in global token order) unless the
        attention is data-parallel (then only this rank's rows are needed)."""
        pc = self.pctx
        lo, hi = pc.local
        cu_l = [c - lo for c in fb.cu_seqlens if lo <= c <= hi]
        lmax = max(b - a for a, b in zip(fb.cu_seqlens[:-1], fb.cu_seqlens[1:]))
        if lmax <= self.cfg.index_topk:
            return None
        q, k, w = idx_l
        m = A.indexer_prefill_mask(q, k, w, cu_l if len(cu_l) > 1 else [0, 0], self.cfg.index_topk, lmax=lmax,
                                   fp8=self.cfg.index_fp8 and k.shape[-1] % 128 == 0)
        return pc.gather_rows(m) if gather else m

    def _attn_prefill(self, i, q, latent, fb, idx_l, cache, dp: bool = False):
        cfg, L, pc = self.cfg, self.layers[i], self.pctx
        T, Hl = q.shape[0], self.H_local
        dn, dr, dv, r = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
        cu = fb.cu_seqlens
        if dp:
            lo, hi = pc.local
            cu = [c - lo for c in fb.cu_seqlens if lo <= c <= hi]
            if len(cu) < 2:
                cu = [0, 0]
        with region("attn.kv_up"):
            kvb = L.wkv_b(latent[:, :r].contiguous()).view(T, Hl, dn + dv)
        src = cfg.index_source(i)
        masks = None
        if src == i:
            with region("attn.indexer_topk"):
                masks = self._prefill_key_masks(idx_l, fb, gather=not dp)
            self._dsa[i] = masks
        elif src is not None:
            masks = self._dsa.get(src)              # selection shared with the index-source layer
        with region("attn.core_prefill"):
            return A.mla_prefill(q, kvb, latent[:, r:].contiguous(), cu, cfg.softmax_scale, masks, sink=L.sink)

    def _latent_keys(self, i, fb, cache, idx_l, rows, local: bool) -> torch.Tensor:
        """Cache slots each query in ``rows`` (a slice of the batch) attends to, [Tq, K] int32 (-1 pad): the last
        swa_window positions, plus the DSA top-k over the older keys (or every causal key without an indexer)."""
        cfg, pc = self.cfg, self.pctx
        W, lo, hi = cfg.swa_window, pc.local[0], pc.local[1]
        dev = fb.pos.device
        if fb.is_prefill:
            # keys of a prefill query: its own sequence's slots, positions 0..p (prompts start at position 0)
            cu = fb.cu_seqlens
            lens = [b - a for a, b in zip(cu[:-1], cu[1:])]
            start = torch.repeat_interleave(torch.tensor(cu[:-1], dtype=torch.long),
                                            torch.tensor(lens, dtype=torch.long)).to(dev)[rows]
            # keys: the sequence's batch tokens up to the query (a bounded-replay tail starts after position 0)
            nk = fb.pos[rows].long() - fb.pos[start].long() + 1
            Lmax = max(lens) if lens else 1
            j = torch.arange(Lmax, device=dev)
            src_i = (start[:, None] + j[None, :]).clamp(max=fb.out_loc.shape[0] - 1)
            ks = torch.where(j[None, :] < nk[:, None], fb.out_loc[src_i].long(), -1).to(torch.int32)
        else:
            ks, nk = fb.key_slots[rows], fb.n_keys[rows].long()
        parts = []
        src = cfg.index_source(i)
        if src is not None:
            if src == i:
                with region("attn.indexer_topk"):
                    qi, _, wi = idx_l
                    if fb.is_prefill:
                        ks_l = ks if local else self._latent_key_table(fb, lo, hi)
                        nk_l = (fb.pos[lo:hi].long() + 1) if not local else nk
                    else:
                        ks_l, nk_l = fb.key_slots[lo:hi], fb.n_keys[lo:hi].long()
                    cand = (nk_l - W).clamp(min=0).to(torch.int32).contiguous()      # keys older than the window
                    sel = A.indexer_topk(qi, wi, cache.index_k[i], ks_l.contiguous(), cand, cfg.index_topk)
                    sel = sel if local else pc.gather_rows(sel)
                if self.trace is not None and fb.is_prefill:
                    # selected key positions (debugging: lets an oracle follow this selection exactly)
                    inv = torch.full((int(fb.out_loc.max()) + 1,), -1, dtype=torch.long, device=dev)
                    inv[fb.out_loc.long()] = fb.pos.long()
                    self._tr(f"{i}.dsa_pos", torch.where(sel >= 0, inv[sel.long().clamp(min=0)], -1))
                self._dsa[i] = sel
            else:
                sel = self._dsa[src]                # selection shared with the index-source layer
            parts.append(sel)
        if W > 0:
            wj = nk[:, None] - W + torch.arange(W, device=dev)[None, :]
            lowest = 0
            if not fb.is_prefill and fb.late_from is not None and cfg.is_late_layer(i):
                lowest = fb.late_from[rows].long()[:, None]      # keys before the replayed tail do not exist here
            win = torch.where(wj >= lowest, ks.gather(1, wj.clamp(min=0)).long(), -1).to(torch.int32)
            parts.append(win)
        elif src is None:
            parts.append(ks)                        # dense causal
        return torch.cat([p.to(torch.int32) for p in parts], dim=1).contiguous()

    def _latent_key_table(self, fb, lo, hi) -> torch.Tensor:
        """Prefill key slots [hi-lo, Lmax] of this rank's queries (the indexer's candidate table)."""
        cu = fb.cu_seqlens
        lens = [b - a for a, b in zip(cu[:-1], cu[1:])]
        dev = fb.pos.device
        start = torch.repeat_interleave(torch.tensor(cu[:-1], dtype=torch.long),
                                        torch.tensor(lens, dtype=torch.long)).to(dev)[lo:hi]
        nk = fb.pos[lo:hi].long() - fb.pos[start].long() + 1
        j = torch.arange(max(lens) if lens else 1, device=dev)
        src_i = (start[:, None] + j[None, :]).clamp(max=fb.out_loc.shape[0] - 1)
        return torch.where(j[None, :] < nk[:, None], fb.out_loc[src_i].long(), -1).to(torch.int32)

    def _attn_latent(self, i, q, fb, cache, idx_l, dp: bool = False):
        """Latent MQA (DeepSeek-V4 layout), prefill and decode alike: every head attends over explicit per-query key
        lists of cached latent rows (sparse kernel), then the output's RoPE dims are rotated back by the query
        position.  Tensor-parallel heads run token-parallel through a head/token all-to-all, so every rank reads
        only its own queries' key rows."""
        cfg, L, pc = self.cfg, self.layers[i], self.pctx
        r, dr = cfg.kv_lora_rank, cfg.qk_rope_head_dim
        lo, hi = pc.local
        swap = not dp and pc.world > 1 and hasattr(pc, "heads_to_tokens")
        local = dp or swap
        rows = slice(lo, hi) if local else slice(0, q.shape[0])
        idx = self._latent_keys(i, fb, cache, idx_l, rows, local)
        pos_q = fb.pos[lo:hi] if dp else fb.pos
        tok_major = swap and self.o_a2a      # the owner keeps its tokens' outputs (all heads) for the projection
        with region("attn.core_prefill" if fb.is_prefill else "attn.core_decode"):
            if swap:
                q_tok = pc.heads_to_tokens(q.contiguous())                          # [n_r, H, r]
                o = A.sparse_mla(q_tok, cache.latent[i], idx, cfg.softmax_scale, r, sink=L.sink_all)
                if not tok_major:
                    o = pc.tokens_to_heads(o.contiguous()) if self.on_gpu else pc.tokens_to_heads(o)
            else:
                o = A.sparse_mla(q.contiguous(), cache.latent[i], idx, cfg.softmax_scale, r, sink=L.sink)
            o = o.to(self.act_dtype).contiguous() if self.on_gpu else o.float().contiguous()
            C.rope_(o, r - dr, dr, self.cos_sin, fb.pos[lo:hi] if tok_major else pos_q, inverse=True)
        return o, tok_major

    def _sparse_prefill(self, i, fb) -> bool:
        """MLA prefill of this layer as absorbed sparse attention: the batch holds a sequence longer than
        cfg.sparse_prefill_min and the layer has a DSA selection."""
        cfg = self.cfg
        if cfg.sparse_prefill_min <= 0 or cfg.attn_kind != "mla" or cfg.index_source(i) is None:
            return False
        cu = fb.cu_seqlens
        return max(b - a for a, b in zip(cu[:-1], cu[1:])) > cfg.sparse_prefill_min

    def _attn_prefill_sparse(self, i, q, fb, cache, idx_l, dp: bool = False):
        """Long-prompt MLA prefill: every query attends to the cached latent rows of its DSA top-k keys through the
        absorbed sparse kernel (the decode core), token-parallel; the new rows were written to the cache above."""
        cfg, pc = self.cfg, self.pctx
        lo, hi = pc.local
        src = cfg.index_source(i)
        if src == i:
            with region("attn.indexer_topk"):
                qi, ki, wi = idx_l
                cu_l = [c - lo for c in fb.cu_seqlens if lo <= c <= hi]
                sel = A.indexer_prefill_slots(qi, ki, wi, cu_l if len(cu_l) > 1 else [0, 0], cfg.index_topk,
                                              fb.out_loc[lo:hi], fp8=cfg.index_fp8 and ki.shape[-1] % 128 == 0)
            self._dsa[i] = sel
        else:
            sel = self._dsa[src]                    # selection shared with the index-source layer
        return self._attn_decode(i, q, fb, cache, idx_l, dp, sel=sel)

    def _attn_decode(self, i, q, fb, cache, idx_l, dp: bool = False, sel=None):
        """Absorbed attention over cached latent rows (decode, verify, chunked prefill; and long prompts with
        ``sel``: the DSA selection of this rank's queries as cache slots)."""
        cfg, L, pc = self.cfg, self.layers[i], self.pctx
        T, Hl = q.shape[0], self.H_local
        dn, r = cfg.qk_nope_head_dim, cfg.kv_lora_rank
        lo, hi = pc.local
        # Tensor-parallel heads, but the core runs token-parallel: every rank would otherwise stream the selected
        # latent rows of ALL tokens for its few heads.  Two small all-to-alls (q in, o_lat out) let each rank read
        # only its own tokens' rows, for every head.
        swap = not dp and pc.world > 1 and hasattr(pc, "heads_to_tokens")
        local = dp or swap
        src = cfg.index_source(i)
        if sel is not None:
            idx = sel if local or pc.world == 1 else pc.gather_rows(sel)
        else:
            idx = fb.key_slots[lo:hi] if local else fb.key_slots
        pending = None
        early = self._early_sel.pop(i, None)
        if sel is None and src is not None and int(fb.key_slots.shape[1]) > cfg.index_topk:
            if src == i:
                qi, _, wi = idx_l
                ks, nk = fb.key_slots[lo:hi].contiguous(), fb.n_keys[lo:hi].contiguous()
                if early is not None:
                    pending = early                 # started on the side stream right after the key-cache write
                elif self.on_gpu and (local or pc.world == 1):
                    pending = self._start_selection(i, fb, cache, idx_l)
                else:
                    with region("attn.indexer_topk"):
                        sel = A.indexer_topk(qi, wi, cache.index_k[i], ks, nk, cfg.index_topk)
                        idx = sel if local else pc.gather_rows(sel)
                    self._dsa[i] = idx
            else:
                idx = self._dsa[src]                # selection shared with the index-source layer
        with region("attn.absorb_q"):
            # [q_nope · W_uk | q_rope] -> [T, Hl, r + dr], in fp16 when the kernel reads fp8 cache rows
            qf = head_bmm(q, L.w_uk, tail=q.shape[-1] - dn,
                          out_dtype=torch.float16 if (self.on_gpu and cfg.kv_fp8) else self.act_dtype).contiguous()
        if pending is not None:
            idx = pending.get()
            self._dsa[i] = idx
        if swap:
            with region("attn.core_decode"):
                q_tok = pc.heads_to_tokens(qf)                                      # [n_r, H, r + dr]
                o_tok = A.sparse_mla(q_tok, cache.latent[i], idx.contiguous(), cfg.softmax_scale, r,
                                     sink=L.sink_all)
            if self.o_a2a:
                # the owner keeps its tokens' outputs: every head's value projection here, no way back
                with region("attn.absorb_o"):
                    return head_bmm(o_tok, L.w_uv_all), True                         # [n_r, H, dv]
            with region("attn.core_decode"):
                o_lat = pc.tokens_to_heads(o_tok)                                   # [T, Hl, r]
        else:
            with region("attn.core_decode"):
                o_lat = A.sparse_mla(qf, cache.latent[i], idx.contiguous(), cfg.softmax_scale, r, sink=L.sink)
        with region("attn.absorb_o"):
            return head_bmm(o_lat, L.w_uv), False                                    # [T, Hl, dv]

    def _selection_early(self, i: int, fb, dp: bool) -> bool:
        """Whether this decode layer's DSA selection can start on the side stream as soon as the new index keys are
        in the cache (before the query projections): the GPU path of an index-source MLA layer whose core reads
        only this rank's queries (token-parallel TP, data-parallel attention, or one rank)."""
        cfg, pc = self.cfg, self.pctx
        if not self.on_gpu or fb.is_prefill or cfg.attn_kind != "mla" or cfg.index_source(i) != i:
            return False
        if int(fb.key_slots.shape[1]) <= cfg.index_topk:
            return False
        swap = not dp and pc.world > 1 and hasattr(pc, "heads_to_tokens")
        return dp or swap or pc.world == 1

    def _start_selection(self, i: int, fb, cache, idx_l) -> Pending:
        """DSA top-k of this rank's decode queries on the side stream (the reference's decode index streams): it
        overlaps the query projection and absorption on the main stream until ``Pending.get()``."""
        cfg = self.cfg
        lo, hi = self.pctx.local
        qi, _, wi = idx_l
        ks, nk = fb.key_slots[lo:hi].contiguous(), fb.n_keys[lo:hi].contiguous()
        side = self._index_stream()
        side.wait_stream(torch.cuda.current_stream())
        for t_ in (qi, wi, ks, nk):
            t_.record_stream(side)
        with torch.cuda.stream(side), region("attn.indexer_topk"):
            return Pending(A.indexer_topk(qi, wi, cache.index_k[i], ks, nk, cfg.index_topk), side)

    def _index_stream(self):
        if getattr(self, "_idx_side", None) is None:
            self._idx_side = torch.cuda.Stream()
        return self._idx_side

    # ------------------------------------------------------------------------------------------------------------------
    # FFN
    # ------------------------------------------------------------------------------------------------------------------
    def ffn(self, i: int, h: torch.Tensor, hq) -> torch.Tensor:
        cfg, L = self.cfg, self.layers[i]
        if not L.moe:
            with region("ffn.dense"):
                return L.dense(h, xq=hq)
        T = h.shape[0]
        with region("moe.router"):
            logits = L.gate(h, out_dtype=torch.float32)
            w, ids = C.router_topk(logits, L.gate_b, cfg.n_activated_experts, cfg.score_func, cfg.route_scale,
                                   cfg.norm_topk_prob, bias_img=L.gate_b_img,
                                   tok=self._tok_local if L.gate_b_img is not None else None,
                                   img_id=cfg.image_token_id, n_groups=cfg.n_groups, topk_groups=cfg.topk_groups)
        self._tr(f"{i}.router_ids", ids)
        if self.expert_load is not None:
            self.expert_load.record_device(i, ids)
        shared = None
        if L.shared is not None:
            if self.on_gpu:
                # shared expert on a side stream, overlapping the routed experts; the combine joins it
                if self._side is None:
                    self._side = torch.cuda.Stream()
                self._side.wait_stream(torch.cuda.current_stream())
                # h / hq belong to the main stream's allocator pool: keep them alive until the side stream is done
                h.record_stream(self._side)
                if hq is not None:
                    hq[0].record_stream(self._side)
                    hq[1].record_stream(self._side)
                with torch.cuda.stream(self._side), region("moe.shared"):
                    shared = Pending(L.shared(h, xq=hq), self._side)
            else:
                shared = L.shared(h, xq=hq)
        return self.pctx.moe(self, L, h, w, ids, shared, hq=hq)

    def moe_local(self, L, h, w, ids, shared, hq=None):
        """All experts local (EP = 1): sort rows by expert, grouped GEMMs, weighted combine."""
        cfg = self.cfg
        T, k = ids.shape
        if not self.on_gpu:
            out = torch.zeros_like(h)
            for e in range(self.E_local):
                rows, slot = torch.nonzero(ids == e, as_tuple=True)
                if rows.numel() == 0:
                    continue
                x = h[rows]
                y = R.swiglu(x @ L.e_w1[e].t(), x @ L.e_w3[e].t(), cfg.swiglu_limit) @ L.e_w2[e].t()
                out.index_add_(0, rows, y * w[rows, slot][:, None])
            return out + shared if shared is not None else out
        with region("moe.dispatch"):
            lay = C.MoeLayout(ids, self.E_local)
            # quantise every token once, then gather rows; quantised from the bf16 rows like the multi-GPU dispatch
            # kernels do, so that every parallel layout feeds the experts identical bytes
            tq, tsf = quant_act(h)
            a_q, a_sf = gather_rows_fp8(tq, tsf, lay.row_src, n_blocks=lay.num_blocks)
        I2 = 2 * cfg.moe_intermediate
        with region("moe.gemm_up"):
            act, act_sf = fp8_gemm_swiglu(a_q, a_sf, L.e_w13, cfg.swiglu_limit, lay.m_block_expert, lay.num_blocks,
                                          I2, pair=lay.pair, row_valid=lay.row_src)
        with region("moe.gemm_down"):
            y = fp8_gemm(act, act_sf, L.e_w2, m_block_expert=lay.m_block_expert, num_m_blocks=lay.num_blocks,
                         n_per_group=cfg.hidden_size, pair=lay.pair, row_valid=lay.row_src)
        with region("moe.combine"):
            return C.moe_combine(y, w, lay.slot_pos, resolve(shared), T)

    # ------------------------------------------------------------------------------------------------------------------
    # whole model
    # ------------------------------------------------------------------------------------------------------------------
    def embed_tokens(self, ids: torch.Tensor):
        """ids: every token of the batch; returns this rank's residual streams [T_l, hc, D] (and Σx² on GPU)."""
        cfg = self.cfg
        if not self.on_gpu and self.pctx.world == 1:
            T = ids.shape[0]
            X = self.embed[ids.long()][:, None, :].expand(T, cfg.hc_streams, cfg.hidden_size).clone()
            return X, None
        return self.pctx.embed(self, ids)

    def forward(self, fb: ForwardBatch, cache) -> torch.Tensor:
        cfg = self.cfg
        T_all = fb.ids.shape[0]
        self.pctx.set_bounds(fb.bounds if fb.bounds is not None else [0, T_all])
        self._dsa = {}                 # DSA selections of this forward's index-source layers
        self._early_sel = {}
        lo, hi = self.pctx.local
        self._tok_local = fb.ids[lo:hi]    # this rank's token ids (multimodal router bias, Engram image skip)
        with region("embed"):
            X, sumsq = self.embed_tokens(fb.ids)
        if cfg.engram_layers:
            cache.write_tokens(fb.out_loc, fb.ids)
        # decode-sized batches run each mHC boundary as one fused kernel; `pend` is then the last sublayer's output
        # with its post / comb coefficients, mixed into X by the next boundary (or by post_mix before anything else
        # reads X)
        fuse = self._boundary_fusable(X)
        pend = None
        for i in range(cfg.n_layers):
            L = self.layers[i]
            if i == cfg.late_layer_start and fb.is_prefill:
                X, sumsq, pend = self._flush(X, sumsq, pend)
                with region("late.enter_tail"):
                    fb, X, sumsq = self._enter_tail(fb, X, sumsq)
            if L.engram is not None:
                X, sumsq, pend = self._flush(X, sumsq, pend)
                with region("engram"):
                    X, sumsq = self.engram(i, X, sumsq, fb, cache)
            if cfg.plain_residual:
                with region("norm"):
                    h, hq = self.plain_norm(X, L.attn_norm, want_fp8=self.on_gpu)
                a = self.attention(i, h, hq, fb, cache)
                X = self.plain_add(X, a)
                with region("norm"):
                    h, hq = self.plain_norm(X, L.ffn_norm, want_fp8=self.on_gpu)
                X = self.plain_add(X, self.ffn(i, h, hq))
                continue
            if fuse:
                with region("mhc.boundary"):
                    h, hq, post, comb = self.hc_boundary(X, pend, L.attn_hc, L.attn_norm)
                a = self.attention(i, h, hq, fb, cache)
                with region("mhc.boundary"):
                    h, hq, post, comb = self.hc_boundary(X, (a, post, comb), L.ffn_hc, L.ffn_norm)
                pend = (self.ffn(i, h, hq), post, comb)
                continue
            with region("mhc.coeffs"):
                pre, post, comb = self.hc_coeffs(X, sumsq, L.attn_hc)
            with region("mhc.pre_norm"):
                h, hq = self.pre_norm(X, pre, L.attn_norm, want_fp8=self.on_gpu)
            a = self.attention(i, h, hq, fb, cache)
            self._tr(f"{i}.attn_in", h); self._tr(f"{i}.attn_pre", pre); self._tr(f"{i}.attn_out", a)
            with region("mhc.post_mix"):
                X, sumsq = self.post_mix(X, a, post, comb)
            self._tr(f"{i}.X_attn", X)
            with region("mhc.coeffs"):
                pre, post, comb = self.hc_coeffs(X, sumsq, L.ffn_hc)
            with region("mhc.pre_norm"):
                h, hq = self.pre_norm(X, pre, L.ffn_norm, want_fp8=self.on_gpu)
            f = self.ffn(i, h, hq)
            self._tr(f"{i}.ffn_in", h); self._tr(f"{i}.ffn_out", f)
            with region("mhc.post_mix"):
                X, sumsq = self.post_mix(X, f, post, comb)
            self._tr(f"{i}.X_ffn", X)
        X, sumsq, pend = self._flush(X, sumsq, pend)
        with region("head"):
            return self.logits(X, sumsq, fb)

    def _enter_tail(self, fb: ForwardBatch, X, sumsq):
        """Bounded late-layer replay: from here on a prefill keeps only each sequence's last late_replay tokens.
        Returns the tail batch (same sequences, fewer tokens; shard bounds recomputed, still sequence-aligned) and
        this rank's rows of X / sumsq for it."""
        cfg, pc = self.cfg, self.pctx
        cu, R_ = fb.cu_seqlens, cfg.late_replay
        old_bounds = fb.bounds if fb.bounds is not None else [0, cu[-1]]
        keep, tail_cu = [], [0]
        for a, e in zip(cu[:-1], cu[1:]):
            s0 = max(a, e - R_)
            keep += range(s0, e)
            tail_cu.append(tail_cu[-1] + e - s0)
        bounds = [sum(1 for k in keep if k < b) for b in old_bounds]
        lo = old_bounds[pc.rank] if len(old_bounds) > 2 else 0
        hi = old_bounds[pc.rank + 1] if len(old_bounds) > 2 else old_bounds[-1]
        dev = X.device
        keep_t = torch.tensor(keep, dtype=torch.long).to(dev)
        local = torch.tensor([k - lo for k in keep if lo <= k < hi], dtype=torch.long).to(dev)
        rows = torch.tensor([c - 1 for c in tail_cu[1:]], dtype=torch.int32).to(dev)
        tb = ForwardBatch(ids=fb.ids[keep_t], pos=fb.pos[keep_t], out_loc=fb.out_loc[keep_t], is_prefill=True,
                          cu_seqlens=tail_cu, logits_rows=rows, bounds=bounds)
        pc.set_bounds(bounds)
        lo2, hi2 = pc.local
        self._tok_local = tb.ids[lo2:hi2]
        return tb, X[local].contiguous(), (sumsq[local].contiguous() if sumsq is not None else None)

    def _tr(self, name, t):
        if self.trace is not None:
            self.trace.append((name, t.detach().float().cpu().clone()))

    def logits(self, X, sumsq, fb: ForwardBatch) -> torch.Tensor:
        """Final mHC head mix + norm for the requested rows of this rank, gathered, then the (vocab-parallel) head."""
        cfg, pc = self.cfg, self.pctx
        lo, hi = pc.local
        rows = fb.logits_rows
        counts = None
        if rows is not None:
            if pc.world > 1:
                # prefill: one logits row per sequence; shards hold whole sequences
                ends = fb.cu_seqlens[1:]
                counts = [sum(1 for e in ends if pc.bounds[r] < e <= pc.bounds[r + 1]) for r in range(pc.world)]
                local_rows = torch.tensor([e - 1 - lo for e in ends if lo < e <= hi], dtype=torch.long,
                                          device=X.device)
            else:
                local_rows = rows.long()
            X = X[local_rows].contiguous()
            sumsq = sumsq[local_rows] if sumsq is not None else None
        if cfg.plain_residual:
            y, _ = self.plain_norm(X, self.norm_w, want_fp8=False)
        elif not self.on_gpu:
            pre = R.mhc_head_coeffs(X, self.head_hc.fn, self.head_hc.base, self.head_hc.scale, cfg.hc_eps,
                                    cfg.rms_eps)
            y = R.rms_norm(R.mhc_pre_mix(X, pre), self.norm_w, cfg.rms_eps)
        else:
            from ..ops._ext import ext

            T = X.shape[0]
            pre = torch.empty(T, 4, device=X.device)
            if T > 0:
                mix = mhc_mix(X.view(T, X.shape[1] * X.shape[2]), self.head_hc.fn)
                ext().mhc_head_coeffs(mix, sumsq, self.head_hc.base, self.head_hc.scale, X.shape[1] * X.shape[2],
                                      cfg.hc_eps, cfg.rms_eps, pre)
            y, _ = self.pre_norm(X, pre, self.norm_w, want_fp8=False)
        if pc.world > 1:
            y = pc.gather_var(y, counts) if counts is not None else pc.gather_rows(y)
        if not self.on_gpu and pc.world == 1:
            return y @ self.head_w.w.t()
        return pc.lm_head(self, y)


def mhc_mix(x: torch.Tensor, fn: torch.Tensor) -> torch.Tensor:
    """mHC statistics x · fnᵀ (fp32 [T, rows of fn]) on the GPU: the tensor-core GEMM for prefill-sized batches, a
    CUDA-core kernel with one CTA per (token, 8 rows) for decode-sized ones (a GEMM would run one tile split over
    the 28k-long K)."""
    T = x.shape[0]
    if T <= 64:
        from ..ops._ext import ext

        out = torch.empty(T, fn.shape[0], dtype=torch.float32, device=x.device)
        ext().mhc_stats_small(x, fn, fn.shape[0], out)
        return out
    return bf16_gemm(x, fn, out_dtype=torch.float32)


def head_bmm(x: torch.Tensor, w: torch.Tensor, tail: int = 0, out_dtype=torch.bfloat16) -> torch.Tensor:
    """Per-head matmul: x [T, H, K(+tail)] · w[h]ᵀ (w [H, N, K]) -> [T, H, N(+tail)]; with ``tail`` the last
    columns of x are appended unchanged (the absorbed query [q_nope · W_uk | q_rope]) in ``out_dtype``."""
    T, H, Kx = x.shape
    N, K = w.shape[1], w.shape[2]
    if not x.is_cuda:
        out = torch.einsum("thk,hnk->thn", x[..., :K].float(), w.float())
        return torch.cat([out, x[..., K:K + tail].float()], dim=-1) if tail else out
    if _head_bmm_direct(x, w, tail, out_dtype):
        # decode batch: one swap-AB tcgen05 launch reads the token rows in place and writes [T, H, N + tail]
        from ..ops._ext import ext
        out = torch.empty(T, H, N + tail, dtype=out_dtype, device=x.device)
        ext().head_bmm(x, w, tail, out, None)
        return out
    if tail:                            # two strided copies into the output, no concatenation
        out = torch.empty(T, H, N + tail, dtype=out_dtype, device=x.device)
        out[..., :N] = head_bmm(x[..., :K], w)
        out[..., N:] = x[..., K:K + tail]
        return out
    x = x[..., :K]
    Tp = ((T + 127) // 128) * 128
    # head-major rows, each head's block padded to 128 rows; the padding rows are never read back (every output
    # row depends only on its own input row), so they stay uninitialised
    xt = torch.empty(H, Tp, K, dtype=torch.bfloat16, device=x.device)
    xt[:, :T] = x.transpose(0, 1)
    key = (H, Tp // 128, x.device)
    mbe = _HEAD_BLOCKS.get(key)
    if mbe is None:
        mbe = torch.arange(H, dtype=torch.int32, device=x.device).repeat_interleave(Tp // 128)
        _HEAD_BLOCKS[key] = mbe
    out = bf16_gemm(xt.view(H * Tp, K), w.reshape(H * N, K), m_block_expert=mbe, n_per_group=N)
    return out.view(H, Tp, N)[:, :T].transpose(0, 1)


def _head_bmm_direct(x: torch.Tensor, w: torch.Tensor, tail: int, out_dtype) -> bool:
    """Whether the decode-batch kernel takes this per-head matmul: at most 256 tokens, 128-multiple N, 64-multiple K,
    8-multiple tail, bf16 operands with 16-byte aligned rows (its tensor maps), bf16 / fp16 output.
    CARBON_HEAD_BMM=0 turns it off (the grouped-GEMM path over head-major copies then runs)."""
    T, H, Kx = x.shape
    N, K = w.shape[1], w.shape[2]
    return (_HEAD_BMM_ON and 0 < T <= 256 and N % 128 == 0 and K % 64 == 0 and x.dtype == torch.bfloat16
            and w.dtype == torch.bfloat16 and w.is_contiguous() and x.stride(2) == 1 and x.stride(1) % 8 == 0
            and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0 and out_dtype in (torch.bfloat16, torch.float16)
            and Kx >= K + tail and tail % 8 == 0)


_HEAD_BMM_ON = os.environ.get("CARBON_HEAD_BMM", "1") != "0"
_HEAD_BLOCKS: Dict[tuple, torch.Tensor] = {}      # expert (= head) of each 128-row block, per (heads, blocks, device)

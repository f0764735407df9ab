"""Typed configuration for the engine: model shape, parallel layout, quantisation and kernel flags.

One dataclass tree drives the CPU fp32 oracle (``carbon_b200.ref``), the GPU model (``carbon_b200.models``) and the
serving engine (``carbon_b200.engine``).  The reference keeps these facts as module constants and domain checks
(``king_v10/bundle_v9/slots.py:133-158`` checks 40 layers / hidden 5120 / 384 experts / top-6; ``moe_front.py:17``
etc.); here every one of them is a field so that the DeepSeek-V3 shape (61 layers, hidden 7168, 256 experts top-8)
and the V4.1-Flash shape are both expressible.

Overrides: ``ModelConfig.from_dict`` / ``from_yaml`` and ``CARBON_<FIELD>=value`` environment variables
(``apply_env``), mirroring the reference's module-level switches (``EVL_ON``, ``WTILE`` …) with one typed mechanism.
"""
from __future__ import annotations

import dataclasses
import json
import math
import os
from dataclasses import dataclass, field
from typing import Any, Dict, Optional


@dataclass
class ModelConfig:
    """Shape of a DeepSeek-V3/V4-style transformer: MLA + DSA indexer + fine-grained MoE + mHC."""

    vocab_size: int = 129280
    hidden_size: int = 7168
    n_layers: int = 61
    n_dense_layers: int = 3            # first layers use a dense SwiGLU FFN instead of MoE
    dense_intermediate: int = 18432
    # MLA attention
    n_heads: int = 128
    q_lora_rank: int = 1536            # 0 => q projected directly from hidden
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    rope_theta: float = 10000.0
    # YaRN context extension (DeepSeek-V3's rope_scaling): 1.0 = off
    rope_factor: float = 1.0
    rope_orig_max: int = 4096
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    rope_mscale_all_dim: float = 1.0
    max_position: int = 16384
    # DSA lightning indexer (0 heads => dense attention)
    index_n_heads: int = 64
    index_head_dim: int = 128
    index_topk: int = 2048
    # DSA selection sharing (DeepSeek-V4.1 style): when non-empty, only these layers run the indexer; every later
    # layer reuses the selection of the most recent source layer; layers before the first source attend densely.
    # Empty: every layer runs its own indexer.
    index_sources: tuple = ()
    # indexer q and k in MXFP4 (e2m1 + UE8M0 per 32 dims; the reference's 68-byte index keys,
    # dec/cuda_paged_logits.py:35-37): both are rounded to fp4 values before the logits
    index_fp4: bool = False
    # indexer q and k in fp8 e4m3 with one UE8M0 scale per 128-dim row (per head for q), the DeepSeek-V3.2 indexer
    # precision: the prefill logits run as block-scaled fp8 tcgen05 MMAs; decode sees the same rounded values
    index_fp8: bool = False
    # latent KV cache in fp8: per token, the kv_lora_rank latent values in e4m3 with one UE8M0 scale per 64-dim atom
    # and (MLA) the RoPE key in fp16 -- 656 bytes per MLA token instead of 1152 in bf16, 528 per latent-MQA token
    # instead of 1024 (the reference's fp8 SWA pages: king_v10/bundle_v9/cuda_prefill_attn.py:2312-2340)
    kv_fp8: bool = False
    # MLA prefill over sequences longer than this runs as absorbed sparse attention over each query's top-k cached
    # latent rows (cost linear in length at a fixed top-k) instead of the dense causal kernel with a DSA key mask
    # (cheaper for short prompts: 320 vs 1088 MACs per key and head); 0 = always the dense kernel
    sparse_prefill_min: int = 12288
    # per-head learned attention sink: one extra logit in each softmax denominator (attn.sink [n_heads] fp32)
    attn_sink: bool = False
    # attention kind.  "mla": q/k = [nope | RoPE] per head, keys and values up-projected from the kv latent (wkv_b);
    # "latent_mqa" (DeepSeek-V4 family): every head's q lives in the kv_lora_rank-dim latent space, the one shared
    # KV head is the normalised latent itself (its last qk_rope_head_dim dims carry RoPE), the value is the same
    # row, and the output's RoPE dims are rotated back by the query position
    # (king_v10/bundle_v9/cuda_prefill_attn.py:5124-5195: q [s,64,512], kv [s,1,512], d_qk = d_v = 512, rope 64)
    attn_kind: str = "mla"
    # grouped low-rank output projection: heads in o_groups groups, each group's concatenated head outputs projected
    # to o_lora_rank (wo_a, a grouped matmul), then wo_b maps the o_groups*o_lora_rank concatenation to hidden
    # (reference: wo_a grouped einsum "bhr,hdr->bhd" with 8 groups, wo_b 8192 -> hidden; prefill_gemm.py:15-21).
    # 0: one dense wo.
    o_groups: int = 0
    o_lora_rank: int = 0
    # sliding window: every query also attends to the last swa_window positions (itself included); with an indexer
    # the top-k selection is taken over the keys older than the window, so the two sets are disjoint
    # (reference: SWA window 128, per-row index width 512 top-k + 128 window; rehome_attn.py:8,17-19).  0: off.
    swa_window: int = 0
    # Engram (hashed n-gram memory; reference layers 1 and 14, peer_read.py:15, dspd_w22/dspd/engram.py:259-268):
    # each token's n-grams (orders engram_orders, engram_heads hash heads per order) index one row of a hashed table
    # per column; the engram_dim-wide rows of all columns are concatenated, projected by wkv to one key per mHC stream
    # plus one shared value, and every stream gets x_c += sigmoid(clamp(<rms(x_c)*q_w, rms(k_c)*k_w> / sqrt(D))) * value.
    # The hash and the gate are this framework's own definitions (the reference's live in its sealed engine).
    engram_layers: tuple = ()
    engram_orders: tuple = (2, 3)
    engram_heads: int = 12
    engram_dim: int = 256
    engram_rows: int = 4096            # rows per column (each column's modulus is the first prime >= this)
    engram_clamp: float = 10.0
    # multimodal: tokens with this id are image tokens; they rank experts with a second router bias
    # (ffn.gate.bias_img) and take no Engram update (cuda_moe_front.py:265-269, dspd_w22/dspd/engram.py:261).
    # -1: text only.
    image_token_id: int = -1
    # bounded replay of the late layers (the reference's "decoder SWA bounded replay": layers >= 20 of a prefill run
    # only each request's last <= 128 tokens; rehome_block.py:195-197, dspd_w22/dspd/mlp.py:15-18).  Layers from
    # late_layer_start on are window-only (no DSA selection).  A prefill keeps only each request's last late_replay
    # tokens from that layer on; keys older than that tail never exist at the late layers, for the request's later
    # decode steps too.  -1: off.
    late_layer_start: int = -1
    late_replay: int = 128
    # MoE
    n_routed_experts: int = 256
    n_activated_experts: int = 8
    n_shared_experts: int = 1
    moe_intermediate: int = 2048
    score_func: str = "sigmoid"        # sigmoid | sqrtsoftplus | softmax
    n_groups: int = 1                  # group-limited routing (DeepSeek-V3: 8 groups, the best 4 by top-2 score sum)
    topk_groups: int = 1
    route_scale: float = 2.5
    norm_topk_prob: bool = True
    swiglu_limit: float = 0.0          # 0 => no clamp
    # mHC (manifold-constrained hyper-connections)
    hc_mult: int = 4   # 0: no hyper-connections (one residual stream, x + f(norm(x)): DeepSeek-V3 / V3.2)
    sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    rms_eps: float = 1e-6
    init_std: float = 0.02
    tie_word_embeddings: bool = False

    # ---- derived -------------------------------------------------------------------------------------------------
    @property
    def qk_head_dim(self) -> int:
        """Per-head q (and k) width."""
        if self.attn_kind == "latent_mqa":
            return self.kv_lora_rank
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def latent_dim(self) -> int:
        """Width of one cached token row: MLA keeps [kv_lora | RoPE key]; latent MQA keeps the kv_lora_rank row."""
        if self.attn_kind == "latent_mqa":
            return self.kv_lora_rank
        return self.kv_lora_rank + self.qk_rope_head_dim

    @property
    def head_out_dim(self) -> int:
        """Per-head attention output width (the input of the output projection per head)."""
        return self.kv_lora_rank if self.attn_kind == "latent_mqa" else self.v_head_dim

    @property
    def plain_residual(self) -> bool:
        """hc_mult == 0: the standard pre-norm residual instead of mHC (checkpoints without hyper-connections)."""
        return self.hc_mult == 0

    @property
    def hc_streams(self) -> int:
        """Residual streams carried between sublayers (one for the plain residual)."""
        return max(1, self.hc_mult)

    @property
    def hc_mix_dim(self) -> int:
        """Number of mHC mixing outputs: hc pre + hc post + hc×hc comb."""
        return 2 * self.hc_mult + self.hc_mult * self.hc_mult

    @property
    def use_indexer(self) -> bool:
        return self.index_n_heads > 0 and self.index_topk > 0

    def is_late_layer(self, layer: int) -> bool:
        return 0 <= self.late_layer_start <= layer

    def index_source(self, layer: int) -> Optional[int]:
        """Layer whose DSA selection this layer's attention uses (None: dense or window-only attention)."""
        if not self.use_indexer or self.is_late_layer(layer):
            return None
        if not self.index_sources:
            return layer
        srcs = [s for s in self.index_sources if s <= layer]
        return max(srcs) if srcs else None

    def has_indexer(self, layer: int) -> bool:
        """Whether this layer holds indexer weights and writes indexer keys to the cache."""
        if self.is_late_layer(layer):
            return False
        return self.use_indexer and (not self.index_sources or layer in self.index_sources)

    def is_moe_layer(self, layer: int) -> bool:
        return layer >= self.n_dense_layers and self.n_routed_experts > 0

    @property
    def engram_cols(self) -> int:
        return len(self.engram_orders) * self.engram_heads

    @property
    def engram_primes(self) -> tuple:
        """Modulus of each hash column: distinct primes >= engram_rows, in column order."""
        out, n = [], max(2, self.engram_rows)
        while len(out) < self.engram_cols:
            if all(n % d for d in range(2, int(n ** 0.5) + 1)):
                out.append(n)
            n += 1
        return tuple(out)

    @property
    def engram_table_rows(self) -> int:
        return sum(self.engram_primes)

    @property
    def softmax_scale(self) -> float:
        s = self.qk_head_dim ** -0.5
        if self.rope_factor > 1.0:          # YaRN attention temperature, applied to the logits as mscale^2
            m = 0.1 * self.rope_mscale_all_dim * math.log(self.rope_factor) + 1.0
            s *= m * m
        return s

    @property
    def rope(self):
        """RoPE spec for ``ref.ops.rope_cos_sin``: theta, or (theta, factor, orig_max, beta_fast, beta_slow) with YaRN."""
        if self.rope_factor > 1.0:
            return (self.rope_theta, self.rope_factor, self.rope_orig_max, self.rope_beta_fast, self.rope_beta_slow)
        return self.rope_theta

    # ---- construction --------------------------------------------------------------------------------------------
    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        unknown = set(d) - names
        if unknown:
            raise ValueError(f"unknown ModelConfig fields: {sorted(unknown)}")
        return cls(**d)

    @classmethod
    def from_yaml(cls, path: str) -> "ModelConfig":
        import yaml

        with open(path) as f:
            return cls.from_dict(yaml.safe_load(f) or {})

    @classmethod
    def from_hf(cls, src) -> "ModelConfig":
        """A Hugging Face DeepSeek-V3 / V3.2 ``config.json`` (a path, a directory holding one, or its dict):
        plain residual (no hyper-connections), group-limited sigmoid routing, YaRN RoPE scaling and, for V3.2,
        the DSA indexer.  The multi-token-prediction layers are not part of the model here."""
        if not isinstance(src, dict):
            path = os.path.join(src, "config.json") if os.path.isdir(src) else src
            with open(path) as f:
                src = json.load(f)
        d = src
        kw: Dict[str, Any] = dict(
            vocab_size=d["vocab_size"], hidden_size=d["hidden_size"], n_layers=d["num_hidden_layers"],
            n_dense_layers=d.get("first_k_dense_replace", 0), dense_intermediate=d["intermediate_size"],
            n_heads=d["num_attention_heads"], q_lora_rank=d.get("q_lora_rank") or 0, kv_lora_rank=d["kv_lora_rank"],
            qk_nope_head_dim=d["qk_nope_head_dim"], qk_rope_head_dim=d["qk_rope_head_dim"],
            v_head_dim=d["v_head_dim"], rope_theta=float(d.get("rope_theta", 10000.0)),
            max_position=d.get("max_position_embeddings", 4096),
            n_routed_experts=d.get("n_routed_experts") or 0, n_activated_experts=d.get("num_experts_per_tok") or 0,
            n_shared_experts=d.get("n_shared_experts") or 0, moe_intermediate=d.get("moe_intermediate_size", 0),
            score_func=d.get("scoring_func", "softmax"), route_scale=float(d.get("routed_scaling_factor", 1.0)),
            norm_topk_prob=bool(d.get("norm_topk_prob", False)), n_groups=d.get("n_group") or 1,
            topk_groups=d.get("topk_group") or 1, rms_eps=float(d.get("rms_norm_eps", 1e-6)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)), hc_mult=0,
            index_n_heads=d.get("index_n_heads", 0), index_head_dim=d.get("index_head_dim", 128),
            index_topk=d.get("index_topk", 0))
        rs = d.get("rope_scaling") or {}
        if rs.get("type", rs.get("rope_type")) == "yarn":
            kw.update(rope_factor=float(rs["factor"]),
                      rope_orig_max=int(rs.get("original_max_position_embeddings", 4096)),
                      rope_beta_fast=float(rs.get("beta_fast", 32)), rope_beta_slow=float(rs.get("beta_slow", 1)),
                      rope_mscale_all_dim=float(rs.get("mscale_all_dim", 1.0)))
        return cls(**kw)

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def validate(self) -> None:
        assert self.hidden_size % 128 == 0 or self.hidden_size < 128, "hidden must be a multiple of 128 (fp8 1x128 blocks)"
        assert self.qk_rope_head_dim % 2 == 0
        assert self.n_activated_experts <= max(self.n_routed_experts, 1)
        assert self.score_func in ("sigmoid", "sqrtsoftplus", "softmax")
        if self.use_indexer:
            assert self.index_head_dim >= self.qk_rope_head_dim
        assert self.attn_kind in ("mla", "latent_mqa")
        if self.attn_kind == "latent_mqa":
            assert 0 < self.qk_rope_head_dim < self.kv_lora_rank
        if self.o_groups:
            assert self.n_heads % self.o_groups == 0 and self.o_lora_rank > 0
        assert self.swa_window >= 0
        if self.engram_layers:
            assert self.engram_dim % 32 == 0 and self.engram_cols > 0 and min(self.engram_orders) >= 1
        if self.late_layer_start >= 0:
            assert self.attn_kind == "latent_mqa" and 0 < self.swa_window <= self.late_replay, \
                "bounded late-layer replay needs window-only latent-MQA late layers with swa_window <= late_replay"
            assert all(l < self.late_layer_start for l in self.engram_layers), "Engram layers precede the late layers"


def tiny_config() -> ModelConfig:
    """The tiny CPU model (2 layers, hidden 256, vocab 1024) checked against the fp32 oracle within 1e-4."""
    return ModelConfig(
        vocab_size=1024, hidden_size=256, n_layers=2, n_dense_layers=0, dense_intermediate=512,
        n_heads=4, q_lora_rank=128, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32,
        max_position=1024,
        index_n_heads=2, index_head_dim=32, index_topk=32,
        n_routed_experts=8, n_activated_experts=2, n_shared_experts=1, moe_intermediate=128,
        score_func="sigmoid", route_scale=1.0,
        hc_mult=4, sinkhorn_iters=20, rms_eps=1e-6,
    )


def deepseek_v3_config() -> ModelConfig:
    """The full-size DeepSeek-V3/V4-class model of the serving benchmark (61 layers, hidden 7168, 256 experts top-8).
    The indexer stays bf16 here: the fp8 option (index_fp8) measured slower end to end on B200 (the rounding of q and
    k costs more than the fp8 logits save until it is fused into the q projection)."""
    return ModelConfig()


def small_gpu_config() -> ModelConfig:
    """A 4-layer slice at reduced width that keeps every full-size kernel constraint (multiples of 128)."""
    return ModelConfig(
        vocab_size=8192, hidden_size=1024, n_layers=4, n_dense_layers=1, dense_intermediate=2048,
        n_heads=16, q_lora_rank=512, kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
        max_position=8192, index_n_heads=16, index_head_dim=128, index_topk=256,
        n_routed_experts=32, n_activated_experts=4, n_shared_experts=1, moe_intermediate=256,
        route_scale=2.5,
    )


def tiny_v4_config() -> ModelConfig:
    """The tiny CPU model in the DeepSeek-V4 attention layout: latent MQA (one 64-dim latent head with 16 RoPE dims),
    grouped low-rank output projection, sliding window 16, per-head sinks, DSA index sources, sqrt-softplus router."""
    return tiny_config().replace(attn_kind="latent_mqa", o_groups=2, o_lora_rank=64, swa_window=16, attn_sink=True,
                                 index_sources=(0,), index_topk=16, score_func="sqrtsoftplus", engram_layers=(1,),
                                 engram_heads=2, engram_dim=64, engram_rows=97, index_fp4=True)


def deepseek_v4_config() -> ModelConfig:
    """DeepSeek-V4.1-Flash-shaped model (the reference's target model): 40 layers, hidden 5120, 64 heads of
    latent MQA over a 512-dim latent (64 RoPE dims), q_lora 1280, 8 output groups with o_lora 1024, window 128,
    indexer 32 heads x 128 top-512 on source layers 2, 8, 14, 384 experts top-6 (intermediate 2304, sqrt-softplus
    router), mHC 4 streams, Engram on layers 1 and 14 (24 hash columns of 256-dim rows).  The compressed KV pool is
    not modelled (its keys come from the same latent cache); MXFP4 experts load through the checkpoint format."""
    return ModelConfig(
        vocab_size=129280, hidden_size=5120, n_layers=40, n_dense_layers=0, dense_intermediate=12288,
        n_heads=64, q_lora_rank=1280, kv_lora_rank=512, qk_nope_head_dim=448, qk_rope_head_dim=64, v_head_dim=512,
        max_position=65536, index_n_heads=32, index_head_dim=128, index_topk=512, index_sources=(2, 8, 14),
        attn_sink=True, attn_kind="latent_mqa", o_groups=8, o_lora_rank=1024, swa_window=128, engram_layers=(1, 14),
        index_fp4=True, late_layer_start=20, late_replay=128,
        engram_orders=(2, 3), engram_heads=12, engram_dim=256, engram_rows=1 << 20,
        n_routed_experts=384, n_activated_experts=6, n_shared_experts=1, moe_intermediate=2304,
        score_func="sqrtsoftplus", route_scale=2.5,
    )


PRESETS = {"tiny": tiny_config, "tiny_v4": tiny_v4_config, "deepseek_v3": deepseek_v3_config,
           "small": small_gpu_config, "deepseek_v4": deepseek_v4_config}


@dataclass
class ParallelConfig:
    """Parallel layout on one node: tensor-parallel attention, expert-parallel MoE, DP-attention."""

    world_size: int = 1
    rank: int = 0
    tp: int = 1                  # attention tensor parallel (heads split)
    ep: int = 1                  # expert parallel (experts split)
    dp_attention: bool = False   # attention data-parallel (each rank its own requests), MoE EP
    vocab_parallel: bool = True  # embedding / LM head split over ranks, served from peer HBM

    def validate(self, cfg: ModelConfig) -> None:
        assert self.world_size >= 1
        if self.tp > 1:
            assert cfg.n_heads % self.tp == 0, "heads must divide TP"
        if self.ep > 1:
            assert cfg.n_routed_experts % self.ep == 0, "experts must divide EP"


@dataclass
class KernelFlags:
    """Per-path switches (the reference's lever constants, as one typed record)."""

    fused_ep_moe: bool = True       # in-kernel NVLink dispatch/combine (else NCCL all-to-all baseline)
    fused_tp_attn: bool = True      # o_proj GEMM -> reduce-scatter over peer memory (else NCCL)
    peer_vocab: bool = True         # embedding / LM head from peer HBM (else NCCL all-gather)
    cuda_graphs: bool = True        # capture decode steps
    fp8_gemm: bool = True           # block-scaled fp8 GEMMs (else bf16)
    sparse_attention: bool = True   # DSA top-k attention when the model has an indexer
    moe_align: int = 0              # expert segment padding: 0 automatic, 128, or 256 (CTA-pair GEMM tiles)

    @classmethod
    def from_env(cls) -> "KernelFlags":
        f = cls()
        apply_env(f, prefix="CARBON_")
        return f


@dataclass
class EngineConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    flags: KernelFlags = field(default_factory=KernelFlags)
    kv_page_size: int = 64
    max_batch: int = 256
    max_seq_len: int = 8192
    decode_graph_buckets: tuple = (1, 2, 4, 8, 16, 32, 64, 128, 256)
    seed: int = 0
    weight_layer_sets: Optional[int] = None  # None => one weight set per layer


def _coerce(val: str, typ):
    if typ in (bool, "bool"):
        return val.lower() in ("1", "true", "yes", "on")
    if typ in (int, "int"):
        return int(val)
    if typ in (float, "float"):
        return float(val)
    return val


def apply_env(obj, prefix: str = "CARBON_") -> None:
    """Override dataclass fields from ``<prefix><FIELD_NAME_UPPER>`` environment variables."""
    for f in dataclasses.fields(obj):
        key = prefix + f.name.upper()
        if key in os.environ:
            setattr(obj, f.name, _coerce(os.environ[key], f.type))


def dump(obj) -> str:
    return json.dumps(dataclasses.asdict(obj), sort_keys=True)

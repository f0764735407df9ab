"""Checkpoints in the DeepSeek block-scaled fp8 format (safetensors).

* A quantised linear weight ``<name>`` is stored as float8_e4m3fn [N, K] next to ``<name>_scale_inv`` — fp32
  [ceil(N/128), ceil(K/128)], the value that multiplies each 128×128 block (DeepSeek-V3's ``weight_scale_inv``).
* Everything else (norms, router, mHC parameters, embedding, head) is stored in bf16 / fp32 as is.
* Experts may be stored stacked (``ffn.experts.w1`` [E, I, D]) or per expert (``ffn.experts.{e}.w1``); both load.
* Routed-expert weights may instead be MXFP4 (the reference's expert format, ``moe_prefill.py:14-16``): ``<name>`` is
  uint8 [.., N, K/2] (two e2m1 codes per byte, low nibble first) next to ``<name>_scale`` uint8 [.., N, K/32] (UE8M0
  exponent of each 32-element block).  They load as their exact values; the engine then stores them in its fp8
  128x128 block format (exact whenever a 128x128 block's 32-element scales span at most 2^7, i.e. almost always;
  otherwise the smallest values round).

``save_checkpoint`` writes this format from a state dict (quantising the fp8 names with ``ref.ops.quant_fp8_blocks``,
so scales are powers of two); ``CheckpointSource`` is a ``WeightSource`` that reads it lazily, dequantising on the
target device.  The reference receives its weights from the sealed engine in the same fp8 + 128×128 block format
(``king_v10/bundle_v9/placement.py:133-134``).
"""
from __future__ import annotations

import json
import os
import re
from typing import Dict, Iterable, Optional

import torch

from ..config import ModelConfig
from ..ref import ops as R
from .weights import WeightSource

FP8_SUFFIXES = ("wq_a.weight", "wq_b.weight", "wkv_a.weight", "wkv_b.weight", "wo.weight", "wo_b.weight",
                "engram.wkv.weight", "ffn.w1", "ffn.w2",
                "ffn.w3", "experts.w1", "experts.w2", "experts.w3", "shared.w1", "shared.w2", "shared.w3")
_EXPERT_RE = re.compile(r"^(layers\.\d+\.ffn\.experts)\.(\d+)\.(w[123])$")


def is_fp8_name(name: str) -> bool:
    return name.endswith(FP8_SUFFIXES)


# Hugging Face DeepSeek-V3 / V3.2 module names -> this loader's names (the same correspondence DeepSeek's own
# inference code applies when it converts those checkpoints).  Linear layers whose name here has no ".weight" (the
# FFN matrices) take "<name>_scale_inv" for the HF "weight_scale_inv".
_HF_ATTN = {"q_a_proj": "attn.wq_a", "q_b_proj": "attn.wq_b", "q_proj": "attn.wq", "kv_a_proj_with_mqa": "attn.wkv_a",
            "kv_b_proj": "attn.wkv_b", "o_proj": "attn.wo", "q_a_layernorm": "attn.q_norm",
            "kv_a_layernorm": "attn.kv_norm", "indexer.wq_b": "attn.indexer.wq", "indexer.wk": "attn.indexer.wk",
            "indexer.k_norm": "attn.indexer.k_norm", "indexer.weights_proj": "attn.indexer.weights_proj"}
_HF_FFN = {"gate_proj": "w1", "down_proj": "w2", "up_proj": "w3"}
_HF_LAYER_RE = re.compile(r"^model\.layers\.(\d+)\.(.+)$")


def hf_to_internal(name: str, n_layers: int) -> Optional[str]:
    """Internal name of a Hugging Face DeepSeek checkpoint tensor; None for tensors the model does not use (layers
    at or beyond ``n_layers``, e.g. the multi-token-prediction layer).  Names not in HF form pass through."""
    top = {"model.embed_tokens.weight": "embed.weight", "model.norm.weight": "norm.weight",
           "lm_head.weight": "head.weight"}
    if name in top:
        return top[name]
    m = _HF_LAYER_RE.match(name)
    if m is None:
        return None if name.startswith("model.") else name
    layer, rest = int(m.group(1)), m.group(2)
    if layer >= n_layers:
        return None
    pre = f"layers.{layer}."
    if rest == "input_layernorm.weight":
        return pre + "attn_norm.weight"
    if rest == "post_attention_layernorm.weight":
        return pre + "ffn_norm.weight"
    if rest.startswith("self_attn."):
        mod, _, leaf = rest[len("self_attn."):].rpartition(".")
        if mod in _HF_ATTN and leaf in ("weight", "bias", "weight_scale_inv"):
            return pre + _HF_ATTN[mod] + "." + leaf
        return None
    if rest.startswith("mlp."):
        r = rest[len("mlp."):]
        if r == "gate.weight":
            return pre + "ffn.gate.weight"
        if r == "gate.e_score_correction_bias":
            return pre + "ffn.gate.bias"
        mod, _, leaf = r.rpartition(".")
        if leaf not in ("weight", "weight_scale_inv"):
            return None
        suffix = "" if leaf == "weight" else "_scale_inv"
        parts = mod.split(".")
        if len(parts) == 3 and parts[0] == "experts" and parts[2] in _HF_FFN:
            return f"{pre}ffn.experts.{int(parts[1])}.{_HF_FFN[parts[2]]}{suffix}"
        if len(parts) == 2 and parts[0] == "shared_experts" and parts[1] in _HF_FFN:
            return f"{pre}ffn.shared.{_HF_FFN[parts[1]]}{suffix}"
        if len(parts) == 1 and parts[0] in _HF_FFN:
            return f"{pre}ffn.{_HF_FFN[parts[0]]}{suffix}"
    return None


def save_checkpoint(state: Dict[str, torch.Tensor], path: str, shard_bytes: int = 2 << 30,
                    per_expert: bool = False, mxfp4_experts: bool = False) -> None:
    """Write ``state`` (fp32 tensors) as fp8 block-scaled safetensors shards + an index JSON (routed experts in MXFP4
    when ``mxfp4_experts``)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    out: Dict[str, torch.Tensor] = {}
    for name, t in state.items():
        if mxfp4_experts and name.endswith(("experts.w1", "experts.w2", "experts.w3")):
            qs = [R.quant_mxfp4(t[e].float()) for e in range(t.shape[0])]
            if per_expert:
                for e, (q, s) in enumerate(qs):
                    n2 = f"{name[:-3]}.{e}.{name[-2:]}"
                    out[n2], out[n2 + "_scale"] = q, s
            else:
                out[name] = torch.stack([q for q, _ in qs])
                out[name + "_scale"] = torch.stack([s for _, s in qs])
        elif name.endswith("engram.table"):
            # Engram rows: e4m3 with one UE8M0 byte per 32 elements (the reference's 256 e4m3 + UE8M0/32 rows)
            out[name], out[name + "_sf32"] = R.quant_fp8_rows32(t.float())
        elif is_fp8_name(name):
            if t.dim() == 3:
                mats = [(f"{name[:-3]}.{e}.{name[-2:]}" if per_expert else None, t[e]) for e in range(t.shape[0])]
                if per_expert:
                    for n2, m in mats:
                        q, s = R.quant_fp8_blocks(m.float())
                        out[n2], out[n2 + "_scale_inv"] = q, s
                else:
                    qs = [R.quant_fp8_blocks(m.float()) for _, m in mats]
                    out[name] = torch.stack([q for q, _ in qs])
                    out[name + "_scale_inv"] = torch.stack([s for _, s in qs])
            else:
                q, s = R.quant_fp8_blocks(t.float())
                out[name], out[name + "_scale_inv"] = q, s
        else:
            out[name] = t.to(torch.bfloat16) if t.dim() >= 2 and t.numel() > 4096 else t.float()
    index, shard, size, k = {}, {}, 0, 0

    def flush():
        nonlocal shard, size, k
        if shard:
            fn = f"model-{k:05d}.safetensors"
            save_file({n: v.contiguous() for n, v in shard.items()}, os.path.join(path, fn))
            for n in shard:
                index[n] = fn
            k += 1
            shard, size = {}, 0

    for n, v in out.items():
        shard[n] = v
        size += v.numel() * v.element_size()
        if size >= shard_bytes:
            flush()
    flush()
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": index}, f)


class CheckpointSource(WeightSource):
    """WeightSource over a directory of safetensors shards (block-scaled fp8 names dequantised on load).  Both this
    loader's names and Hugging Face DeepSeek names (``model.layers.N.self_attn.q_a_proj.weight``, ``weight_scale_inv``,
    ``mlp.experts.E.gate_proj`` ...) are accepted; parameters that HF DeepSeek checkpoints do not carry (mHC) must then
    come under this loader's names in the same directory."""

    def __init__(self, cfg: ModelConfig, path: str, layer_sets: Optional[int] = None):
        super().__init__(cfg, state=None, seed=0, layer_sets=layer_sets)
        from safetensors import safe_open

        self.path = path
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                wm = json.load(f)["weight_map"]
        else:
            wm = {}
            for fn in sorted(os.listdir(path)):
                if fn.endswith(".safetensors"):
                    with safe_open(os.path.join(path, fn), "pt") as h:
                        for n in h.keys():
                            wm[n] = fn
        self.stored: Dict[str, str] = {}                 # internal name -> name in the file (HF checkpoints)
        if any(n.startswith("model.") for n in wm):
            conv = {}
            for n, fn in wm.items():
                k = hf_to_internal(n, cfg.n_layers)
                if k is not None:
                    conv[k] = fn
                    if k != n:
                        self.stored[k] = n
            wm = conv
        self.weight_map = wm
        self._handles = {}
        self._safe_open = safe_open

    def _tensor(self, name: str) -> torch.Tensor:
        fn = self.weight_map[name]
        h = self._handles.get(fn)
        if h is None:
            h = self._safe_open(os.path.join(self.path, fn), "pt")
            self._handles[fn] = h
        return h.get_tensor(self.stored.get(name, name))

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def get(self, name: str, device, rows: Optional[slice] = None) -> torch.Tensor:
        cname = self.canonical(name)
        if cname not in self.weight_map and cname.endswith(("experts.w1", "experts.w2", "experts.w3")):
            # per-expert storage: assemble the requested experts
            base, w = cname.rsplit(".", 1)
            E = self.cfg.n_routed_experts
            rng = range(E) if rows is None else range(rows.start or 0, rows.stop if rows.stop is not None else E)
            mats = [self._load(f"{base}.{e}.{w}", device) for e in rng]
            return torch.stack(mats)
        t = self._load(cname, device)
        return t if rows is None else t[rows]

    def _load(self, name: str, device) -> torch.Tensor:
        t = self._tensor(name)
        if t.dtype == torch.uint8 and self.has(name + "_scale"):          # MXFP4
            s = self._tensor(name + "_scale")
            if t.dim() == 3:
                return torch.stack([R.dequant_mxfp4(t[e].to(device), s[e].to(device)) for e in range(t.shape[0])])
            return R.dequant_mxfp4(t.to(device), s.to(device))
        if t.dtype == torch.float8_e4m3fn and self.has(name + "_sf32"):        # Engram rows
            return R.dequant_fp8_rows32(t.to(device), self._tensor(name + "_sf32").to(device))
        if t.dtype == torch.float8_e4m3fn:
            s = self._tensor(name + "_scale_inv").float()
            if t.dim() == 3:
                return torch.stack([R.dequant_fp8_blocks(t[e].to(device), s[e].to(device)) for e in range(t.shape[0])])
            return R.dequant_fp8_blocks(t.to(device), s.to(device))
        return t.to(device=device, dtype=torch.float32)

"""Paged latent KV cache.

Per layer the cache holds, for every token slot, the latent row: ``[kv_lora | RoPE key]`` for MLA (the only
per-token state absorbed MLA needs; one row serves all heads) or the kv_lora_rank row itself for latent MQA and, when the model has a DSA indexer, the indexer key row.  Slots are
grouped into pages of ``page_size`` tokens; a request owns a list of pages (its page table) and token ``p`` of the
request lives in slot ``pages[p // page_size] * page_size + p % page_size``.

Reference: the engine's ``token_to_kv_pool`` with fp8 SWA / fp4 compressed / fp4 index-K pools
(``king_v10/bundle_v9/dec/index_reuse.py:10-17``, ``dec/cuda_decode_attn.py:41-43``).  Page allocation is done by
the native block allocator in ``carbon_b200.engine.allocator`` (C++).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from ..config import ModelConfig
from ..ops._ext import ext
from ..ref import ops as R
from .allocator import BlockAllocator


class PagedLatentCache:
    def __init__(self, cfg: ModelConfig, n_layers: int, num_pages: int, page_size: int, device, dtype):
        self.cfg = cfg
        self.page_size = page_size
        self.num_pages = num_pages
        self.num_slots = num_pages * page_size
        # fp8 rows (cfg.kv_fp8): uint8 [slots, row_bytes] in the format of ref.ops.quant_latent_fp8
        self.fp8 = cfg.kv_fp8
        width = self.row_bytes(cfg) if self.fp8 else cfg.latent_dim
        self.latent: List[torch.Tensor] = [torch.zeros(self.num_slots, width, device=device,
                                                       dtype=torch.uint8 if self.fp8 else dtype)
                                           for _ in range(n_layers)]
        # indexer keys only for layers that run the indexer (index-source layers share their selection)
        self.index_k: List[Optional[torch.Tensor]] = []
        if cfg.use_indexer:
            self.index_k = [torch.zeros(self.num_slots, cfg.index_head_dim, dtype=dtype, device=device)
                            if cfg.has_indexer(l) else None for l in range(n_layers)]
        # token id of every slot (Engram hashes each token's preceding n-gram; decode reads them through key slots)
        self.tok = torch.zeros(self.num_slots, dtype=torch.int32, device=device) if cfg.engram_layers else None
        self.alloc = BlockAllocator(num_pages)

    def write_tokens(self, loc: torch.Tensor, ids: torch.Tensor) -> None:
        self.tok.index_copy_(0, loc.long(), ids.to(torch.int32))

    @staticmethod
    def row_bytes(cfg: ModelConfig) -> int:
        """Bytes of one cached fp8 latent row (656 for the 512 + 64 MLA row, 528 for a 512-dim latent-MQA row)."""
        return R.latent_fp8_row_bytes(cfg.kv_lora_rank, cfg.qk_rope_head_dim, cfg.attn_kind == "mla")

    def write_latent(self, layer: int, loc: torch.Tensor, rows: torch.Tensor) -> None:
        if not self.fp8:
            self.latent[layer].index_copy_(0, loc.long(), rows.to(self.latent[layer].dtype))
        elif rows.is_cuda:
            ext().latent_store_fp8(rows.to(torch.bfloat16), loc.to(torch.int32).contiguous(), self.latent[layer])
        else:
            cfg = self.cfg
            q = R.quant_latent_fp8(rows, cfg.kv_lora_rank, cfg.qk_rope_head_dim, cfg.attn_kind == "mla")
            self.latent[layer].index_copy_(0, loc.long(), q)

    def write_index_k(self, layer: int, loc: torch.Tensor, rows: torch.Tensor) -> None:
        self.index_k[layer].index_copy_(0, loc.long(), rows.to(self.index_k[layer].dtype))

    def bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.latent + self.index_k if t is not None)

    @staticmethod
    def bytes_per_token(cfg: ModelConfig, n_layers: int, elem: int = 2) -> int:
        n_idx = sum(1 for l in range(n_layers) if cfg.has_indexer(l))
        lat = PagedLatentCache.row_bytes(cfg) if cfg.kv_fp8 else cfg.latent_dim * elem
        return lat * n_layers + cfg.index_head_dim * elem * n_idx

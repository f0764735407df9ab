"""Small, self-contained kernel cases for profiler captures (one launch of one kernel each, a few GB at most).

    python -m carbon_b200.profile_cases gemm|grouped|moe_decode|attn|decode|indexer

Each case sets up inputs larger than L2 where it can, runs its kernel twice (warm-up + the launch to capture) and
exits 0, so that ``ncu -k regex:<kernel> -s 1 -c 1`` captures exactly one warm launch.
"""
from __future__ import annotations

import sys

import torch


def gemm():
    from .ops.gemm import fp8_gemm
    from .ops.quant import quant_act, quantize_weight

    x = torch.randn(8192, 7168, device="cuda").to(torch.bfloat16)
    W = quantize_weight(torch.randn(8192, 7168, device="cuda") * 0.02)
    q, sf = quant_act(x)
    out = torch.empty(8192, 8192, dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        fp8_gemm(q, sf, W, out=out)


def grouped():
    from .models.deepseek import DeepseekModel
    from .config import ModelConfig
    from .models.weights import WeightSource
    from .ops import core as C

    cfg = ModelConfig(n_layers=1, n_dense_layers=0, vocab_size=1024, n_routed_experts=64, index_n_heads=0)
    m = DeepseekModel(cfg, WeightSource(cfg, seed=0), "cuda")
    h = torch.randn(4096, cfg.hidden_size, device="cuda").to(torch.bfloat16)
    w, ids = C.router_topk(torch.randn(4096, 64, device="cuda"), None, 8, "sigmoid", 2.5, True)
    m.pctx.set_bounds([0, 4096])
    for _ in range(2):
        m.moe_local(m.layers[0], h, w, ids, None)


def moe_decode():
    """Decode-sized MoE (32 tokens x top-8 over 64 experts): the grouped GEMMs stream expert weights."""
    from .config import ModelConfig
    from .models.deepseek import DeepseekModel
    from .models.weights import WeightSource
    from .ops import core as C

    cfg = ModelConfig(n_layers=1, n_dense_layers=0, vocab_size=1024, n_routed_experts=64, index_n_heads=0)
    m = DeepseekModel(cfg, WeightSource(cfg, seed=0), "cuda")
    h = torch.randn(32, cfg.hidden_size, device="cuda").to(torch.bfloat16)
    w, ids = C.router_topk(torch.randn(32, 64, device="cuda"), None, 8, "sigmoid", 2.5, True)
    m.pctx.set_bounds([0, 32])
    for _ in range(2):
        m.moe_local(m.layers[0], h, w, ids, None)


def attn():
    from .ops.attention import mla_prefill

    T, H = 8192, 16
    q = torch.randn(T, H, 192, device="cuda").to(torch.bfloat16)
    kvb = torch.randn(T, H, 256, device="cuda").to(torch.bfloat16)
    kpe = torch.randn(T, 64, device="cuda").to(torch.bfloat16)
    for _ in range(2):
        mla_prefill(q, kvb, kpe, [0, 4096, 8192], 192 ** -0.5)


def decode():
    from .ops.attention import sparse_mla

    T, K, S = 32, 2048, 32 * 4096
    q = torch.randn(T, 128, 576, device="cuda").to(torch.bfloat16)
    kv = torch.randn(S, 576, device="cuda").to(torch.bfloat16)
    idx = torch.stack([torch.randperm(4096, device="cuda")[:K] + b * 4096 for b in range(T)]).int()
    for _ in range(2):
        sparse_mla(q, kv, idx, 192 ** -0.5, 512)


def indexer():
    from .ops.attention import indexer_prefill_mask

    T = 8192
    q = torch.randn(T, 64, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, 128, device="cuda").to(torch.bfloat16)
    w = torch.randn(T, 64, device="cuda") * 0.01
    for _ in range(2):
        indexer_prefill_mask(q, k, w, [0, 4096, 8192], 2048)


if __name__ == "__main__":
    {"gemm": gemm, "grouped": grouped, "moe_decode": moe_decode, "attn": attn, "decode": decode,
     "indexer": indexer}[sys.argv[1]]()
    torch.cuda.synchronize()
    print("ok", sys.argv[1])

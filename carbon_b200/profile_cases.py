"""Small, self-contained kernel cases for profiler captures (one launch of one kernel each, a few GB at most).

    python -m carbon_b200.profile_cases gemm|grouped|moe_decode|attn|decode|decode_fp8|boundary|indexer|indexer_decode|ep_moe|oproj_a2a

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
    idx = torch.stack([torch.randperm(4096, device="cuda")[:K] + b * 4096 for b in range(T)]).int().sort(1).values
    for _ in range(2):
        sparse_mla(q, kv, idx, 192 ** -0.5, 512)


def decode_fp8():
    """The decode case over the fp8 cache format (656-byte rows; q in fp16)."""
    from .ops._ext import ext
    from .ops.attention import sparse_mla

    T, K, S = 32, 2048, 32 * 4096
    q = torch.randn(T, 128, 576, device="cuda").to(torch.float16)
    rows = torch.randn(S, 576, device="cuda").to(torch.bfloat16)
    kv = torch.empty(S, 656, dtype=torch.uint8, device="cuda")
    ext().latent_store_fp8(rows, torch.arange(S, dtype=torch.int32, device="cuda"), kv)
    idx = torch.stack([torch.randperm(4096, device="cuda")[:K] + b * 4096 for b in range(T)]).int().sort(1).values
    for _ in range(2):
        sparse_mla(q, kv, idx, 192 ** -0.5, 512)


def boundary():
    """Fused decode mHC boundary at the full width: 32 tokens x 4 streams x 7168, post-mix + stats + coefficients +
    pre-norm (two launches)."""
    from .models.deepseek import make_hc
    from .ops._ext import ext
    from .ops.quant import empty_sf

    T, D = 32, 7168
    dev = torch.device("cuda")
    hp = make_hc(torch.randn(24, 4 * D) * 0.02, torch.randn(24) * 0.5, torch.rand(3) + 0.5, dev)
    w = torch.rand(D, device=dev) + 0.5
    X = torch.randn(T, 4, D, device=dev).to(torch.bfloat16)
    out = torch.randn(T, D, device=dev).to(torch.bfloat16)
    post = torch.rand(T, 4, device=dev)
    comb = torch.softmax(torch.randn(T, 4, 4, device=dev), -1)
    y = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    q = torch.empty(T, D, dtype=torch.float8_e4m3fn, device=dev)
    sf = empty_sf(T, D, dev)
    p2, po2, c2 = torch.empty(T, 4, device=dev), torch.empty(T, 4, device=dev), torch.empty(T, 4, 4, device=dev)
    for _ in range(2):
        ext().mhc_boundary_small(X, out, post, comb, hp.fn, hp.base, hp.scale, 20, 1e-6, 1e-6, w, y, q, sf, p2, po2, c2)


def indexer():
    from .ops.attention import indexer_prefill_mask

    T = 8192
    q = torch.randn(T, 64, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, 128, device="cuda").to(torch.bfloat16)
    w = torch.randn(T, 64, device="cuda") * 0.01
    for _ in range(2):
        indexer_prefill_mask(q, k, w, [0, 4096, 8192], 2048)


def indexer_decode():
    """Decode DSA indexer logits: 32 tokens x 4097 paged keys (64-token pages) x 64 heads (tcgen05 kernel)."""
    from .ops._ext import ext

    T, L, H, page = 32, 4097, 64, 64
    S = T * (L // page + 2) * page
    q = torch.randn(T, H, 128, device="cuda").to(torch.bfloat16)
    w = torch.randn(T, H, device="cuda") * 0.01
    kc = torch.randn(S, 128, device="cuda").to(torch.bfloat16)
    pages = torch.randperm(S // page, device="cuda")[: T * (L // page + 1)].view(T, -1)
    pos = torch.arange(L, device="cuda")
    slots = (pages[:, pos // page] * page + pos % page).int().contiguous()
    n = torch.full((T,), L, dtype=torch.int32, device="cuda")
    out = torch.empty(T, L, device="cuda")
    for _ in range(2):
        ext().indexer_decode_logits(q, w, kc, slots, n, out)


def _fused_one_rank():
    """A one-rank FusedCtx (every peer pointer is this GPU's own heap): the fused collective kernels run alone."""
    import os

    import torch.distributed as dist

    from .parallel.fused import FusedCtx

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    if not dist.is_initialized():
        dist.init_process_group("gloo", rank=0, world_size=1)
    return FusedCtx(0, 1, heap_bytes=4 << 30, max_tokens=8192, max_seq=4096)


def ep_moe():
    """EP MoE layer through the fused path on one rank, 8192 tokens x top-8 of 64 experts (hidden 7168): count,
    dispatch (quantise + row stores), grouped GEMMs with the push-combine epilogue, local combine (two pipelined
    chunks of 4096 tokens)."""
    from .config import ModelConfig
    from .models.deepseek import DeepseekModel
    from .models.weights import WeightSource
    from .ops import core as C

    f = _fused_one_rank()
    cfg = ModelConfig(n_layers=1, n_dense_layers=0, vocab_size=1024, n_routed_experts=64, index_n_heads=0)
    m = DeepseekModel(cfg, WeightSource(cfg, seed=0), "cuda", pctx=f)
    T = 8192
    h = torch.randn(T, cfg.hidden_size, device="cuda").to(torch.bfloat16)
    w, ids = C.router_topk(torch.randn(T, 64, device="cuda"), None, 8, "sigmoid", 2.5, True)
    f.set_bounds([0, T])
    for _ in range(2):
        f.moe(m, m.layers[0], h, w, ids, None)


def oproj_a2a():
    """Head -> token all-to-all of 8192 tokens x 128 heads x 128 dims (bf16) on one rank (p2p_a2a_heads)."""
    f = _fused_one_rank()
    T = 8192
    f.set_bounds([0, T])
    o = torch.randn(T, 128, 128, device="cuda").to(torch.bfloat16)
    for _ in range(2):
        f.heads_to_tokens(o)


if __name__ == "__main__":
    {"gemm": gemm, "grouped": grouped, "moe_decode": moe_decode, "attn": attn, "decode": decode,
     "decode_fp8": decode_fp8, "boundary": boundary,
     "indexer": indexer, "indexer_decode": indexer_decode, "ep_moe": ep_moe, "oproj_a2a": oproj_a2a}[sys.argv[1]]()
    torch.cuda.synchronize()
    print("ok", sys.argv[1])

"""Op-level benchmarks (attention, mHC + GEMM, decode mHC boundary, MoE, GEMM, decode attention and indexer), timed
on the device with CUDA events and reported against the measured roofline (``MEASURED_PEAKS.json`` when present: ``bf16_tflops``, ``hbm_gbs``).

    python -m carbon_b200.benchmarks attn  [--batch 4 --seq 8192 --heads 128 --dsa]   # config 2
    python -m carbon_b200.benchmarks mhc   [--tokens 16384 --hidden 7168 --n 24576]   # config 3
    python -m carbon_b200.benchmarks gemm  [--m 16384 --n 24576 --k 7168]             # fp8 block-scaled GEMM
    python -m carbon_b200.benchmarks moe   [--tokens 4096 --experts 256 --topk 8]     # config 4, one GPU
    python -m carbon_b200.benchmarks decode_attn [--batch 32 --topk 2048]
    python -m carbon_b200.benchmarks decode_indexer [--batch 32 --context 4096 --topk 2048]

Each prints one JSON line.  Inputs are larger than L2 where the config allows; between timed iterations a 256 MB
buffer is rewritten to flush L2 (``flush_l2``) for the ones that are not.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"bf16_tflops": d.get("bf16_tflops", 1590.0), "hbm_gbs": d.get("hbm_gbs", 6650.0), "src": "measured"}
    return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "src": "fallback"}


_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def time_fn(fn, iters=10, warmup=3, flush=True):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if flush:
            flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


def bench_attn(a):
    from .ops.attention import indexer_prefill_mask, mla_prefill

    torch.manual_seed(0)
    B, S, H = a.batch, a.seq, a.heads
    T = B * S
    q = torch.randn(T, H, 192, device="cuda", dtype=torch.bfloat16)
    kvb = torch.randn(T, H, 256, device="cuda", dtype=torch.bfloat16)   # (k_nope | v) as the wkv_b GEMM writes it
    kpe = torch.randn(T, 64, device="cuda", dtype=torch.bfloat16)       # shared RoPE key
    cu = [i * S for i in range(B + 1)]
    mask = None
    res = {}
    if a.dsa:
        qi = torch.randn(T, 64, 128, device="cuda").to(torch.float8_e4m3fn).to(torch.bfloat16)
        ki = torch.randn(T, 128, device="cuda").to(torch.float8_e4m3fn).to(torch.bfloat16)
        wi = torch.randn(T, 64, device="cuda") * (64 ** -0.5) * (128 ** -0.5)
        # fp8 e4m3 inputs (the config's indexer precision): block-scaled fp8 logits; bf16 kernel for comparison
        fp8 = not a.indexer_bf16
        ms = time_fn(lambda: indexer_prefill_mask(qi, ki, wi, cu, a.topk, fp8=fp8), iters=5)
        mask = indexer_prefill_mask(qi, ki, wi, cu, a.topk, fp8=fp8)
        idx_flops = B * (S * S / 2) * 64 * 128 * 2
        res["indexer_ms"] = round(ms, 3)
        res["indexer_tflops"] = round(idx_flops / ms / 1e9, 1)
        res["indexer_inputs"] = "fp8 e4m3" if fp8 else "bf16"
    ms = time_fn(lambda: mla_prefill(q, kvb, kpe, cu, 192 ** -0.5, mask, version=a.attn_version), iters=5)
    flops = B * H * (S * S / 2) * (192 + 128) * 2
    pk = peaks()
    res.update({"bench": "mla_prefill_attention", "kernel_version": a.attn_version or (3 if a.dsa else 2), "batch": B, "seq": S, "heads": H, "dsa": a.dsa, "ms": round(ms, 3),
                "tflops": round(flops / ms / 1e9, 1),
                "frac_of_bf16_peak": round(flops / ms / 1e9 / pk["bf16_tflops"], 3), "peak_src": pk["src"],
                "flops_counted": "dense causal (masked DSA keys still cost a full tile)"})
    print(json.dumps(res))


def bench_gemm(a):
    from .ops.gemm import fp8_gemm
    from .ops.quant import quant_act, quantize_weight

    x = torch.randn(a.m, a.k, device="cuda").to(torch.bfloat16)
    W = quantize_weight(torch.randn(a.n, a.k, device="cuda") * 0.02)
    q, sf = quant_act(x)
    out = torch.empty(a.m, a.n, dtype=torch.bfloat16, device="cuda")
    ms = time_fn(lambda: fp8_gemm(q, sf, W, out=out, pair=a.pair))
    flops = 2 * a.m * a.n * a.k
    pk = peaks()
    print(json.dumps({"bench": "fp8_gemm", "m": a.m, "n": a.n, "k": a.k, "pair": a.pair, "ms": round(ms, 3),
                      "tflops": round(flops / ms / 1e9, 1),
                      "frac_of_bf16_peak_x2": round(flops / ms / 1e9 / (2 * pk["bf16_tflops"]), 3),
                      "peak_src": pk["src"]}))


def bench_mhc(a):
    """Config 3: mHC stream mix (Sinkhorn-projected comb) + RMSNorm + fp8 quant feeding a 7168->24576 fp8 GEMM."""
    from .ops._ext import ext
    from .ops.gemm import fp8_gemm
    from .ops.quant import empty_sf, quantize_weight
    from .ref import ops as R

    T, D, N = a.tokens, a.hidden, a.n
    X = torch.randn(T, 4, D, device="cuda").to(torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    comb = R.sinkhorn(torch.randn(4, 4, generator=g), 20, 1e-6)
    pre = comb.sum(0) / 4                              # stream weights of the mixed read (column means)
    pre_t = pre.to("cuda").expand(T, 4).contiguous()
    w_norm = torch.ones(D, device="cuda")
    W = quantize_weight(torch.randn(N, D, device="cuda") * 0.02)
    y = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(T, D, dtype=torch.float8_e4m3fn, device="cuda")
    sf = empty_sf(T, D, "cuda")
    out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")

    def step():
        ext().mhc_pre_norm(X, pre_t, w_norm, 1e-6, None, q, sf, None)
        fp8_gemm(q, sf, W, out=out)

    ms = time_fn(step, flush=False)
    ms_mix = time_fn(lambda: ext().mhc_pre_norm(X, pre_t, w_norm, 1e-6, None, q, sf, None), flush=False)
    flops = 2 * T * N * D
    bytes_mix = T * 4 * D * 2 + T * D
    pk = peaks()
    print(json.dumps({"bench": "mhc_mix_norm_fp8_gemm", "tokens": T, "hidden": D, "n": N, "ms": round(ms, 3),
                      "mix_norm_quant_ms": round(ms_mix, 3),
                      "mix_gbs": round(bytes_mix / ms_mix / 1e6, 1),
                      "mix_frac_of_hbm": round(bytes_mix / ms_mix / 1e6 / pk["hbm_gbs"], 3),
                      "gemm_tflops": round(flops / (ms - ms_mix) / 1e9, 1), "peak_src": pk["src"]}))


def bench_boundary(a):
    """Fused decode mHC boundary (post-mix + statistics + Sinkhorn coefficients + pre-norm, one launch) at the full
    width: --decode-tokens tokens x 4 streams x --hidden; cold L2 (flushed) and warm."""
    from .models.deepseek import make_hc
    from .ops._ext import ext
    from .ops.quant import empty_sf

    T, D, dev = a.decode_tokens, a.hidden, torch.device("cuda")
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

    def step():
        ext().mhc_boundary_small(X, out, post, comb, hp.fn, hp.base, hp.scale, 20, 1e-6, 1e-6, w, y, q, sf, p2, po2,
                                 c2)

    cold = time_fn(step, iters=20, flush=True)
    warm = time_fn(step, iters=20, flush=False)
    print(json.dumps({"bench": "mhc_boundary_decode", "tokens": T, "hidden": D, "us_cold_l2": round(cold * 1e3, 2),
                      "us_warm_l2": round(warm * 1e3, 2)}))


def bench_decode_attn(a):
    from .ops.attention import sparse_mla

    T, H, K, S = a.batch, a.heads, a.topk, a.batch * a.context
    q = torch.randn(T, H, 576, device="cuda").to(torch.bfloat16)
    kv = torch.randn(S, 576, device="cuda").to(torch.bfloat16)
    row = 576 * 2
    if a.kv == "fp8":                  # the fp8 cache format (656 bytes per row); the kernel takes q in fp16
        from .ops._ext import ext

        kv8 = torch.empty(S, 656, dtype=torch.uint8, device="cuda")
        ext().latent_store_fp8(kv, torch.arange(S, dtype=torch.int32, device="cuda"), kv8)
        kv, q, row = kv8, q.half(), 656
    idx = torch.stack([torch.randperm(a.context, device="cuda")[:K] + b * a.context for b in range(T)]).int()
    if not a.unsorted:
        idx = idx.sort(dim=1).values      # the DSA top-k hands keys over in key order (page order in the cache)
    ms = time_fn(lambda: sparse_mla(q, kv, idx, 192 ** -0.5, 512))
    bytes_kv = T * K * row
    pk = peaks()
    print(json.dumps({"bench": "sparse_mla_decode", "kv": a.kv, "key_order": "random" if a.unsorted else "sorted",
                      "batch": T, "heads": H, "topk": K, "ms": round(ms, 4),
                      "kv_gbs": round(bytes_kv / ms / 1e6, 1),
                      "frac_of_hbm": round(bytes_kv / ms / 1e6 / pk["hbm_gbs"], 3),
                      "tflops": round(T * H * K * (576 + 512) * 2 / ms / 1e9, 1), "peak_src": pk["src"]}))


def bench_decode_indexer(a):
    """Decode DSA indexer: logits of `batch` tokens over `context` paged keys each (64-token pages), then top-k."""
    from .ops._ext import ext

    T, L, H, k = a.batch, a.context + 1, 64, a.topk
    page = 64
    S = T * (L // page + 2) * page
    q = torch.randn(T, H, 128, device="cuda").to(torch.bfloat16)
    w = torch.randn(T, H, device="cuda") * 0.01
    kc = torch.randn(S, 128, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(S // page, device="cuda")
    pages = perm[: T * (L // page + 1)].view(T, -1)
    pos = torch.arange(L, device="cuda")
    slots = (pages[:, pos // page] * page + pos % page).int().contiguous()
    n = torch.full((T,), L, dtype=torch.int32, device="cuda")
    logits = torch.empty(T, L, device="cuda")
    out = torch.empty(T, k, dtype=torch.int32, device="cuda")
    e = ext()
    ms_logits = time_fn(lambda: e.indexer_decode_logits(q, w, kc, slots, n, logits))
    ms_all = time_fn(lambda: e.indexer_topk(q, w, kc, slots, n, out))
    bytes_k = T * L * 128 * 2
    pk = peaks()
    print(json.dumps({"bench": "indexer_decode", "batch": T, "keys": L, "heads": H, "topk": k,
                      "logits_us": round(ms_logits * 1e3, 2), "logits_plus_topk_us": round(ms_all * 1e3, 2),
                      "logits_frac_of_hbm": round(bytes_k / ms_logits / 1e6 / pk["hbm_gbs"], 3),
                      "peak_src": pk["src"]}))


def bench_moe(a):
    """Config 4 MoE layer (router top-k + routed experts + shared expert) on one GPU, or EP over all ranks of a
    torchrun job (``--comm fused|nccl``): 256 experts top-8 + 1 shared, hidden 7168, intermediate 2048, fp8
    block-scaled weights ~N(0, 0.02); router logits ~N(0,1) + per-expert bias ~N(0, 0.5) (Zipf-like skew)."""
    import torch.distributed as dist

    from .config import ModelConfig
    from .models.deepseek import DeepseekModel
    from .models.weights import WeightSource
    from .parallel.context import ParallelCtx

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    cfg = ModelConfig(n_layers=1, n_dense_layers=0, vocab_size=1024, n_routed_experts=a.experts,
                      n_activated_experts=a.moe_topk, hidden_size=a.hidden, moe_intermediate=a.inter, index_n_heads=0)
    if world == 1:
        pctx = ParallelCtx.single()
    elif a.comm == "nccl":
        from .parallel.dist import DistCtx

        pctx = DistCtx(rank, world)
    else:
        from .parallel.fused import FusedCtx

        pctx = FusedCtx(rank, world, heap_bytes=12 << 30, max_tokens=a.tokens * world, max_seq=a.tokens)
    model = DeepseekModel(cfg, WeightSource(cfg, seed=0), "cuda", pctx=pctx)
    L = model.layers[0]
    T = a.tokens
    g = torch.Generator(device="cuda").manual_seed(rank)
    h = torch.randn(T, a.hidden, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(a.experts, device="cuda", generator=torch.Generator(device="cuda").manual_seed(0)) * 0.5
    logits = torch.randn(T, a.experts, device="cuda", generator=g)
    from .ops import core as C

    w, ids = C.router_topk(logits, bias, a.moe_topk, "sigmoid", 2.5, True)
    pctx.set_bounds([i * T for i in range(world + 1)])
    shared = L.shared(h)

    def step():
        return pctx.moe(model, L, h, w, ids, shared)

    ms = time_fn(step, iters=5, flush=False)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = 2 * T * a.moe_topk * 3 * a.hidden * a.inter      # routed experts (per rank's tokens)
    bytes_nvlink = T * a.moe_topk * a.hidden * (1 + 2) * (world - 1) / max(world, 1)   # fp8 dispatch + bf16 combine
    pk = peaks()
    if rank == 0:
        print(json.dumps({"bench": "moe_layer", "world": world, "comm": a.comm if world > 1 else "local",
                          "tokens_per_rank": T, "experts": a.experts, "topk": a.moe_topk, "ms": round(ms, 3),
                          "routed_tflops_per_gpu": round(flops / ms / 1e9, 1),
                          "frac_of_fp8_peak(2x bf16 measured)": round(flops / ms / 1e9 / (2 * pk["bf16_tflops"]), 3),
                          "nvlink_bytes_per_rank": int(bytes_nvlink), "peak_src": pk["src"]}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["attn", "gemm", "mhc", "boundary", "decode_attn", "decode_indexer", "moe"])
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--heads", type=int, default=128)
    ap.add_argument("--dsa", action="store_true")
    ap.add_argument("--kv", default="bf16", choices=["bf16", "fp8"], help="decode_attn: latent cache format")
    ap.add_argument("--unsorted", action="store_true",
                    help="decode_attn: selected keys in random order (the engine passes them in key order)")
    ap.add_argument("--indexer-bf16", action="store_true", help="attn --dsa: bf16 indexer logits instead of fp8")
    ap.add_argument("--topk", type=int, default=2048, help="DSA top-k")
    ap.add_argument("--moe-topk", type=int, default=8, help="router top-k (moe)")
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=24576)
    ap.add_argument("--k", type=int, default=7168)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--decode-tokens", type=int, default=32, help="boundary: decode batch")
    ap.add_argument("--attn-version", type=int, default=0,
                    help="attn: 3 = two Q tiles, 64-key steps, double-buffered S; 2 = two Q tiles, 128-key steps; 1 = one")
    ap.add_argument("--pair", type=int, default=-1, help="gemm: -1 auto, 1 CTA-pair 256x256 tiles, 0 128x128 tiles")
    a = ap.parse_args(argv)
    sys.path.insert(0, ROOT)
    {"attn": bench_attn, "gemm": bench_gemm, "mhc": bench_mhc, "boundary": bench_boundary,
     "decode_attn": bench_decode_attn,
     "decode_indexer": bench_decode_indexer, "moe": bench_moe}[a.what](a)


if __name__ == "__main__":
    main()

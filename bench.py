"""Serving benchmark on the full-size DeepSeek-V3/V4-class model (fp8 block-scaled, random init).

    python bench.py --gpus N --steps K --warmup W            # our engine (default N=1)
    python bench.py --impl reference ...                     # the reference's own build (see --impl reference)

Per GPU (weak scaling; 8 GPUs = the headline configuration): prefill 4 prompts × 4096 uniform-random token ids per step,
decode a batch of 32 requests at context 4096 per step (global 32 prompts / batch 256 at N=8).  Timing: W untimed
warm-up steps, then K steps bracketed by barrier + synchronize, CUDA events on the launching stream, max over
ranks.  The weights (>100 GB) are far larger than L2, so every step streams them from HBM (no L2 flush needed).

Rank 0 prints one JSON line; `value` is whole-job prefill tokens/s, decode output tokens/s and p50 TPOT are
extra keys.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "prefill tok/s & decode out tok/s (8×B200, max over ranks); p50 TPOT; roofline %"
BASELINE_VALUE = None  # the reference publishes no end-to-end number for this metric


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="deepseek_v3")
    ap.add_argument("--prompts-per-gpu", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=4096)
    ap.add_argument("--decode-batch-per-gpu", type=int, default=32)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--decode-steps", type=int, default=16)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (0 = config's)")
    ap.add_argument("--mem-frac", type=float, default=0.62, help="HBM fraction for weights (rest: cache, acts)")
    ap.add_argument("--profile", action="store_true", help="print per-region device times (stderr)")
    ap.add_argument("--kernel-table", action="store_true",
                    help="print the device time per kernel of one graph-replayed decode step (CUPTI activity records "
                         "through torch.profiler; for analysis, never a bench value)")
    ap.add_argument("--trace-dir", default=None,
                    help="with --profile: write Chrome trace files of the traced decode and prefill steps here "
                         "(one per rank)")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                    help="multi-GPU data movement: our NVLink kernels (fused) or the NCCL baseline")
    ap.add_argument("--oproj", default="a2a", choices=["a2a", "rs"],
                    help="TP attention output: heads -> tokens all-to-all + whole projection on the token's owner "
                         "(a2a) or row-parallel projection + reduce-scatter (rs)")
    ap.add_argument("--replicated-kv", action="store_true",
                    help="N>1: every rank caches every request's KV (default: only each request's home rank does)")
    ap.add_argument("--decode-cache", default="random", choices=["random", "zeros"],
                    help="content of the decode requests' cached context rows: random latent rows and indexer keys "
                         "(DSA selects real, scattered keys) or the zero rows of a fresh cache")
    ap.add_argument("--kv", default="fp8", choices=["fp8", "bf16"],
                    help="latent KV cache format (fp8: 656 bytes per token and layer, bf16: 1152)")
    ap.add_argument("--attn", default="tp", choices=["tp", "dp"],
                    help="attention parallelism for N>1: tensor-parallel over heads (the headline configuration) or "
                         "data-parallel over each rank's own sequences")
    return ap.parse_args()


# ----------------------------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                f = [x.strip() for x in out.stdout.strip().split(",")]
                if len(f) >= 9:
                    self.samples.append(f)
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for s in self.samples for j in range(4) if "Active" in s[5 + j]
                          and "Not" not in s[5 + j]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------------------------------------
def reference_arm(args):
    """The reference is a set of slot bundles for a sealed SGLang-fork engine (sglang, deep_gemm 0.2.3, FlashMLA,
    torch 2.14+cu130) gated to sm_103; it has no installable package and cannot run offline here."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    why = ("pip install of the reference failed: 'not installable, neither setup.py nor pyproject.toml found'; it is "
           "slot bundles for a sealed SGLang-fork engine (needs sglang, deep_gemm 0.2.3.post2, FlashMLA; levers "
           "gated to sm_103), none of which is in the image")
    if os.path.isdir(ref_dir) and os.listdir(ref_dir):
        why = "baseline/_ref holds no importable engine: " + why
    line = {"impl": "reference", "unavailable": why}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)


def pick_layer_sets(cfg, ep: int, mem_bytes: float, frac: float) -> int:
    """Number of distinct MoE-layer weight sets that fit `frac` of HBM (the rest of the layers reuse them)."""
    D, E, I = cfg.hidden_size, cfg.n_routed_experts, cfg.moe_intermediate
    per_moe = (E // ep) * 3 * D * I + 3 * D * I * cfg.n_shared_experts + 300e6
    dense = cfg.n_dense_layers * (3 * D * cfg.dense_intermediate + 300e6)
    emb = 2 * cfg.vocab_size * D * 2
    budget = mem_bytes * frac - dense - emb
    n_moe = cfg.n_layers - cfg.n_dense_layers
    return max(1, min(n_moe, int(budget // per_moe)))


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import torch.distributed as dist

    from carbon_b200.config import PRESETS
    from carbon_b200.engine.engine import Engine
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.ops._ext import ext
    from carbon_b200.parallel.context import ParallelCtx

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    ext()
    cfg = PRESETS[args.config]().replace(kv_fp8=args.kv == "fp8")
    if args.layers:
        cfg = cfg.replace(n_layers=args.layers)
    P, S = args.prompts_per_gpu, args.prompt_len
    B, ctx = args.decode_batch_per_gpu, args.context
    if world == 1:
        pctx = ParallelCtx.single()
    elif args.comm == "nccl":
        from carbon_b200.parallel.dist import DistCtx

        pctx = DistCtx(rank, world, attn_dp=args.attn == "dp")
    else:
        from carbon_b200.parallel.fused import FusedCtx

        max_tokens = max(P * S, B) * world
        a2a = args.oproj == "a2a" and args.attn == "tp"
        pctx = FusedCtx(rank, world, heap_bytes=heap_bytes(cfg, world, max_tokens, S, a2a), max_tokens=max_tokens,
                        max_seq=S, attn_dp=args.attn == "dp", oproj_a2a=a2a)
    mem = torch.cuda.get_device_properties(dev).total_memory
    page = 64
    # owner-only KV (N > 1): a rank holds pages only for the requests whose home it is (B per GPU at decode, about
    # P per GPU at prefill); replicated KV holds every request's pages on every rank
    owner_kv = world > 1 and not args.replicated_kv
    kv_ranks = 1 if owner_kv else world
    dec_pages = (B * kv_ranks) * ((ctx + args.decode_steps * (args.warmup + args.steps) * 2 + 2 * page) // page + 1)
    pf_pages = (P * kv_ranks + (P if owner_kv else 0)) * (S // page + 2)     # owner: room for an uneven plan
    num_pages = max(dec_pages, pf_pages) + 8
    from carbon_b200.engine.kv_cache import PagedLatentCache

    cache_b = num_pages * page * PagedLatentCache.bytes_per_token(cfg, cfg.n_layers)
    heap_b = getattr(getattr(pctx, "heap", None), "nbytes", 0)
    weight_budget = 0.90 * mem - cache_b - heap_b - (14 << 30)
    sets = pick_layer_sets(cfg, pctx.ep, weight_budget / args.mem_frac, args.mem_frac)
    n_moe = cfg.n_layers - cfg.n_dense_layers
    tied = sets < n_moe
    src = WeightSource(cfg, seed=0, layer_sets=sets if tied else None)
    t0 = time.time()
    P, S = P * world, S                      # weak scaling: global prompts / decode batch grow with N
    B = B * world
    pages_needed = num_pages
    graphs = world == 1 or args.comm == "fused"
    # decode graphs: one bucket of the per-rank block (owner-only KV pads each home rank's rows to a fixed block) or
    # of the whole batch
    eng = Engine(cfg, device=dev, source=src, num_pages=pages_needed, page_size=page, cuda_graphs=graphs,
                 graph_buckets=(B // world if owner_kv else B,), pctx=pctx, owner_kv=owner_kv)
    torch.cuda.synchronize()
    init_s = time.time() - t0
    gen = torch.Generator().manual_seed(1234)     # SPMD: every rank builds the same requests
    t_start = time.time()

    def phase(name):                      # progress on stderr: a stalled run shows where it stopped
        if rank == 0:
            mem = torch.cuda.max_memory_allocated(dev) / 2 ** 30
            print(f"[bench] {time.time() - t_start:8.1f}s {name} (peak {mem:.1f} GiB allocated)", file=sys.stderr,
                  flush=True)

    phase(f"engine ready (init {init_s:.1f}s)")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        code = pctx.check() if hasattr(pctx, "check") else 0
        if world > 1:                     # every rank learns of any rank's error, so all raise together
            t = torch.tensor([code], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            code = int(t.item())
        if code:
            raise RuntimeError(f"rank {rank}: device collective error code {code} (peer wait timed out or buffer "
                               "capacity exceeded)")

    # ---------------- prefill (device-timed) ----------------
    def prefill_step():
        reqs = [eng.add_request(torch.randint(0, cfg.vocab_size, (S,), generator=gen).tolist()) for _ in range(P)]
        logits = eng.prefill(reqs)
        for r in reqs:
            eng.release(r)
        return logits

    for w_ in range(args.warmup):
        prefill_step()
        phase(f"prefill warm-up {w_ + 1}/{args.warmup}")
    barrier()
    phase("prefill timed")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with ClockSampler(local) as clk:
        ev[0].record()
        for _ in range(args.steps):
            prefill_step()
        ev[1].record()
        barrier()
    pf_ms = ev[0].elapsed_time(ev[1]) / args.steps
    pf_ms = max_over_ranks(pf_ms, world)

    # ---------------- prefill end to end through the public API (H2D ids from pinned host, D2H next tokens) ------
    phase("prefill end-to-end")
    host_ids = [torch.randint(0, cfg.vocab_size, (S,), generator=gen).pin_memory() for _ in range(P)]
    barrier()
    ee = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ee[0].record()
    d2h = 0
    for _ in range(args.steps):
        reqs = [eng.add_request(h.tolist()) for h in host_ids]
        nxt = torch.argmax(eng.prefill(reqs), dim=-1).cpu()
        d2h += nxt.numel() * nxt.element_size()
        for r in reqs:
            eng.release(r)
    ee[1].record()
    barrier()
    e2e_ms = max_over_ranks(ee[0].elapsed_time(ee[1]) / args.steps, world)

    # ---------------- decode (CUDA graphs, context `ctx`) ----------------
    reqs = []
    for j in range(B):
        r = eng.add_request(torch.randint(0, cfg.vocab_size, (ctx,), generator=gen).tolist())
        if owner_kv:
            r.home = j // (B // world)          # B / N requests per home rank
        eng._ensure_pages(r, r.seq_len)
        r.n_cached = ctx          # the context rows are synthetic (not computed by a prefill)
        reqs.append(r)
    if args.decode_cache == "random":
        fill_cache_rows(eng, reqs, ctx, gen)
    # every decode step feeds fresh uniform-random token ids (synthetic data): routing stays as diverse as a real
    # batch's, so each step streams the weights of every expert its tokens select
    def next_ids():
        return torch.randint(0, cfg.vocab_size, (B,), generator=gen).tolist()

    phase("decode warm-up (graph capture)")
    for _ in range(args.warmup):
        for _ in range(2):
            eng.decode(reqs, next_ids())
    barrier()
    phase("decode timed")
    step_ms = []
    for _ in range(args.steps):
        for _ in range(args.decode_steps):
            nxt = next_ids()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            eng.decode(reqs, nxt)
            b.record()
            step_ms.append((a, b))
    barrier()
    tp = [a.elapsed_time(b) for a, b in step_ms]
    dec_ms = max_over_ranks(sum(tp) / len(tp), world)
    tpot_p50 = max_over_ranks(statistics.median(tp), world)

    tables = []
    if args.kernel_table:                  # every rank replays the same step (it contains collectives)
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            eng.decode(reqs, next_ids())
            torch.cuda.synchronize()
        agg = {}
        for ev in prof.events():
            if ev.device_type.name == "CUDA":
                k = ev.name.split("(")[0][:70]
                n, us = agg.get(k, (0, 0.0))
                agg[k] = (n + 1, us + ev.device_time)
        total = sum(us for _, us in agg.values())
        rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
        tables.append("== decode step, device time per kernel (graph replay) ==\n" + "\n".join(
            f"{us:10.1f} us {n:5d}  {100 * us / max(total, 1e-9):5.1f}%  {k}" for k, (n, us) in rows[:40]) +
            f"\n{total:10.1f} us total")
    if args.profile:                       # every rank runs the traced steps (they contain collectives)
        from carbon_b200.utils.trace import tracing

        eng.cuda_graphs = False
        with tracing() as t:
            eng.decode(reqs, next_ids())
        eng.cuda_graphs = graphs
        tables.append("== decode regions (eager) ==\n" + t.table())
        if args.trace_dir:
            os.makedirs(args.trace_dir, exist_ok=True)
            t.chrome_trace(os.path.join(args.trace_dir, f"decode_rank{rank}.json"), pid=rank)
    for r in reqs:
        eng.release(r)
    launches = count_launches(eng, P, S)
    if args.profile:
        with tracing() as t:
            prefill_step()
        tables.append("== prefill regions ==\n" + t.table())
        if args.trace_dir:
            t.chrome_trace(os.path.join(args.trace_dir, f"prefill_rank{rank}.json"), pid=rank)
    if tables and rank == 0:
        print("\n".join(tables), file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier()
    if rank == 0:
        pf_tok_s = P * S / (pf_ms / 1e3)
        line = {
            "metric": METRIC, "value": round(pf_tok_s, 1), "unit": "tokens/s (prefill, whole job)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(pf_ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp8 weights+GEMM inputs, "
            "bf16 activations", "data": "synthetic uniform-random token ids; random-init weights (N(0,0.02))",
            "decode_out_tok_s": round(B / (dec_ms / 1e3), 1), "tpot_p50_ms": round(tpot_p50, 3),
            "decode_ms_per_step": round(dec_ms, 3),
            "e2e": {"value": round(P * S / (e2e_ms / 1e3), 1), "unit": "tokens/s (prefill via Engine.prefill)",
                    "h2d_bytes_per_step": P * S * 4, "d2h_bytes_per_step": d2h // max(args.steps, 1)},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "roofline": roofline(cfg, world, args.prompts_per_gpu, S, args.decode_batch_per_gpu, ctx, pf_ms, dec_ms,
                                 load_peaks()),
            "config": {"model": f"{args.config} ({cfg.n_layers} layers, hidden {cfg.hidden_size}, "
                                f"{cfg.n_routed_experts} experts top-{cfg.n_activated_experts})",
                       "global_batch": P, "seq_len": S, "decode_batch": B, "context": ctx,
                       "parallelism": pctx_name(pctx, world, owner_kv),
                       "weights": (f"{sets} distinct MoE-layer weight sets cycled over {n_moe} MoE layers "
                                   "(every layer still runs; the full untied model needs 8 GPUs)") if tied
                       else "all layers distinct", "l2": "inputs (weights) larger than L2",
                       "decode_cache": args.decode_cache + " context rows",
                       "kv_cache": "fp8 e4m3 latent rows, UE8M0 per 64 dims + fp16 RoPE key (656 B/token/layer)"
                       if cfg.kv_fp8 else "bf16 latent rows (1152 B/token/layer)",
                       "init_s": round(init_s, 1)},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def fill_cache_rows(eng, reqs, ctx, gen):
    """Random context rows for the decode requests this rank holds: latent rows ~N(0, 1) (the scale of RMSNorm'd
    latents) and indexer keys, written through the cache's own store path, so the DSA indexer selects real, scattered
    keys and the attention gathers them.  One block of rows is generated and written into every layer."""
    from carbon_b200.engine.pd import request_slots

    cache, cfg = eng.cache, eng.cfg
    mine = [r for r in reqs if not eng.owner_kv or r.home == eng.model.pctx.rank]
    if not mine:
        return
    g = torch.Generator(device=eng.device).manual_seed(int(torch.randint(0, 1 << 30, (1,), generator=gen)))
    for r in mine:
        slots = request_slots(eng, r, ctx).to(torch.int32)
        rows = torch.randn(ctx, cfg.latent_dim, generator=g, device=eng.device).to(torch.bfloat16)
        keys = torch.randn(ctx, cfg.index_head_dim, generator=g, device=eng.device).to(torch.bfloat16)
        for layer in range(cfg.n_layers):
            cache.write_latent(layer, slots, rows)
            if cache.index_k and cache.index_k[layer] is not None:
                cache.write_index_k(layer, slots, keys)
    if eng.device.type == "cuda":
        torch.cuda.synchronize()


def pctx_name(p, world, owner_kv=False):
    if world == 1:
        return "single GPU"
    kind = "NVLink peer-memory kernels" if type(p).__name__ == "FusedCtx" else "NCCL baseline"
    if getattr(p, "attn_dp", False):
        attn = f"dp{world} attention"
    else:
        attn = f"tp{p.tp} attention" + (" (output projection after a heads->tokens all-to-all)"
                                         if getattr(p, "oproj_a2a", False) else "")
    kv = "KV on each request's home rank" if owner_kv else "KV replicated on every rank"
    return f"{attn} + ep{p.ep} MoE, sequence-sharded residual, {kv} ({kind})"


def heap_bytes(cfg, world, max_tokens, max_seq, oproj_a2a=True):
    """Symmetric-heap size: reduce-scatter slots (or heads -> tokens buffers), MoE receive/output rows, gathers,
    vocab shard, slack."""
    D = cfg.hidden_size
    max_local = min(max_tokens, (max_tokens + world - 1) // world + max_seq)
    pow2 = 1 << max(4, (max_local - 1).bit_length())          # gather slots grow in powers of two rows
    if oproj_a2a:
        rs = 2 * pow2 * cfg.n_heads * cfg.head_out_dim * 2    # double-buffered per-head outputs of this rank's tokens
    else:
        rs = 2 * world * max_local * D * 2
    cap = int(max_local * cfg.n_activated_experts * 1.6) + (cfg.n_routed_experts // world) * 256 + 256
    cap2 = int((max_local + 1) // 2 * cfg.n_activated_experts * 1.6) + (cfg.n_routed_experts // world) * 256 + 256
    moe = (cap + cap2) * (D * 3 + D // 32) + (2 << 20)       # buffer sets of a whole call and of a second chunk
    width = cfg.q_lora_rank + cfg.latent_dim + cfg.index_head_dim
    gathers = 2 * 2 * max_tokens * (width * 2 + (max_seq // 32 + 1) * 4 + cfg.index_topk * 4)
    emb = (cfg.vocab_size // world + 1) * D * 2
    return int(rs + moe + gathers + emb + (1 << 30))


def roofline(cfg, world: int, prompts_per_gpu: int, seq: int, decode_per_gpu: int, ctx: int, prefill_ms: float,
             decode_ms: float, peak: dict) -> dict:
    """Fraction of a hardware bound reached per GPU per step (estimates from the model shape).

    Prefill (compute bound): the step's model FLOPs at the measured peaks (fp8 GEMMs at 2x the sustained bf16 rate,
    attention and indexer at the sustained bf16 rate) divided by the measured step time.  Decode (memory bound):
    the bytes a step must stream (expected distinct routed experts per rank under uniform routing, this rank's
    attention / shared / dense weights, the selected latent rows and the indexer keys of its tokens) at the
    measured HBM bandwidth, divided by the measured step time."""
    D, H, L = cfg.hidden_size, cfg.n_heads, cfg.n_layers
    dq, dv, r, dr = cfg.qk_head_dim, cfg.head_out_dim, cfg.kv_lora_rank, cfg.qk_rope_head_dim
    dn = cfg.qk_nope_head_dim
    E, k, I, ql = cfg.n_routed_experts, cfg.n_activated_experts, cfg.moe_intermediate, cfg.q_lora_rank
    n_idx = sum(1 for l in range(L) if cfg.has_indexer(l))
    n_moe = sum(1 for l in range(L) if cfg.is_moe_layer(l))
    n_dense = L - n_moe
    attn_w = D * ql + ql * H * dq + D * cfg.latent_dim + r * H * (dn + dv) + H * dv * D        # params / layer
    idx_w = ql * cfg.index_n_heads * cfg.index_head_dim + D * cfg.index_head_dim + D * cfg.index_n_heads
    expert = 3 * D * I
    topk = cfg.index_topk if cfg.use_indexer else seq
    avg_keys = sum(min(p + 1, topk) for p in range(seq)) / seq
    avg_all = (seq + 1) / 2
    tok = prompts_per_gpu * seq
    fp8_flops = tok * 2 * (L * attn_w + n_moe * (k + cfg.n_shared_experts) * expert + n_dense * 3 * D *
                           cfg.dense_intermediate)
    bf16_flops = tok * 2 * (L * H * (dq + dv) * avg_keys + n_idx * (idx_w + cfg.index_n_heads *
                                                                    cfg.index_head_dim * avg_all))
    bf16 = peak["bf16_tflops_sustained"] * 1e12
    t_pf = fp8_flops / (2 * bf16) + bf16_flops / bf16
    B_tot = decode_per_gpu * world
    El = E // world
    touched = El * (1 - (1 - 1 / E) ** (B_tot * k)) if E else 0
    wbytes = n_moe * (touched * expert + cfg.n_shared_experts * expert) + L * attn_w / world + \
        n_dense * 3 * D * cfg.dense_intermediate + n_idx * idx_w * 2
    from carbon_b200.ref import ops as R

    row = R.latent_fp8_row_bytes(cfg.kv_lora_rank, cfg.qk_rope_head_dim, cfg.attn_kind == "mla") if cfg.kv_fp8 \
        else cfg.latent_dim * 2
    kv = decode_per_gpu * (L * min(ctx, topk) * row + n_idx * ctx * cfg.index_head_dim * 2)
    t_dec = (wbytes + kv) / (peak["hbm_gbs"] * 1e9)
    return {"prefill_frac": round(t_pf / (prefill_ms / 1e3), 3), "decode_frac": round(t_dec / (decode_ms / 1e3), 3),
            "prefill_tflop_per_gpu_step": round((fp8_flops + bf16_flops) / 1e12, 1),
            "decode_gb_per_gpu_step": round((wbytes + kv) / 1e9, 1),
            "basis": "per GPU per step; prefill: model FLOPs at measured peaks (fp8 = 2x sustained bf16); decode: "
                     "streamed bytes (expected routed experts touched, weights, selected KV rows, indexer keys) at "
                     "measured HBM bandwidth"}


def load_peaks() -> dict:
    """Measured peaks of this pool (driver-written MEASURED_PEAKS.json); the pool's earlier measurement otherwise."""
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "hbm_gbs": float(d["hbm_gbs"])}
    except (OSError, KeyError, ValueError):
        return {"bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def count_launches(eng, P, S) -> int:
    """Kernel launches of this repo's extension during one prefill step (counted by the bindings)."""
    from carbon_b200.ops._ext import ext

    e = ext()
    if not hasattr(e, "launch_count"):
        return 0
    reqs = [eng.add_request([1] * S) for _ in range(P)]
    torch.cuda.synchronize()
    c0 = e.launch_count()
    eng.prefill(reqs)
    torch.cuda.synchronize()
    c1 = e.launch_count()
    for r in reqs:
        eng.release(r)
    return int(c1 - c0)


if __name__ == "__main__":
    main()

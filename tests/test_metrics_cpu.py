"""Engine step metrics: counts, tokens/s, TPOT percentiles, JSON line and Prometheus exposition."""
import json

import torch

from carbon_b200.config import tiny_config
from carbon_b200.engine.engine import Engine
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights


def test_engine_metrics():
    cfg = tiny_config()
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=init_weights(cfg, seed=0)), num_pages=16, page_size=16)
    eng.generate([list(range(1, 30)), list(range(5, 20))], max_new_tokens=5)
    s = eng.metrics.summary()
    assert s["prefill"]["steps"] == 1 and s["prefill"]["tokens"] == 29 + 15
    assert s["decode"]["steps"] == 4 and s["decode"]["tokens"] == 8
    assert s["decode"]["tpot_p50_ms"] > 0 and s["decode"]["tokens_per_s"] > 0
    rec = json.loads(eng.metrics.json_line(rank=0))
    assert rec["rank"] == 0 and "decode" in rec["metrics"]
    prom = eng.metrics.prometheus()
    assert 'carbon_tokens_total{kind="prefill"} 44' in prom and 'carbon_tpot_ms{quantile="50"}' in prom


def test_bench_roofline_estimate():
    """The bench's roofline fractions: ~83 GFLOP per prefill token and ~440 GB per one-GPU decode step for the
    full-size model (37B active parameters; ~160 of 256 experts touched per layer by 32 tokens x top-8)."""
    import importlib.util
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")
    spec = importlib.util.spec_from_file_location("carbon_bench", path)
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    from carbon_b200.config import PRESETS

    cfg = PRESETS["deepseek_v3"]()
    peak = {"bf16_tflops_sustained": 1400.0, "hbm_gbs": 6500.0}
    r1 = b.roofline(cfg, 1, 4, 4096, 32, 4096, 1200.0, 110.0, peak)
    assert 70 < r1["prefill_tflop_per_gpu_step"] * 1e12 / (4 * 4096) / 1e9 < 95
    assert 400 < r1["decode_gb_per_gpu_step"] < 480
    assert 0 < r1["prefill_frac"] < 1 and 0 < r1["decode_frac"] < 1
    r8 = b.roofline(cfg, 8, 4, 4096, 32, 4096, 1680.0, 74.0, peak)
    assert r8["decode_gb_per_gpu_step"] < r1["decode_gb_per_gpu_step"] / 4          # 32 experts per rank


def test_tracing_on_cpu_and_chrome_trace(tmp_path):
    import json

    from carbon_b200.config import tiny_config
    from carbon_b200.engine.engine import Engine
    from carbon_b200.utils.trace import tracing

    eng = Engine(tiny_config(), "cpu", num_pages=16, page_size=16)
    with tracing() as t:
        eng.generate([list(range(20)), list(range(5, 17))], 3)
    tot = t.totals()
    assert any(k.startswith("attn.") for k in tot) and any(k.startswith("moe.") for k in tot)
    assert all(c > 0 and ms >= 0 for c, ms in tot.values())
    assert "region" in t.table()
    path = tmp_path / "trace.json"
    n = t.chrome_trace(str(path))
    ev = json.loads(path.read_text())["traceEvents"]
    assert n == len(ev) == len(t.events) > 0
    assert all(e["ph"] == "X" and e["dur"] >= 0 and e["ts"] >= 0 for e in ev)


def test_bench_fills_decode_context_rows():
    """The bench's random decode context: every held request's slots get nonzero latent rows (through the cache's own
    store path, fp8 rows here) and indexer keys, in every layer; slots of other requests stay untouched."""
    import importlib.util
    import os

    import torch

    from carbon_b200.config import tiny_config
    from carbon_b200.engine.engine import Engine
    from carbon_b200.engine.pd import request_slots
    from carbon_b200.models.weights import WeightSource

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")
    spec = importlib.util.spec_from_file_location("carbon_bench_fill", path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = tiny_config().replace(kv_fp8=True)
    eng = Engine(cfg, device="cpu", source=WeightSource(cfg, seed=0), num_pages=16, page_size=16)
    ctx = 40
    reqs = []
    for _ in range(2):
        r = eng.add_request(list(range(ctx)))
        eng._ensure_pages(r, ctx)
        reqs.append(r)
    bench.fill_cache_rows(eng, reqs[:1], ctx, torch.Generator().manual_seed(0))
    s0, s1 = request_slots(eng, reqs[0], ctx), request_slots(eng, reqs[1], ctx)
    for layer in range(cfg.n_layers):
        lat = eng.cache.latent[layer]
        assert bool((lat[s0].float().abs().sum(dim=1) > 0).all())
        assert bool((lat[s1] == 0).all())
        if eng.cache.index_k and eng.cache.index_k[layer] is not None:
            assert bool((eng.cache.index_k[layer][s0].abs().sum(dim=1) > 0).all())

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

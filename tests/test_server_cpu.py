"""HTTP front end: concurrent /generate requests share the scheduler and return each prompt's greedy tokens;
/metrics exposes the step metrics; bad token ids are rejected."""
import threading

import torch

from carbon_b200.config import tiny_config
from carbon_b200.engine.engine import Engine
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights


def test_server_generate_and_metrics():
    from fastapi.testclient import TestClient

    from carbon_b200.engine.server import make_app

    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 7, 33)]
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    want = [ref.generate([p], 5)[0] for p in prompts]
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    with TestClient(make_app(eng)) as client:
        assert client.get("/health").json()["status"] == "ok"
        got = [None] * len(prompts)

        def call(i):
            r = client.post("/generate", json={"input_ids": prompts[i], "max_new_tokens": 5})
            got[i] = r.json()["output_ids"]

        ts = [threading.Thread(target=call, args=(i,)) for i in range(len(prompts))]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=120)
        assert got == want
        assert client.post("/generate", json={"input_ids": [cfg.vocab_size], "max_new_tokens": 2}).status_code == 400
        m = client.get("/metrics").text
        assert 'carbon_tokens_total{kind="decode"}' in m

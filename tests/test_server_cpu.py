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


def test_server_streams_tokens_as_events():
    import json

    from fastapi.testclient import TestClient

    from carbon_b200.engine.server import make_app

    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    prompt = list(range(3, 40))
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    want = ref.generate([prompt], 6)[0]
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    with TestClient(make_app(eng)) as client:
        events = []
        with client.stream("POST", "/generate", json={"input_ids": prompt, "max_new_tokens": 6,
                                                      "stream": True}) as r:
            assert r.status_code == 200
            assert r.headers["content-type"].startswith("text/event-stream")
            for line in r.iter_lines():
                if line.startswith("data: "):
                    events.append(line[len("data: "):])
        assert events[-1] == "[DONE]"
        tokens = [json.loads(e)["token"] for e in events[:-2]]
        assert tokens == want
        assert json.loads(events[-2])["output_ids"] == want
        # a request that can never fit the cache is rejected up front
        big = client.post("/generate", json={"input_ids": [1] * 400, "max_new_tokens": 200})
        assert big.status_code == 400

"""Prefix cache: requests sharing a prompt prefix reuse its KV pages and give the same tokens and logits as an engine
without the cache; eviction frees pages when the allocator runs short."""
import torch

from carbon_b200.config import tiny_config, tiny_v4_config
from carbon_b200.engine.engine import Engine
from carbon_b200.engine.scheduler import Scheduler
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights

import pytest


@pytest.mark.parametrize("variant", ["v3", "v4"])
def test_prefix_reuse_matches_no_cache(variant):
    cfg = tiny_config() if variant == "v3" else tiny_v4_config().replace(n_layers=3, index_sources=(1,))
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(11)
    system = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()        # shared 40-token prefix
    prompts = [system + torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 3, 17)]
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    want, want_lg = ref.generate(prompts, 5, return_logits=True)
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16, prefix_cache=True)
    got = []
    for p in prompts:                               # one at a time: later prompts find the earlier prefixes cached
        out, lg = eng.generate([p], 5, return_logits=True)
        got.append(out[0])
    assert got == want
    assert eng.prefix.hits_tokens == 2 * 32                                       # 2 full pages reused, twice
    # the cache keeps one reference per cached page; everything else went back to the allocator
    assert eng.cache.alloc.num_free() == 32 - 1 - len(eng.prefix.entries)
    eng.prefix.clear()
    assert eng.cache.alloc.num_free() == 32 - 1


def test_prefix_cache_evicts_when_pages_run_short():
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(12)
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=12, page_size=16, prefix_cache=True)
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=12, page_size=16)
    for _ in range(4):                              # distinct 100-token prompts: 7 pages each, 11 usable pages
        p = torch.randint(0, cfg.vocab_size, (100,), generator=g).tolist()
        assert eng.generate([p], 3) == ref.generate([p], 3)
    assert len(eng.prefix.entries) <= 11


def test_scheduler_with_prefix_cache():
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(13)
    system = torch.randint(0, cfg.vocab_size, (48,), generator=g).tolist()
    prompts = [system + torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 20)]
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    want = [ref.generate([p], 4)[0] for p in prompts]
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16, prefix_cache=True)
    sch = Scheduler(eng, prefill_tokens=64)
    a = sch.submit(prompts[0], 4)
    sch.run()
    b = sch.submit(prompts[1], 4)                   # arrives after the first finished: its prefix is cached
    out = sch.run()
    assert [out[a], out[b]] == want and eng.prefix.hits_tokens == 48

"""Speculative decoding: draft + multi-row target verify produces exactly the greedy tokens of plain decoding."""
import torch

from carbon_b200.config import tiny_config
from carbon_b200.engine.engine import Engine
from carbon_b200.engine.spec import NgramDrafter
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights


def test_ngram_drafter():
    d = NgramDrafter()
    assert d.propose([1, 2, 3, 9, 1, 2, 3], 3) == [9, 1, 2]
    assert d.propose([5, 6, 7], 2) == []


def test_speculative_matches_greedy():
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(3)
    base = torch.randint(0, cfg.vocab_size, (20,), generator=g).tolist()
    prompts = [base * 3, torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()]   # repetitive + random
    e1 = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    ref = e1.generate(prompts, 12)
    e2 = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    out = e2.generate_speculative(prompts, 12, NgramDrafter(), n_draft=5)
    assert out == ref
    assert e2.stats["verify_steps"] <= 12

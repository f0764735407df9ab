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


def test_model_drafter_matches_greedy():
    """A draft model proposes, the target verifies: the output is exactly the target's greedy continuation.  With
    the target's own weights as the draft every proposal is accepted (6 tokens per verify step); a 1-layer draft of
    other weights still gives the greedy tokens.  The draft engine's prefix cache reuses the sequence's pages."""
    from carbon_b200.engine.spec import ModelDrafter

    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (37, 21)]
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16).generate(prompts, 12)
    same = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16, prefix_cache=True)
    tgt = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    assert tgt.generate_speculative(prompts, 12, ModelDrafter(same), n_draft=5) == ref
    assert tgt.stats["verify_steps"] == 2                        # 1 + 5 accepted + the bonus token per step
    assert same.prefix.hits_tokens > 0
    small_cfg = cfg.replace(n_layers=1)
    small = Engine(small_cfg, "cpu", source=WeightSource(small_cfg, state=init_weights(small_cfg, seed=3)),
                   num_pages=32, page_size=16, prefix_cache=True)
    tgt2 = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    assert tgt2.generate_speculative(prompts, 12, ModelDrafter(small), n_draft=4) == ref

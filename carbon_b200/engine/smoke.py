"""One tiny serving step on cuda:0: prefill (dense and DSA-sparse prompts) + CUDA-graph decode of a 2-layer
(dense + MoE) model at the reduced-width "small" shape, which keeps every full-size kernel constraint."""
from __future__ import annotations

import torch

from ..config import small_gpu_config
from ..models.weights import WeightSource
from .engine import Engine


def run_smoke(n_layers: int = 2) -> dict:
    assert torch.cuda.is_available(), "smoke() needs a GPU"
    from ..ops._ext import ext

    ext()  # fail loudly if the extension is missing
    cfg = small_gpu_config().replace(n_layers=n_layers)
    eng = Engine(cfg, device="cuda", source=WeightSource(cfg, seed=0), num_pages=64, page_size=64, cuda_graphs=True,
                 graph_buckets=(2, 4))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (300, 40)]
    outs, hist = eng.generate(prompts, max_new_tokens=4, return_logits=True)
    torch.cuda.synchronize()
    for h in hist:
        assert torch.isfinite(h).all(), "non-finite logits"
    info = {"tokens": outs, "logit_absmax": float(max(h.abs().max() for h in hist))}
    print("smoke ok", info)
    return info

"""Multi-rank engine on CPU (gloo, 2 ranks): TP attention over heads (or DP attention over each rank's own
sequences), EP MoE over experts, vocab-parallel embedding and LM head, sequence-sharded residual.  Every rank's
logits must equal the single-process engine's within 1e-4."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from carbon_b200.config import tiny_config
from carbon_b200.engine.engine import Engine
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts(cfg, variant="v3"):
    g = torch.Generator().manual_seed(1)
    # "skewed": prefill shards by tokens (rank 0: the 200-token prompt; rank 1: the short ones) but decode shards by
    # rows (rank 0: requests 0-1), so request 1 decodes on a rank that did not prefill it
    lens = (200, 10, 10) if variant.startswith("skewed") else (64, 50, 70)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]


def _cfg(variant):
    from carbon_b200.config import tiny_v4_config

    variant = variant.replace("+a2a", "")
    if variant.endswith("_fp8kv"):          # the same model over the fp8 latent KV cache
        return _cfg(variant[: -len("_fp8kv")]).replace(kv_fp8=True)
    if variant == "sparse":                 # long-prompt MLA prefill as absorbed sparse attention
        return tiny_config().replace(sparse_prefill_min=40)
    if variant == "v4_late":
        return tiny_v4_config().replace(n_layers=3, index_sources=(1,), late_layer_start=2, late_replay=24)
    if variant == "v3_plain":
        return tiny_config().replace(hc_mult=0)
    return tiny_v4_config().replace(n_layers=3, index_sources=(1,)) if variant == "v4" else tiny_config()


def _worker(rank, world, port, q, attn_dp=False, variant="v3"):
    from datetime import timedelta

    from carbon_b200.parallel.dist import DistCtx

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        cfg = _cfg(variant)
        w = init_weights(cfg, seed=0)
        eng = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16,
                     pctx=DistCtx(rank, world, attn_dp=attn_dp, oproj_a2a=variant.endswith("+a2a")))
        outs, hist = eng.generate(_prompts(cfg, variant), max_new_tokens=6, return_logits=True)
        q.put((rank, outs, [h.numpy().copy() for h in hist]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,attn_dp,variant", [(2, False, "v3"), (2, True, "v3"), (2, False, "v4"),
                                                   (2, True, "v4"), (2, False, "v4_late"), (2, True, "v4_late"),
                                                   (2, True, "skewed"), (2, False, "skewed"), (4, False, "v3"),
                                                   (4, True, "v3"), (2, False, "v3_plain"),
                                                   # TP attention with the head -> token all-to-all output projection
                                                   (2, False, "v3+a2a"), (4, False, "v3+a2a"), (2, False, "v4+a2a"),
                                                   (2, False, "v4_late+a2a"), (2, False, "skewed+a2a"),
                                                   (2, False, "sparse"), (2, False, "sparse+a2a"), (2, True, "sparse"),
                                                   (2, False, "v3_fp8kv+a2a"), (2, True, "v4_fp8kv")])
def test_tp_ep_engine_matches_single_rank(world, attn_dp, variant):
    cfg = _cfg(variant)
    w = init_weights(cfg, seed=0)
    single = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    outs_ref, hist_ref = single.generate(_prompts(cfg, variant), max_new_tokens=6, return_logits=True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, attn_dp, variant)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, outs, hist in results:
        assert outs == outs_ref, rank
        for a, b in zip(hist, hist_ref):
            assert (torch.from_numpy(a) - b).abs().max().item() < 1e-4, rank

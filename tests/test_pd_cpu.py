"""Prefill/decode disaggregation on CPU (gloo): rank 0 prefills and ships KV, rank 1 decodes; tokens equal a single
engine's greedy generation."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from carbon_b200.config import tiny_config
from carbon_b200.engine.engine import Engine
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts(cfg):
    g = torch.Generator().manual_seed(7)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 64, 33)]


def _worker(rank, port, q):
    from datetime import timedelta

    from carbon_b200.engine.pd import DecodeRole, PrefillRole

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=120))
    try:
        cfg = tiny_config()
        w = init_weights(cfg, seed=0)
        eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
        prompts = _prompts(cfg)
        if rank == 0:
            PrefillRole(eng, decode_rank=1).submit(prompts)
        else:
            role = DecodeRole(eng, prefill_rank=0)
            reqs, first = role.receive(len(prompts), prompts)
            q.put(role.generate(reqs, first, 6))
    finally:
        dist.destroy_process_group()


def test_prefill_decode_handoff_matches_single_engine():
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16).generate(_prompts(cfg), 6)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = q.get(timeout=300)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == ref

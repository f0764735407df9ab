"""Prefill/decode disaggregation on 2 GPUs over NCCL: rank 0 prefills on cuda:0 and ships each request's KV rows
(latent and indexer keys of every layer) with isend from a side stream; rank 1 receives them into its own paged cache
on cuda:1 and decodes.  The tokens equal one engine's greedy generation on one GPU (the same kernels in the same
order produce the same bits on either GPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from carbon_b200.config import small_gpu_config

    return small_gpu_config().replace(n_layers=2, vocab_size=2048)


def _prompts(cfg):
    g = torch.Generator().manual_seed(7)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (300, 64, 130)]


def _worker(rank, port, q):
    from datetime import timedelta

    from carbon_b200.engine.engine import Engine
    from carbon_b200.engine.pd import DecodeRole, PrefillRole
    from carbon_b200.models.weights import WeightSource

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=120), device_id=dev)
    try:
        cfg = _cfg()
        eng = Engine(cfg, dev, source=WeightSource(cfg, seed=0), num_pages=32, page_size=64)
        prompts = _prompts(cfg)
        if rank == 0:
            role = PrefillRole(eng, decode_rank=1)
            role.submit(prompts)
            role.flush()
            torch.cuda.synchronize()
            q.put((0, None))
        else:
            role = DecodeRole(eng, prefill_rank=0)
            reqs, first = role.receive(len(prompts), prompts)
            q.put((1, role.generate(reqs, first, 6)))
        dist.barrier()
    except Exception as ex:
        q.put((rank, repr(ex)[:1500]))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_prefill_decode_handoff_over_nccl_matches_one_gpu():
    from carbon_b200.engine.engine import Engine
    from carbon_b200.models.weights import WeightSource

    cfg = _cfg()
    ref = Engine(cfg, "cuda:0", source=WeightSource(cfg, seed=0), num_pages=32, page_size=64).generate(
        _prompts(cfg), 6)
    torch.cuda.empty_cache()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0, res
    assert res[1] == ref, (res[1], ref)

"""Continuous-batching scheduler: jobs admitted at different times, chunked prefill under a token budget and one
shared decode batch produce exactly each job's own greedy continuation; stop tokens end a job early."""
import torch

from carbon_b200.config import tiny_config, tiny_v4_config
from carbon_b200.engine.engine import Engine
from carbon_b200.engine.scheduler import Scheduler
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import init_weights

import pytest


@pytest.mark.parametrize("variant", ["v3", "v4"])
def test_scheduler_matches_greedy(variant):
    cfg = tiny_config() if variant == "v3" else tiny_v4_config().replace(n_layers=3, index_sources=(1,))
    w = init_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 12, 33, 5)]
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    want = [ref.generate([p], 6)[0] for p in prompts]
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=32, page_size=16)
    sch = Scheduler(eng, max_running=3, prefill_tokens=40)      # the 70-token prompt is prefilled in two chunks
    ids = [sch.submit(p, 6) for p in prompts[:2]]
    sch.step()
    sch.step()
    ids += [sch.submit(p, 6) for p in prompts[2:]]             # late arrivals join the running batch
    out = sch.run()
    assert [out[i] for i in ids] == want
    assert sch.steps["prefill"] >= 3 and sch.steps["decode"] >= 5
    assert eng.cache.alloc.num_free() == 32 - 1               # every page returned


def test_scheduler_stop_token_and_sampling():
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=16, page_size=16)
    greedy = eng.generate([[3, 1, 4, 1, 5]], 8)[0]
    sch = Scheduler(eng)
    a = sch.submit([3, 1, 4, 1, 5], 8, stop=(greedy[2],))
    b = sch.submit([3, 1, 4, 1, 5], 8, temperature=0.8, top_k=20, seed=7)
    c = sch.submit([3, 1, 4, 1, 5], 8, temperature=0.8, top_k=20, seed=7)
    out = sch.run()
    assert out[a] == greedy[:greedy.index(greedy[2]) + 1]
    assert out[b] == out[c] and len(out[b]) == 8                # seeded sampling is reproducible


def _sched_worker(rank, world, port, q):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from carbon_b200.parallel.dist import DistCtx

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        cfg = tiny_config()
        eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=init_weights(cfg, seed=0)), num_pages=32,
                     page_size=16, pctx=DistCtx(rank, world))
        g = torch.Generator().manual_seed(5)
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 12, 33)]
        sch = Scheduler(eng, max_running=2, prefill_tokens=40)
        ids = [sch.submit(p, 5) for p in prompts]
        out = sch.run()
        q.put((rank, [out[i] for i in ids]))
    finally:
        dist.destroy_process_group()


def test_scheduler_spmd_two_ranks():
    """Every rank runs the same scheduler on the same submissions (TP attention + EP MoE over gloo): the ranks take
    the same steps and produce the single-rank tokens."""
    import socket

    import torch.multiprocessing as mp

    cfg = tiny_config()
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 12, 33)]
    ref = Engine(cfg, "cpu", source=WeightSource(cfg, state=init_weights(cfg, seed=0)), num_pages=32, page_size=16)
    want = [ref.generate([p], 5)[0] for p in prompts]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_sched_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, outs in res:
        assert outs == want, rank


def test_preemption_under_kv_pressure_keeps_outputs():
    """A cache far smaller than the batch's final footprint: admission waits for pages, decode preempts the youngest
    requests (their KV is freed and recomputed on readmission), and every request still gets the tokens it gets
    with a large cache."""
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    prompts = [((torch.arange(30) * (k + 3) + k) % cfg.vocab_size).tolist() for k in range(4)]

    def serve(num_pages, prefill_tokens=4096):
        eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=num_pages, page_size=16)
        s = Scheduler(eng, prefill_tokens=prefill_tokens)
        ids = [s.submit(p, 40) for p in prompts]
        out = s.run()
        assert eng.cache.alloc.num_free() == num_pages - 1                 # every page back (scratch page kept)
        return [out[i] for i in ids], s

    ref, s_big = serve(64)
    assert s_big.preemptions == 0
    got, s_small = serve(10)                       # 9 usable pages; the four requests end at 5 pages each
    assert s_small.preemptions > 0
    assert got == ref
    got2, s_chunk = serve(10, prefill_tokens=20)   # chunked prefills competing for pages
    assert got2 == ref
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=4, page_size=16)
    with pytest.raises(ValueError):
        Scheduler(eng).submit(list(range(40)), 20)                          # 60 tokens > 3 pages x 16

"""Cost-model balancing of DP attention ranks: the planner evens out skewed batches, and an engine that places its
prefill sequences and decode rows by the plan serves exactly the same tokens as one that splits by count."""
import socket

import pytest

import torch

from carbon_b200.config import deepseek_v3_config, tiny_config
from carbon_b200.parallel import balance
from carbon_b200.parallel.dist import split_bounds


def test_seq_cost_grows_with_context_and_respects_caps():
    cfg = deepseek_v3_config()
    # prefill cost is superlinear in length (attention / indexer pairs), decode cost grows with the context
    assert balance.seq_cost(cfg, 8192) > 2.05 * balance.seq_cost(cfg, 4096)
    assert balance.seq_cost(cfg, 1, 8192) > balance.seq_cost(cfg, 1, 1024)
    assert balance._capped_pairs(0, 10, 0) == 55
    assert balance._capped_pairs(0, 10, 4) == sum(min(p + 1, 4) for p in range(10))
    assert balance._capped_pairs(5, 7, 6) == sum(min(p + 1, 6) for p in range(5, 12))


def test_plan_prefill_beats_token_split_on_skewed_batch():
    cfg = deepseek_v3_config()
    lengths = [8192, 8192] + [1024] * 16                    # the token split puts both long prompts on rank 0
    world = 2
    order, bounds, load = balance.plan_prefill(cfg, lengths, world)
    assert sorted(order) == list(range(len(lengths)))
    assert bounds[0] == 0 and bounds[-1] == sum(lengths)
    # each rank's tokens are whole sequences of the reordered batch
    acc, cuts = 0, {0}
    for i in order:
        acc += lengths[i]
        cuts.add(acc)
    assert set(bounds) <= cuts
    base = balance.split_costs(cfg, lengths, split_bounds(lengths, world))
    assert balance.imbalance(load) < 1.01 < 1.1 < balance.imbalance(base)   # DSA caps attention: ~1.12
    assert abs(sum(load) - sum(base)) / sum(base) < 1e-9


def test_plan_rows_keeps_block_capacities():
    g = torch.Generator().manual_seed(0)
    ctx = torch.randint(16, 30000, (13,), generator=g).tolist()
    cfg = deepseek_v3_config()
    costs = [balance.seq_cost(cfg, 1, c) for c in ctx]
    bounds = split_bounds([1] * 16, 4)                      # bucket 16 (3 padding rows) over 4 ranks
    perm = balance.plan_rows(costs, bounds)
    assert sorted(perm) == list(range(13))
    per = [sum(costs[perm[j]] for j in range(bounds[r], min(bounds[r + 1], 13))) for r in range(4)]
    naive = [sum(costs[j] for j in range(bounds[r], min(bounds[r + 1], 13))) for r in range(4)]
    assert max(per) <= max(naive) + 1e-6


def _prompts(cfg):
    return [(torch.arange(90) * 5 % cfg.vocab_size).tolist(), (torch.arange(60) * 3 % cfg.vocab_size).tolist(),
            list(range(1, 9)), list(range(20, 27)), list(range(40, 50)), list(range(60, 69))]


def _worker(rank, world, port, q, balanced):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from carbon_b200.engine.engine import Engine
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.parallel.dist import DistCtx
    from carbon_b200.ref.model import init_weights

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        cfg = tiny_config()
        w = init_weights(cfg, seed=0)
        e = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=48, page_size=16,
                   pctx=DistCtx(rank, world, attn_dp=True), balance_dp=balanced)
        prompts = _prompts(cfg)
        out, h = e.generate(prompts, 4, return_logits=True)
        q.put((rank, balanced, out, [x.tolist() for x in h]))       # plain lists: no shared-memory handles
    finally:
        dist.destroy_process_group()


def _run(balanced):
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, balanced)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res, key=lambda x: x[0])


def test_balanced_dp_engine_serves_the_same_tokens():
    cfg = tiny_config()
    lens = [len(p) for p in _prompts(cfg)]
    # the plans differ from the count split, so the balanced run really reorders prefill and decode
    assert balance.plan_prefill(cfg, lens, 2)[1] != split_bounds(lens, 2)
    perm = balance.plan_rows([balance.seq_cost(cfg, 1, n + 1) for n in lens], split_bounds([1] * len(lens), 2))
    assert perm != list(range(len(lens)))
    plain = _run(False)
    bal = _run(True)
    for (r0, _, out0, h0), (r1, _, out1, h1) in zip(plain, bal):
        assert out0 == out1, (r0, out0, out1)
        for a, b in zip(h0, h1):
            assert (torch.tensor(a) - torch.tensor(b)).abs().max() < 1e-3


def _owner_cfg(mode):
    if "v4" in mode:
        from carbon_b200.config import tiny_v4_config

        cfg = tiny_v4_config().replace(n_layers=3, index_sources=(1,), engram_layers=())
    else:
        cfg = tiny_config()
    return cfg.replace(kv_fp8=True) if mode.endswith("_fp8kv") else cfg


def _owner_worker(rank, world, port, q, mode="dp"):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from carbon_b200.engine.engine import Engine
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.parallel.dist import DistCtx
    from carbon_b200.ref.model import init_weights

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        cfg = _owner_cfg(mode)
        w = init_weights(cfg, seed=0)
        e = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=48, page_size=16,
                   pctx=DistCtx(rank, world, attn_dp=mode == "dp", oproj_a2a="a2a" in mode), owner_kv=True)
        reqs = [e.add_request(p) for p in _prompts(cfg)]
        logits = e.prefill(reqs)
        hist = [logits.tolist()]
        nxt = torch.argmax(logits, -1).tolist()
        outs = [[t] for t in nxt]
        used = 0
        for _ in range(4):
            logits = e.decode(reqs, nxt)
            hist.append(logits.tolist())
            nxt = torch.argmax(logits, -1).tolist()
            for o, t in zip(outs, nxt):
                o.append(t)
            used = 47 - e.cache.alloc.num_free()
        homes = [r.home for r in reqs]
        mine = sum(len(r.pages) for r in reqs)
        for r in reqs:
            e.release(r)
        # chunked prefill (per-row attention over each home rank's cached chunks), then the same decode steps
        reqs = [e.add_request(p) for p in _prompts(cfg)]
        logits = e.prefill_chunked(reqs, 24)
        hist2 = [logits.tolist()]
        nxt = torch.argmax(logits, -1).tolist()
        for _ in range(4):
            logits = e.decode(reqs, nxt)
            hist2.append(logits.tolist())
            nxt = torch.argmax(logits, -1).tolist()
        for r in reqs:
            e.release(r)
        spec = e.generate_speculative(_prompts(cfg), 5, n_draft=3)     # verify rows grouped by home rank
        q.put((rank, outs, hist, homes, mine, used, e.cache.alloc.num_free(), hist2, spec))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["dp", "tp", "tp_a2a", "tp_a2a_v4", "tp_a2a_fp8kv"])
def test_owner_kv_matches_single_rank_and_splits_pages(mode):
    """Owner-only KV on 2 ranks (DP attention, or TP attention whose cache-reading core runs token-parallel): each
    request's KV lives on its home rank only, yet the served tokens and logits equal the single-rank engine's, with
    whole-prompt and chunked prefill and with speculative verify; the ranks' page counts add up to the single
    rank's."""
    import torch.multiprocessing as mp

    from carbon_b200.engine.engine import Engine
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.ref.model import init_weights

    cfg = _owner_cfg(mode)
    w = init_weights(cfg, seed=0)
    single = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=48, page_size=16)
    ref_out, ref_hist = single.generate(_prompts(cfg), 5, return_logits=True)
    ref_hist2 = []
    if mode.endswith("_fp8kv"):
        reqs = [single.add_request(p) for p in _prompts(cfg)]
        logits = single.prefill_chunked(reqs, 24)
        ref_hist2.append(logits)
        nxt = torch.argmax(logits, -1).tolist()
        for _ in range(4):
            logits = single.decode(reqs, nxt)
            ref_hist2.append(logits)
            nxt = torch.argmax(logits, -1).tolist()
        for r in reqs:
            single.release(r)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_owner_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda x: x[0])
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    total_pages = 0
    for rank, outs, hist, homes, mine, used, free_after, hist2, spec in res:
        assert outs == ref_out, (rank, outs, ref_out)
        assert spec == ref_out, (rank, spec, ref_out)
        for a, b in zip(hist, ref_hist):
            assert (torch.tensor(a) - b).abs().max() < 1e-3
        # chunked prefill: the same logits as the whole prompt (fp8 cache: as the single rank's chunked prefill, whose
        # later chunks likewise attend over fp8-cached rows)
        for a, b in zip(hist2, ref_hist2 if mode.endswith("_fp8kv") else ref_hist):
            assert (torch.tensor(a) - b).abs().max() < 1e-3
        assert sorted(set(homes)) == [0, 1]                         # both ranks own requests
        assert used == mine                                          # pages only for this rank's own requests
        assert free_after == 47
        total_pages += mine
    lens = [len(p) + 4 for p in _prompts(cfg)]                      # prompt + 4 decoded tokens cached
    assert total_pages == sum((n + 15) // 16 for n in lens)         # the KV of each request is held once


def _owner_sched_worker(rank, world, port, q, num_pages, prefill_tokens):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from carbon_b200.engine.engine import Engine
    from carbon_b200.engine.scheduler import Scheduler
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.parallel.dist import DistCtx
    from carbon_b200.ref.model import init_weights

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        cfg = tiny_config()
        w = init_weights(cfg, seed=0)
        e = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=num_pages, page_size=16,
                   pctx=DistCtx(rank, world, attn_dp=True), owner_kv=True)
        s = Scheduler(e, prefill_tokens=prefill_tokens)
        ids = [s.submit(p, 40) for p in _sched_prompts(cfg)]
        out = s.run()
        q.put((rank, [out[i] for i in ids], s.preemptions, e.cache.alloc.num_free()))
    finally:
        dist.destroy_process_group()


def _sched_prompts(cfg):
    return [((torch.arange(30) * (k + 3) + k) % cfg.vocab_size).tolist() for k in range(4)]


def test_scheduler_with_dp_owner_kv_under_pressure():
    """The serving loop over 2 DP ranks with owner-only KV: homes chosen at admission, pages budgeted per rank.
    With a per-rank cache too small for its two requests' final footprint, the ranks preempt in step (same
    decisions on both) and every request still gets the single-rank engine's tokens, also with chunked prefill."""
    import torch.multiprocessing as mp

    from carbon_b200.engine.engine import Engine
    from carbon_b200.engine.scheduler import Scheduler
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.ref.model import init_weights

    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    eng = Engine(cfg, "cpu", source=WeightSource(cfg, state=w), num_pages=64, page_size=16)
    s = Scheduler(eng)
    ids = [s.submit(p, 40) for p in _sched_prompts(cfg)]
    out = s.run()
    ref = [out[i] for i in ids]
    for num_pages, pressured, chunk in ((64, False, 4096), (9, True, 4096), (9, True, 20)):
        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
        sk.close()
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        ps = [ctx.Process(target=_owner_sched_worker, args=(r, 2, port, q, num_pages, chunk)) for r in range(2)]
        for p in ps:
            p.start()
        res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda x: x[0])
        for p in ps:
            p.join(timeout=60)
            assert p.exitcode == 0
        for rank, got, pre, free in res:
            assert got == ref, (num_pages, rank)
            assert (pre > 0) == pressured, (num_pages, rank, pre)
            assert free == num_pages - 1                          # every page back
        assert res[0][2] == res[1][2]                             # the same preemptions on both ranks

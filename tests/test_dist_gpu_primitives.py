"""Each NVLink collective of FusedCtx against its NCCL counterpart (DistCtx) on identical inputs, 2 GPUs, uneven
token shards: all-gather, reduce-scatter, o_proj GEMM->reduce-scatter, vocab-parallel embedding, EP MoE."""
import os
import socket
import types

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


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-9)).item()


def _worker(rank, world, port, q):
    from datetime import timedelta

    from carbon_b200.config import small_gpu_config
    from carbon_b200.models.deepseek import DeepseekModel, Lin
    from carbon_b200.models.weights import WeightSource
    from carbon_b200.ops import core as C
    from carbon_b200.parallel.dist import DistCtx
    from carbon_b200.parallel.fused import FusedCtx

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    res = {}
    try:
        f = FusedCtx(rank, world, heap_bytes=2 << 30, max_tokens=4608, max_seq=256)
        d = DistCtx(rank, world)
        bounds = [0, 100, 230] if world == 2 else [0, 230]
        f.set_bounds(bounds)
        d.set_bounds(bounds)
        lo, hi = bounds[rank], bounds[rank + 1]
        g = torch.Generator(device=dev).manual_seed(10 + rank)
        gall = torch.Generator(device=dev).manual_seed(99)
        # all-gather (bf16 rows and 40-byte int32 rows)
        x = torch.randn(hi - lo, 576, device=dev, generator=g).to(torch.bfloat16)
        res["gather_bf16"] = _rel(f.gather_rows(x), d.gather_rows(x))
        m = torch.randint(0, 1 << 30, (hi - lo, 10), device=dev, generator=g, dtype=torch.int32)
        res["gather_i32"] = float((f.gather_rows(m) != d.gather_rows(m)).sum().item())
        # reduce-scatter
        part = torch.randn(230, 1024, device=dev, generator=g).to(torch.bfloat16)
        res["rs"] = _rel(f.reduce_scatter_rows(part), d.reduce_scatter_rows(part))
        # o_proj GEMM -> reduce-scatter
        lin = Lin(torch.randn(1024, 2048, device=dev, generator=gall) * 0.02, dev)
        o = torch.randn(230, 2048, device=dev, generator=g).to(torch.bfloat16)
        res["gemm_rs"] = _rel(f.row_parallel_out(lin, o), d.reduce_scatter_rows(lin(o)))
        # vocab-parallel embedding
        V, D = 2048, 1024
        table = (torch.randn(V, D, device=dev, generator=gall) * 0.02).to(torch.bfloat16)
        per = V // world
        ids = torch.randint(0, V, (230,), device=dev, generator=gall, dtype=torch.int32)
        cfg = small_gpu_config().replace(vocab_size=V, hidden_size=D, hc_mult=4)
        md = types.SimpleNamespace(cfg=cfg, embed=table[rank * per:(rank + 1) * per].contiguous(), v_lo=rank * per,
                                   v_hi=(rank + 1) * per, on_gpu=True)
        mf = types.SimpleNamespace(cfg=cfg, embed=md.embed.clone(), v_lo=md.v_lo, v_hi=md.v_hi, on_gpu=True)
        Xf, _ = f.embed(mf, ids)
        Xd, _ = d.embed(md, ids)
        res["embed"] = _rel(Xf, Xd)
        res["embed_vs_table"] = _rel(Xf[:, 0], table[ids[lo:hi].long()])
        # EP MoE
        mcfg = small_gpu_config().replace(n_layers=1, n_dense_layers=0, n_routed_experts=8, n_activated_experts=2,
                                          vocab_size=2048)
        model = DeepseekModel(mcfg, WeightSource(mcfg, seed=3), dev, pctx=f)
        L = model.layers[0]
        h = torch.randn(hi - lo, mcfg.hidden_size, device=dev, generator=g).to(torch.bfloat16)
        w, idx = C.router_topk(torch.randn(hi - lo, 8, device=dev, generator=g), None, 2, "sigmoid", 1.0, True)
        res["moe"] = _rel(f.moe(model, L, h, w, idx, None), d.moe(model, L, h, w, idx, None))
        # prefill-sized shards: CTA-pair o_proj scatter epilogue (M >= 512) and the two-chunk pipelined MoE
        big = [0, 2300, 4608] if world == 2 else [0, 4608]
        f.set_bounds(big)
        d.set_bounds(big)
        blo, bhi = big[rank], big[rank + 1]
        o = torch.randn(4608, 2048, device=dev, generator=g).to(torch.bfloat16)
        res["gemm_rs_big"] = _rel(f.row_parallel_out(lin, o), d.reduce_scatter_rows(lin(o)))
        h = torch.randn(bhi - blo, mcfg.hidden_size, device=dev, generator=g).to(torch.bfloat16)
        w, idx = C.router_topk(torch.randn(bhi - blo, 8, device=dev, generator=g), None, 2, "sigmoid", 1.0, True)
        sh = torch.randn(bhi - blo, mcfg.hidden_size, device=dev, generator=g).to(torch.bfloat16)
        res["moe_big"] = _rel(f.moe(model, L, h, w, idx, sh), d.moe(model, L, h, w, idx, sh))
        torch.cuda.synchronize()
        res["status"] = f.check()
        q.put((rank, res))
        dist.barrier()
    except Exception as ex:
        q.put((rank, {"error": repr(ex)[:1500]}))
        raise
    finally:
        dist.destroy_process_group()


def _run(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    for rank, r in res.items():
        assert "error" not in r, (rank, r)
        assert r["status"] == 0, (rank, r)
        assert r["gather_bf16"] == 0 and r["gather_i32"] == 0, (rank, r)
        assert r["rs"] < 1e-2 and r["gemm_rs"] < 1e-2 and r["gemm_rs_big"] < 1e-2, (rank, r)
        assert r["embed"] == 0 and r["embed_vs_table"] == 0, (rank, r)
        assert r["moe"] < 2e-2 and r["moe_big"] < 2e-2, (rank, r)


def test_fused_collectives_one_rank():
    """The same kernels with every peer pointer local: dispatch / combine / scatter index arithmetic on one GPU."""
    _run(1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_collectives_match_nccl():
    _run(2)

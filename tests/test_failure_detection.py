"""Failure detection without a GPU fault.

* GPU: the cross-rank barrier kernel waits on a flag that nothing sets; its bounded wait must run out after the
  configured limit, record kErrTimeoutPeer in the status word and return — and the CUDA context stays usable.
* CPU (gloo): a rank that raises before a collective makes the surviving rank's collective end with an error
  (short process-group timeout) instead of hanging; both processes exit.
"""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

K_ERR_TIMEOUT_PEER = 4


@pytest.mark.gpu
def test_barrier_times_out_with_status_and_context_survives():
    from carbon_b200.ops._ext import ext

    e = ext()
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # a two-"rank" barrier whose peer slot (index 1) nothing ever writes: both table entries point at our own flags,
    # so the kernel publishes slot 0 and then waits for slot 1
    peers = torch.tensor([flags.data_ptr(), flags.data_ptr()], dtype=torch.int64, device="cuda")
    t0 = time.time()
    e.p2p_barrier(peers, 0, epoch, flags, status, int(0.3e9))
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(status.item()) == K_ERR_TIMEOUT_PEER
    assert 0.25 < dt < 10.0
    # with an error already recorded, later barriers signal but do not wait: the failure surfaces at once
    t1 = time.time()
    e.p2p_barrier(peers, 0, epoch, flags, status, int(0.3e9))
    torch.cuda.synchronize()
    assert time.time() - t1 < 0.2
    x = torch.randn(256, 256, device="cuda")
    assert torch.isfinite(x @ x).all()          # context still usable


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((1, "raised"))
        q.close()
        q.join_thread()                   # make sure the message is delivered before the process disappears
        os._exit(3)                       # the failing rank leaves between steps, no collective in flight
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put((0, "no error"))
    except Exception as ex:                # the survivor learns of it from the collective's error
        q.put((0, "error:" + type(ex).__name__))


def test_dead_rank_surfaces_as_collective_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    assert got[1] == "raised"
    assert got[0].startswith("error:")
    assert all(p.exitcode is not None for p in ps)

"""Host-side failure detection (no GPU): a rank that dies or leaves is seen through the store's heartbeats before
the survivor launches its next step, and a step that overruns the watchdog's limit raises instead of hanging."""
import os
import socket
import time

import pytest
import torch.multiprocessing as mp

from carbon_b200.utils.health import Heartbeat, PeerFailure, StepStalled, Watchdog


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _hb_worker(rank, port, q, mode):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, 2, interval=0.1, max_age=1.5).start()
    dist.barrier()
    if rank == 1:
        for _ in range(3):                       # a few healthy steps
            hb.check()
            time.sleep(0.1)
        if mode == "leave":
            hb.leave()
        q.put((1, "gone"))
        q.close()
        q.join_thread()
        os._exit(0 if mode == "leave" else 3)    # "crash": no goodbye, the heartbeat thread dies with the process
    t0 = time.monotonic()
    try:
        while time.monotonic() - t0 < 30:        # the survivor's serving loop: check, then (would) launch
            hb.check()
            time.sleep(0.05)
        q.put((0, "no failure seen", 0.0))
    except PeerFailure as e:
        q.put((0, f"{e.rank}:{e.reason}", time.monotonic() - t0))
    hb.stop()
    q.close()
    q.join_thread()                              # deliver the result before the process disappears
    os._exit(0)                                  # the process group's peer is gone: skip its teardown


@pytest.mark.parametrize("mode", ["crash", "leave"])
def test_heartbeat_reports_a_dead_or_departed_peer(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_hb_worker, args=(r, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    got = {}
    for _ in range(2):
        m = q.get(timeout=120)
        got[m[0]] = m[1:]
    for p in ps:
        p.join(timeout=60)
    assert got[1] == ("gone",)
    reason, dt = got[0]
    assert reason.startswith("1:"), reason
    if mode == "leave":
        assert "left" in reason and dt < 3.0
    else:
        assert "silent" in reason and dt < 10.0


def test_watchdog_turns_a_stall_into_an_exception():
    wd = Watchdog(timeout=0.3, dump_stacks=False)
    with wd.step("quick"):
        time.sleep(0.01)
    t0 = time.monotonic()
    with pytest.raises(StepStalled):
        with wd.step("stuck"):
            time.sleep(30)
    assert time.monotonic() - t0 < 5
    assert wd.stalls == 1
    with wd.step("after"):                       # usable again, no stray interrupt left behind
        time.sleep(0.01)
    time.sleep(0.5)                              # a late signal, had one been sent, would land here


def test_scheduler_checks_peers_before_each_step():
    from carbon_b200.config import tiny_config
    from carbon_b200.engine.engine import Engine
    from carbon_b200.engine.scheduler import Scheduler

    class DeadPeer:
        def check(self):
            raise PeerFailure(1, "heartbeat silent for 9.9 s")

    eng = Engine(tiny_config(), "cpu", num_pages=16, page_size=16)
    s = Scheduler(eng, heartbeat=DeadPeer(), watchdog=Watchdog(60.0), check_device=True)
    s.submit(list(range(10)), 2)
    with pytest.raises(PeerFailure):
        s.step()
    assert s.steps == {"prefill": 0, "decode": 0}          # nothing was launched
    s.heartbeat = None
    assert len(s.run()[0]) == 2

"""Built-in tracing: NVTX ranges and CUDA-event timers per named region of the forward pass.

The reference has no profiler of its own (boot lines, ``DECODE_GEMM`` traces and CUDA-event best-of-3 timing in its
CHECK twins, ``king_v10/bundle_v9/prefill_gemm.py:79-90``).  Here every op of the model runs inside
``region("name")``; when tracing is enabled each region pushes an NVTX range (visible in nsys/ncu) and records a
pair of CUDA events on the current stream, so per-region device time can be read back without synchronising
inside the step:

    with tracing() as t:
        engine.prefill(reqs)
    print(t.table())
    t.chrome_trace("prefill.json")      # open in Perfetto / chrome://tracing: one track per stream

Without a GPU (the CPU engine) the regions are timed with the host clock instead, so the same tables and traces
come out of CPU runs.  Regions inside CUDA-graph capture are skipped (graph replays show up as one region of the
caller).
"""
from __future__ import annotations

import contextlib
import json
import os
import time
from collections import defaultdict
from typing import Dict, List, Optional, Tuple

import torch

_ACTIVE: Optional["Tracer"] = None


class Tracer:
    def __init__(self):
        # (name, start, end, stream id): CUDA events on the GPU, host perf_counter seconds on the CPU
        self.events: List[Tuple[str, object, object, int]] = []

    def _spans(self) -> List[Tuple[str, float, float, int]]:
        """(name, start ms, duration ms, stream) of every region, starts relative to the first region."""
        if not self.events:
            return []
        first = self.events[0][1]
        if isinstance(first, float):
            return [(n, (a - first) * 1e3, (b - a) * 1e3, st) for n, a, b, st in self.events]
        torch.cuda.synchronize()
        return [(n, first.elapsed_time(a), a.elapsed_time(b), st) for n, a, b, st in self.events]

    def totals(self) -> Dict[str, Tuple[int, float]]:
        agg: Dict[str, List[float]] = defaultdict(lambda: [0, 0.0])
        for name, _, dur, _ in self._spans():
            agg[name][0] += 1
            agg[name][1] += dur
        return {k: (int(v[0]), float(v[1])) for k, v in agg.items()}

    def chrome_trace(self, path: str, pid: Optional[int] = None) -> int:
        """Write the regions as a Chrome trace-event file (complete events, microseconds; one thread per stream,
        the process id defaults to this rank).  Returns the number of events written."""
        if pid is None:
            pid = int(os.environ.get("RANK", "0"))
        ev = [{"name": n, "ph": "X", "ts": round(t0 * 1e3, 3), "dur": round(d * 1e3, 3), "pid": pid, "tid": st,
               "cat": n.split(".")[0]} for n, t0, d, st in self._spans()]
        with open(path, "w") as f:
            json.dump({"traceEvents": ev, "displayTimeUnit": "ms"}, f)
        return len(ev)

    def table(self, top: int = 40) -> str:
        tot = self.totals()
        s = sum(v for _, v in tot.values()) or 1.0
        lines = [f"{'region':28s} {'calls':>6s} {'ms':>10s} {'share':>7s}"]
        for k, (c, v) in sorted(tot.items(), key=lambda x: -x[1][1])[:top]:
            lines.append(f"{k:28s} {c:6d} {v:10.3f} {100 * v / s:6.1f}%")
        return "\n".join(lines)


@contextlib.contextmanager
def tracing():
    global _ACTIVE
    prev, _ACTIVE = _ACTIVE, Tracer()
    try:
        yield _ACTIVE
    finally:
        _ACTIVE = prev


@contextlib.contextmanager
def region(name: str):
    t = _ACTIVE
    if t is None:
        yield
        return
    if not torch.cuda.is_available():
        a = time.perf_counter()
        try:
            yield
        finally:
            t.events.append((name, a, time.perf_counter(), 0))
        return
    if torch.cuda.is_current_stream_capturing():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    try:
        yield
    finally:
        b.record(stream)
        torch.cuda.nvtx.range_pop()
        t.events.append((name, a, b, int(stream.stream_id)))

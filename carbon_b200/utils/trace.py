"""Built-in tracing: NVTX ranges and CUDA-event timers per named region of the forward pass.

The reference has no profiler of its own (boot lines, ``DECODE_GEMM`` traces and CUDA-event best-of-3 timing in its
CHECK twins, ``king_v10/bundle_v9/prefill_gemm.py:79-90``).  Here every op of the model runs inside
``region("name")``; when tracing is enabled each region pushes an NVTX range (visible in nsys/ncu) and records a
pair of CUDA events on the current stream, so per-region device time can be read back without synchronising
inside the step:

    with tracing() as t:
        engine.prefill(reqs)
    print(t.table())
"""
from __future__ import annotations

import contextlib
from collections import defaultdict
from typing import Dict, List, Optional, Tuple

import torch

_ACTIVE: Optional["Tracer"] = None


class Tracer:
    def __init__(self):
        self.events: List[Tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def totals(self) -> Dict[str, Tuple[int, float]]:
        torch.cuda.synchronize()
        agg: Dict[str, List[float]] = defaultdict(lambda: [0, 0.0])
        for name, a, b in self.events:
            agg[name][0] += 1
            agg[name][1] += a.elapsed_time(b)
        return {k: (int(v[0]), float(v[1])) for k, v in agg.items()}

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
    if t is None or not torch.cuda.is_available() or torch.cuda.is_current_stream_capturing():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    try:
        yield
    finally:
        b.record()
        torch.cuda.nvtx.range_pop()
        t.events.append((name, a, b))

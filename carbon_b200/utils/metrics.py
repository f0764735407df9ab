"""Serving metrics: per-step device time, tokens/s, TPOT percentiles; JSON lines and Prometheus exposition.

The reference logs with Python ``logging`` and stderr lines and exports no metrics (its per-lever counters,
``replay_counts.py:8``, ``exchange_fuse.py:13``).  Here the engine records every prefill / decode / verify step
with a pair of CUDA events on the launching stream (no synchronisation inside the step); ``summary()`` reads them
back once, ``json_line()`` gives one structured record and ``prometheus()`` the text exposition format (metric
names prefixed ``carbon_``), so a scraper or a log shipper can take either.
"""
from __future__ import annotations

import json
import time
from collections import defaultdict
from typing import Dict, List, Optional

import torch


def _percentile(xs: List[float], q: float) -> float:
    if not xs:
        return 0.0
    s = sorted(xs)
    i = min(len(s) - 1, max(0, int(round(q * (len(s) - 1)))))
    return s[i]


class StepTimer:
    """Context manager timing one engine step on the device (CPU engines: wall clock)."""

    def __init__(self, metrics: "Metrics", kind: str, tokens: int, rows: int):
        self.m, self.kind, self.tokens, self.rows = metrics, kind, tokens, rows

    def __enter__(self):
        if torch.cuda.is_available() and not torch.cuda.is_current_stream_capturing() and self.m.device_timing:
            self.a = torch.cuda.Event(enable_timing=True)
            self.b = torch.cuda.Event(enable_timing=True)
            self.a.record()
        else:
            self.a = None
            self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.a is not None:
            self.b.record()
            self.m._pending.append((self.kind, self.tokens, self.rows, self.a, self.b))
            if len(self.m._pending) >= 4096:        # bound the events held: read them back (one sync per 4096 steps)
                self.m._resolve()
        else:
            self.m._done.append((self.kind, self.tokens, self.rows, (time.perf_counter() - self.t0) * 1e3))
        return False


class Metrics:
    def __init__(self, device_timing: bool = True, keep: int = 100000):
        self.device_timing = device_timing
        self.keep = keep
        self._pending = []
        self._done = []

    def step(self, kind: str, tokens: int, rows: int = 0) -> StepTimer:
        return StepTimer(self, kind, tokens, rows)

    def _resolve(self):
        if self._pending:
            torch.cuda.synchronize()
            for kind, tok, rows, a, b in self._pending:
                self._done.append((kind, tok, rows, a.elapsed_time(b)))
            self._pending = []
        if len(self._done) > self.keep:
            self._done = self._done[-self.keep:]

    def summary(self) -> Dict[str, Dict[str, float]]:
        """Per step kind: steps, tokens, total ms, tokens/s, and (decode) TPOT p50 / p90 / p99 in ms."""
        self._resolve()
        by = defaultdict(list)
        for kind, tok, rows, ms in self._done:
            by[kind].append((tok, rows, ms))
        out = {}
        for kind, xs in by.items():
            ms = [x[2] for x in xs]
            tok = sum(x[0] for x in xs)
            tot = sum(ms)
            d = {"steps": len(xs), "tokens": tok, "ms": round(tot, 3),
                 "tokens_per_s": round(tok / (tot / 1e3), 1) if tot > 0 else 0.0}
            if kind == "decode":
                d.update({"tpot_p50_ms": round(_percentile(ms, 0.5), 3), "tpot_p90_ms": round(_percentile(ms, 0.9), 3),
                          "tpot_p99_ms": round(_percentile(ms, 0.99), 3)})
            out[kind] = d
        return out

    def json_line(self, **extra) -> str:
        rec = {"ts": round(time.time(), 3), "metrics": self.summary()}
        rec.update(extra)
        return json.dumps(rec)

    def prometheus(self) -> str:
        """Text exposition format (0.0.4)."""
        lines = []
        summ = self.summary()

        def emit(name, help_, typ, vals):
            lines.append(f"# HELP carbon_{name} {help_}")
            lines.append(f"# TYPE carbon_{name} {typ}")
            for labels, v in vals:
                lab = ",".join(f'{k}="{x}"' for k, x in labels.items())
                lines.append(f"carbon_{name}{{{lab}}} {v}")

        emit("steps_total", "engine steps run", "counter", [({"kind": k}, d["steps"]) for k, d in summ.items()])
        emit("tokens_total", "tokens processed", "counter", [({"kind": k}, d["tokens"]) for k, d in summ.items()])
        emit("step_ms_total", "device milliseconds spent in steps", "counter",
             [({"kind": k}, d["ms"]) for k, d in summ.items()])
        emit("tokens_per_second", "tokens per second of step time", "gauge",
             [({"kind": k}, d["tokens_per_s"]) for k, d in summ.items()])
        if "decode" in summ:
            emit("tpot_ms", "decode time per output token", "gauge",
                 [({"quantile": q}, summ["decode"][f"tpot_p{q}_ms"]) for q in ("50", "90", "99")])
        return "\n".join(lines) + "\n"

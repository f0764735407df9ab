"""Continuous-batching scheduler over ``Engine`` (the serving loop the reference's engine provides around its
prefill / decode forwards: admission, chunked prefill under a token budget, decode of every running request,
retirement; ``king_v10/bundle_v9/slots.py:225-288`` runs inside such a loop).

``submit(prompt, max_new_tokens, stop)`` queues a request; each ``step()`` either prefills newly admitted requests
(up to ``prefill_tokens`` prompt tokens per step; a prompt longer than the budget is prefilled in chunks over
several steps, every chunk attending to its cached prefix) or decodes one token for every running request (at most
``max_running``, one batch, CUDA-graph bucketed by the engine).  Prefill has priority, as in the reference's
disaggregated prefill role; finished requests release their KV pages at once.  Admission waits for free KV pages
(keeping one page of headroom per running request); when a decode step would run out of pages, the youngest
requests are preempted by recompute: their pages are freed, they rejoin the queue first and, on readmission,
prefill their prompt plus the tokens they already generated (a prefix-cache hit when enabled) and continue.
With DP owner-only KV the same loop budgets pages per home rank (each request's home: the rank with the most free
pages at admission).  Greedy sampling, or temperature /
top-k sampling with a per-request seed.  On several ranks every rank runs the same scheduler on the same
submissions (SPMD), so all ranks take the same steps.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence

import torch

from .engine import Engine, Request


@dataclass
class Job:
    jid: int
    prompt: List[int]
    max_new_tokens: int
    stop: Sequence[int] = ()
    temperature: float = 0.0
    top_k: int = 0
    seed: int = 0
    req: Optional[Request] = None
    out: List[int] = field(default_factory=list)
    pending: Optional[int] = None          # sampled token not yet fed to the model
    done: bool = False
    admit: int = -1                        # admission order (preemption retracts the youngest first)

    def tokens(self) -> List[int]:
        """Tokens to prefill on (re)admission: the prompt, plus, after a preemption, every output token already fed
        to the model (the last sampled one is still pending)."""
        return self.prompt + self.out[:-1]

    def sample(self, logits: torch.Tensor) -> int:
        if self.temperature <= 0.0:
            return int(torch.argmax(logits.float()))
        lg = logits.float().cpu() / self.temperature
        if self.top_k > 0:
            v, i = torch.topk(lg, min(self.top_k, lg.numel()))
            lg = torch.full_like(lg, float("-inf")).scatter_(0, i, v)
        g = torch.Generator().manual_seed(self.seed * 1000003 + len(self.out))
        return int(torch.multinomial(torch.softmax(lg, -1), 1, generator=g))


class Scheduler:
    def __init__(self, engine: Engine, max_running: int = 256, prefill_tokens: int = 32768, heartbeat=None,
                 watchdog=None, check_device: bool = False):
        """heartbeat (``utils.health.Heartbeat``): checked before every step, so a dead peer stops this rank before
        it launches work that would wait for it; watchdog (``utils.health.Watchdog``): a step that overruns its
        limit raises ``StepStalled``; check_device: read the cross-rank kernels' status word after every step."""
        self.eng = engine
        # Owner-only KV: each admitted request gets a home rank (the one with the most free
        # pages), pages are budgeted per home rank, and preemption picks its victims among the requests of the
        # rank that runs short.  Every rank computes the same decisions.
        self.owner = bool(getattr(engine, "owner_kv", False))
        self.world = engine.model.pctx.world
        self.heartbeat = heartbeat
        self.watchdog = watchdog
        self.check_device = check_device
        self.max_running = max_running
        self.prefill_tokens = prefill_tokens
        self.waiting: Deque[Job] = deque()
        self.prefilling: List[Job] = []        # admitted, prompt partly cached (chunked prefill)
        self.running: List[Job] = []
        self.finished: Dict[int, Job] = {}
        self.jobs: Dict[int, Job] = {}         # submitted, not yet finished (a job's ``out`` grows token by token)
        self._next = 0
        self._admits = 0
        self.preemptions = 0
        self.steps = {"prefill": 0, "decode": 0}

    def submit(self, prompt: Sequence[int], max_new_tokens: int, stop: Sequence[int] = (), temperature: float = 0.0,
               top_k: int = 0, seed: int = 0) -> int:
        cap = (self.eng.cache.alloc.num_pages() - 1) * self.eng.page_size       # page 0 is the graphs' scratch
        if len(prompt) + max_new_tokens > cap:
            raise ValueError(f"prompt + max_new_tokens = {len(prompt) + max_new_tokens} tokens exceed the KV cache "
                             f"({cap} tokens)")
        j = Job(self._next, list(prompt), max_new_tokens, tuple(stop), temperature, top_k, seed)
        self._next += 1
        self.waiting.append(j)
        self.jobs[j.jid] = j
        return j.jid

    def idle(self) -> bool:
        return not (self.waiting or self.prefilling or self.running)

    def _finish(self, j: Job):
        j.done = True
        self.eng.release(j.req)
        self.finished[j.jid] = j
        self.jobs.pop(j.jid, None)

    def _take(self, j: Job, tok: int):
        """Record a sampled token; retire the job when it is complete."""
        j.out.append(tok)
        if len(j.out) >= j.max_new_tokens or tok in j.stop:
            self._finish(j)
        else:
            j.pending = tok
            self.running.append(j)

    def step(self) -> None:
        if self.heartbeat is not None:
            self.heartbeat.check()
        if self.watchdog is None:
            self._step()
        else:
            with self.watchdog.step("scheduler step"):
                self._step()
        if self.check_device:
            self.eng.check_device()

    def _retract(self, j: Job) -> None:
        """Preempt by recompute: free the job's KV pages and queue it first; on readmission it prefills its prompt
        and the tokens it already generated, then continues from its pending token."""
        self.eng.release(j.req)
        j.req = None
        (self.running if j in self.running else self.prefilling).remove(j)
        self.waiting.appendleft(j)
        self.preemptions += 1

    def _step(self) -> None:
        eng = self.eng
        # page budgets: one domain, or (owner-only KV) one per home rank, computed identically on every rank
        doms = self.world if self.owner else 1

        def dom(req) -> int:
            return req.home if self.owner else 0

        def avail(h: int) -> int:
            return eng.pages_available(h) if self.owner else eng.pages_available()

        budget = self.prefill_tokens
        reserve = [0] * doms                        # headroom: one new page per running decode
        for j in self.running:
            reserve[dom(j.req)] += 1
        committed = [0] * doms
        batch: List[Job] = []
        counts: List[int] = []
        # continue chunked prefills first, then admit new requests while the token budget, the batch size and the
        # free KV pages allow
        for j in list(self.prefilling):
            if budget <= 0:
                break
            n = min(budget, j.req.seq_len - j.req.n_cached)
            h = dom(j.req)
            need = eng.pages_for(j.req, j.req.n_cached + n)
            if need > avail(h) - reserve[h] - committed[h]:
                break
            committed[h] += need
            batch.append(j)
            counts.append(n)
            budget -= n
        while self.waiting and budget > 0 and len(self.running) + len(self.prefilling) + 1 <= self.max_running:
            j = self.waiting[0]
            req = eng.add_request(j.tokens())
            if self.owner:                          # home: the rank with the most free pages
                free = [avail(h) - reserve[h] - committed[h] for h in range(doms)]
                req.home = max(range(doms), key=lambda h: (free[h], -h))
            h = dom(req)
            n = min(budget, req.seq_len - req.n_cached)     # a cached prefix (prefix reuse) is skipped
            need = eng.pages_for(req, req.n_cached + n)
            if need > avail(h) - reserve[h] - committed[h]:
                eng.release(req)                            # give back the shared prefix pages
                break
            self.waiting.popleft()
            j.req, j.admit = req, self._admits
            self._admits += 1
            committed[h] += need
            self.prefilling.append(j)
            batch.append(j)
            counts.append(n)
            budget -= n
        if batch:
            self.steps["prefill"] += 1
            whole = all(j.req.n_cached == 0 and n == j.req.seq_len for j, n in zip(batch, counts))
            if whole:
                logits = eng.prefill([j.req for j in batch])
            else:
                if eng.cfg.late_layer_start >= 0:
                    for j in batch:
                        if j.req.n_cached == 0:
                            j.req.late_from = max(0, j.req.seq_len - eng.cfg.late_replay)
                logits = eng._prefill_rows([j.req for j in batch], counts)
            for j, row in zip(batch, logits):
                if j.req.n_cached == j.req.seq_len:             # prompt complete
                    self.prefilling.remove(j)
                    if j.out:                                   # resumed after a preemption: already sampled
                        j.pending = j.out[-1]
                        self.running.append(j)
                    else:
                        self._take(j, j.sample(row))
            return
        if not self.running:
            if len(self.prefilling) > 1:            # chunked prefills that cannot all fit: retract the youngest
                self._retract(max(self.prefilling, key=lambda j: j.admit))
                return
            if self.waiting or self.prefilling:
                raise RuntimeError("KV cache too small for the next request")
            return
        # decode every running job; where a domain's pages for this step are short, preempt its youngest jobs
        oldest = min(self.running, key=lambda j: j.admit)           # always keeps making progress
        for h in range(doms):
            while True:
                need = sum(eng.pages_for(j.req, j.req.seq_len + 1) for j in self.running if dom(j.req) == h)
                if need <= avail(h):
                    break
                victims = sorted((j for j in self.running + self.prefilling if dom(j.req) == h and j is not oldest),
                                 key=lambda j: -j.admit)
                if not victims:
                    raise RuntimeError("KV cache too small for the running request")
                self._retract(victims[0])
        self.steps["decode"] += 1
        run, self.running = self.running, []
        logits = eng.decode([j.req for j in run], [j.pending for j in run])
        for j, row in zip(run, logits):
            self._take(j, j.sample(row))

    def run(self) -> Dict[int, List[int]]:
        """Step until every submitted job finished; returns {job id: output tokens}."""
        while not self.idle():
            self.step()
        return {jid: j.out for jid, j in self.finished.items()}

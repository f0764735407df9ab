"""Prefill/decode disaggregation: a prefill engine hands finished prompts' KV to a decode engine.

The reference serves DeepSeek-V4.1 with separate prefill and decode engines (role from
``get_disagg().disaggregation_mode``, ``king_v10/bundle_v9/slots.py:274-285``; KV moved by the engine's transport).
Here the handoff is point-to-point ``torch.distributed`` send/recv (NCCL over NVLink between GPUs, gloo on CPU):

* ``PrefillRole.submit(prompts)`` runs one prefill step, samples each request's first token and ships, per request,
  a header (prompt length, first token) and the per-layer latent rows (plus indexer key rows) of its tokens.  The
  sends are issued with ``isend`` from a side CUDA stream, so the transfer of batch i overlaps the prefill of
  batch i+1; ``flush()`` waits for them.
* ``DecodeRole.receive(n)`` allocates pages in its own paged cache, posts every receive of the batch at once
  (``irecv`` on a side stream), scatters the rows into the pages and returns requests ready for ``Engine.decode``.
  Slot lists come from the page tables on the device (no per-token host loop).

Both roles must post the same number of requests in the same order (the transport has no reordering).
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from .engine import Engine, Request


def request_slots(eng: Engine, r: Request, n: int) -> torch.Tensor:
    """Cache slots of the first ``n`` tokens of ``r`` (its page table expanded on the device, no per-token loop)."""
    ps = eng.page_size
    pages = torch.tensor(r.pages, dtype=torch.int64).to(eng.device, non_blocking=True)
    pos = torch.arange(n, device=eng.device)
    return pages[pos // ps] * ps + pos % ps


def _cache_tensors(eng: Engine):
    """The per-layer cache tensors a handoff carries: latent rows of every layer, then the indexer keys of the
    layers that run the indexer."""
    return list(eng.cache.latent), [c for c in eng.cache.index_k if c is not None]


class PrefillRole:
    def __init__(self, engine: Engine, decode_rank: int, group=None):
        self.eng, self.peer, self.group = engine, decode_rank, group
        self._pending = []
        self.side = torch.cuda.Stream() if engine.device.type == "cuda" else None

    def submit(self, prompts: List[List[int]]) -> List[int]:
        """Prefill one batch and ship it: per request a header (prompt length, first token), the latent rows
        [layers, n, width] and the indexer keys [indexer layers, n, d], each gathered straight into one send buffer
        (one index_select per layer, no stacking copy)."""
        eng = self.eng
        reqs = [eng.add_request(p) for p in prompts]
        logits = eng.prefill(reqs)
        first = torch.argmax(logits.float(), dim=-1)
        lat, idx = _cache_tensors(eng)
        for r, t in zip(reqs, first.tolist()):
            n = len(r.prompt)
            slots = request_slots(eng, r, n)
            payload = [torch.empty(len(lat), n, lat[0].shape[1], dtype=lat[0].dtype, device=eng.device)]
            for l, c in enumerate(lat):
                torch.index_select(c, 0, slots, out=payload[0][l])
            if idx:
                payload.append(torch.empty(len(idx), n, idx[0].shape[1], dtype=idx[0].dtype, device=eng.device))
                for l, c in enumerate(idx):
                    torch.index_select(c, 0, slots, out=payload[1][l])
            hdr = torch.tensor([n, t], dtype=torch.int64).to(eng.device if self.side else "cpu")
            if self.side is not None:
                self.side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(self.side):
                    works = [dist.isend(hdr, self.peer, group=self.group)]
                    works += [dist.isend(x, self.peer, group=self.group) for x in payload]
                for x in payload + [hdr]:
                    x.record_stream(self.side)
                self._pending.append((works, payload, hdr))
            else:
                dist.send(hdr, self.peer, group=self.group)
                for x in payload:
                    dist.send(x, self.peer, group=self.group)
            eng.release(r)
        return first.tolist()

    def flush(self):
        for works, _, _ in self._pending:
            for w in works:
                w.wait()
        self._pending = []


class DecodeRole:
    def __init__(self, engine: Engine, prefill_rank: int, group=None):
        self.eng, self.peer, self.group = engine, prefill_rank, group
        self.side = torch.cuda.Stream() if engine.device.type == "cuda" else None

    def receive(self, n_requests: int, prompts: List[List[int]]) -> (List[Request], List[int]):
        """Receive ``n_requests`` handoffs (the router that sent them knows the prompts, so every buffer can be
        sized in advance).  Pages are allocated and every receive of the batch is posted at once (``irecv`` on a side
        stream), then each request's rows are scattered into its pages."""
        eng = self.eng
        dev = eng.device
        lat, idx = _cache_tensors(eng)
        reqs, bufs, works = [], [], []
        cur = torch.cuda.current_stream() if self.side is not None else None
        if self.side is not None:
            self.side.wait_stream(cur)
        for i in range(n_requests):
            n = len(prompts[i])
            r = eng.add_request(prompts[i])
            eng._ensure_pages(r, n)
            hdr = torch.empty(2, dtype=torch.int64, device=dev if dev.type == "cuda" else "cpu")
            b = [hdr, torch.empty(len(lat), n, lat[0].shape[1], dtype=lat[0].dtype, device=dev)]
            if idx:
                b.append(torch.empty(len(idx), n, idx[0].shape[1], dtype=idx[0].dtype, device=dev))
            if self.side is not None:
                with torch.cuda.stream(self.side):
                    works += [dist.irecv(x, self.peer, group=self.group) for x in b]
            else:
                for x in b:
                    dist.recv(x, self.peer, group=self.group)
            reqs.append(r)
            bufs.append(b)
        for w in works:
            w.wait()
        if self.side is not None:
            cur.wait_stream(self.side)
        first = []
        for r, b in zip(reqs, bufs):
            n, t = (int(v) for v in b[0].tolist())
            assert len(r.prompt) == n, "handoff length mismatch"
            slots = request_slots(eng, r, n)
            for l, c in enumerate(lat):
                c.index_copy_(0, slots, b[1][l])
            for l, c in enumerate(idx):
                c.index_copy_(0, slots, b[2][l])
            r.n_cached = n
            first.append(t)
        return reqs, first

    def generate(self, reqs: List[Request], first: List[int], max_new_tokens: int) -> List[List[int]]:
        eng = self.eng
        outs = [[t] for t in first]
        nxt = first
        for _ in range(max_new_tokens - 1):
            logits = eng.decode(reqs, nxt)
            nxt = torch.argmax(logits.float(), dim=-1).tolist()
            for o, t in zip(outs, nxt):
                o.append(t)
        for r in reqs:
            eng.release(r)
        return outs

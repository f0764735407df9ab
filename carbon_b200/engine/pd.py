"""Prefill/decode disaggregation: a prefill engine hands finished prompts' KV to a decode engine.

The reference serves DeepSeek-V4.1 with separate prefill and decode engines (role from
``get_disagg().disaggregation_mode``, ``king_v10/bundle_v9/slots.py:274-285``; KV moved by the engine's transport).
Here the handoff is point-to-point ``torch.distributed`` send/recv (NCCL over NVLink between GPUs, gloo on CPU):

* ``PrefillRole.submit(prompts)`` runs one prefill step, samples each request's first token and ships, per request,
  a header (prompt length, first token) and the per-layer latent rows (plus indexer key rows) of its tokens.  The
  sends are issued with ``isend`` from a side CUDA stream, so the transfer of batch i overlaps the prefill of
  batch i+1; ``flush()`` waits for them.
* ``DecodeRole.receive(n)`` allocates pages in its own paged cache, receives the rows straight into them and
  returns requests ready for ``Engine.decode``.

Both roles must post the same number of requests in the same order (the transport has no reordering).
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from .engine import Engine, Request


def _gather_rows(cache_t: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
    return cache_t.index_select(0, slots.long())


class PrefillRole:
    def __init__(self, engine: Engine, decode_rank: int, group=None):
        self.eng, self.peer, self.group = engine, decode_rank, group
        self._pending = []
        self.side = torch.cuda.Stream() if engine.device.type == "cuda" else None

    def submit(self, prompts: List[List[int]]) -> List[int]:
        eng = self.eng
        reqs = [eng.add_request(p) for p in prompts]
        logits = eng.prefill(reqs)
        first = torch.argmax(logits.float(), dim=-1)
        for r, t in zip(reqs, first.tolist()):
            n = len(r.prompt)
            slots = torch.tensor([r.pages[p // eng.page_size] * eng.page_size + p % eng.page_size for p in range(n)],
                                 dtype=torch.int64, device=eng.device)
            payload = [torch.stack([_gather_rows(c, slots) for c in eng.cache.latent])]
            idx_layers = [c for c in eng.cache.index_k if c is not None]     # layers that run the indexer
            if idx_layers:
                payload.append(torch.stack([_gather_rows(c, slots) for c in idx_layers]))
            hdr = torch.tensor([n, t], dtype=torch.int64, device=eng.device if self.side else "cpu")
            if self.side is not None:
                self.side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(self.side):
                    works = [dist.isend(hdr, self.peer, group=self.group)]
                    works += [dist.isend(x.contiguous(), self.peer, group=self.group) for x in payload]
                self._pending.append((works, payload, hdr))
            else:
                dist.send(hdr, self.peer, group=self.group)
                for x in payload:
                    dist.send(x.contiguous(), self.peer, group=self.group)
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

    def receive(self, n_requests: int, prompts: List[List[int]]) -> (List[Request], List[int]):
        """Receive ``n_requests`` handoffs (prompt token ids are known to the router that sent them)."""
        eng = self.eng
        cfg = eng.cfg
        reqs, first = [], []
        dev = eng.device
        for i in range(n_requests):
            hdr = torch.empty(2, dtype=torch.int64, device=dev if dev.type == "cuda" else "cpu")
            dist.recv(hdr, self.peer, group=self.group)
            n, t = int(hdr[0]), int(hdr[1])
            r = eng.add_request(prompts[i])
            assert len(r.prompt) == n, "handoff length mismatch"
            eng._ensure_pages(r, n)
            slots = torch.tensor([r.pages[p // eng.page_size] * eng.page_size + p % eng.page_size for p in range(n)],
                                 dtype=torch.int64, device=dev)
            lat = torch.empty(cfg.n_layers, n, eng.cache.latent[0].shape[1], dtype=eng.cache.latent[0].dtype,
                              device=dev)
            dist.recv(lat, self.peer, group=self.group)
            for l, c in enumerate(eng.cache.latent):
                c.index_copy_(0, slots, lat[l])
            idx_layers = [c for c in eng.cache.index_k if c is not None]
            if idx_layers:
                ik = torch.empty(len(idx_layers), n, idx_layers[0].shape[1], dtype=idx_layers[0].dtype, device=dev)
                dist.recv(ik, self.peer, group=self.group)
                for l, c in enumerate(idx_layers):
                    c.index_copy_(0, slots, ik[l])
            r.n_cached = n
            reqs.append(r)
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

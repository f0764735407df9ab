"""Draft proposers for speculative decoding.

The reference verifies 6 rows per request per decode step against drafts from its "DSpark" draft model
(``king_v10/bundle_v9/dec/gemm_tables.py:51``, ``dspd_w22/dspd/mlp.py:1-10``).  The verify side is
``Engine.verify``; any object with ``propose(tokens, n) -> list[int]`` can draft.  ``NgramDrafter`` is the
weight-free prompt-lookup drafter: it finds the most recent earlier occurrence of the sequence's last n-gram and
proposes the tokens that followed it.  ``ModelDrafter`` runs a draft model (its own engine) greedily.
"""
from __future__ import annotations

from typing import List, Sequence


class NgramDrafter:
    def __init__(self, max_ngram: int = 3, min_ngram: int = 1):
        self.max_ngram, self.min_ngram = max_ngram, min_ngram

    def propose(self, tokens: Sequence[int], n: int) -> List[int]:
        toks = list(tokens)
        L = len(toks)
        for g in range(min(self.max_ngram, L - 1), self.min_ngram - 1, -1):
            key = toks[L - g:]
            for start in range(L - g - 1, -1, -1):
                if toks[start:start + g] == key:
                    cont = toks[start + g:start + g + n]
                    if cont:
                        return cont
        return []


class ModelDrafter:
    """Draft-model proposer: a smaller model (its own ``Engine``) continues the sequence greedily for ``n`` tokens.
    Give the draft engine ``prefix_cache=True``: every call then shares the cached pages of the sequence so far and
    prefills only the tokens accepted since the previous call, instead of the whole sequence."""

    def __init__(self, engine):
        self.eng = engine

    def propose(self, tokens: Sequence[int], n: int) -> List[int]:
        if n <= 0 or not tokens:
            return []
        import torch

        r = self.eng.add_request(list(tokens))
        try:
            out = []
            logits = self.eng.prefill([r])
            for _ in range(n):
                t = int(torch.argmax(logits[0].float()))
                out.append(t)
                if len(out) == n:
                    break
                logits = self.eng.decode([r], [t])
            return out
        finally:
            self.eng.release(r)

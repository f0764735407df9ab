"""Prefix cache: KV pages of earlier prompts reused by later requests that start with the same tokens.

Full pages of a prefilled prompt are keyed by the hash chain of their tokens (page i's key covers tokens
[0, (i+1) * page_size), so equal keys mean equal prefixes) and held by the cache with one reference each in the
ref-counted page allocator.  A new request takes the longest chain of cached full pages of its prompt (always leaving
at least one prompt token to run, which produces the request's first logits), shares those pages, and prefills only
the rest with per-row attention over its cached prefix.  Pages a request shares are never written again: its own new
tokens land in later pages.  When the allocator runs out of pages the least recently used entries are released.
The serving engine around the reference keeps such a cache (radix prefix reuse); the bundles assume it.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import List, Sequence, Tuple


class PrefixCache:
    def __init__(self, alloc, page_size: int):
        self.alloc = alloc
        self.page_size = page_size
        self.entries: "OrderedDict[Tuple, int]" = OrderedDict()     # chain key -> page (LRU order)
        self.hits_tokens = 0

    def _keys(self, tokens: Sequence[int], n_pages: int) -> List[Tuple]:
        keys, prev, ps = [], (), self.page_size
        for i in range(n_pages):
            prev = (hash(prev), tuple(tokens[i * ps:(i + 1) * ps]))
            keys.append(prev)
        return keys

    def match(self, prompt: Sequence[int]) -> List[int]:
        """Pages of the longest cached prefix of ``prompt`` (full pages, leaving at least one token); each returned
        page has one more reference, owned by the caller."""
        n = (len(prompt) - 1) // self.page_size
        pages = []
        for key in self._keys(prompt, n):
            p = self.entries.get(key)
            if p is None:
                break
            self.entries.move_to_end(key)
            pages.append(p)
        if pages:
            self.alloc.share(pages)
            self.hits_tokens += len(pages) * self.page_size
        return pages

    def insert(self, prompt: Sequence[int], pages: Sequence[int]) -> None:
        """Register the full pages of a prefilled prompt (the cache takes one reference to each new entry)."""
        n = min(len(prompt) // self.page_size, len(pages))
        for key, p in zip(self._keys(prompt, n), pages[:n]):
            if key in self.entries:
                self.entries.move_to_end(key)
                continue
            self.alloc.share([p])
            self.entries[key] = p

    def evict(self, n_pages: int) -> int:
        """Release up to ``n_pages`` least recently used entries; returns how many were released."""
        k = 0
        while self.entries and k < n_pages:
            _, p = self.entries.popitem(last=False)
            self.alloc.free([p])
            k += 1
        return k

    def clear(self) -> None:
        self.evict(len(self.entries))

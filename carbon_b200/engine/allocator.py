"""KV page allocator: the native C++ ``BlockAllocator`` (``csrc/runtime.cpp``).

A pure-Python twin with identical semantics exists only so that host-side tests can run in a checkout whose
extension has not been built; ``native()`` reports which one is in use.
"""
from __future__ import annotations

from typing import List


class _PyBlockAllocator:
    def __init__(self, num_pages: int):
        self._refs = [0] * num_pages
        self._free = list(range(num_pages - 1, -1, -1))

    def alloc(self, n: int) -> List[int]:
        if n > len(self._free):
            raise RuntimeError("KV cache out of pages")
        out = [self._free.pop() for _ in range(n)]
        for p in out:
            self._refs[p] = 1
        return out

    def share(self, pages):
        for p in pages:
            if self._refs[p] <= 0:
                raise RuntimeError("share of a free page")
            self._refs[p] += 1

    def free(self, pages):
        for p in pages:
            if self._refs[p] <= 0:
                raise RuntimeError("double free of a KV page")
            self._refs[p] -= 1
            if self._refs[p] == 0:
                self._free.append(p)

    def num_free(self) -> int:
        return len(self._free)

    def num_pages(self) -> int:
        return len(self._refs)

    def refcount(self, p: int) -> int:
        return self._refs[p]


def native() -> bool:
    from ..ops._ext import available

    return available()


def BlockAllocator(num_pages: int):
    if native():
        from ..ops._ext import ext

        return ext().BlockAllocator(num_pages)
    return _PyBlockAllocator(num_pages)

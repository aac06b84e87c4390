"""Paged-KV block allocator: a free list of fixed-size KV blocks and per-slot block lists.

The native C++ allocator (csrc/host_runtime.cpp, module `_host`) is used when it is built; this pure-Python
class has the same interface and is the fallback on machines without the host extension (the allocator is
host-side bookkeeping only: it never touches device memory).
"""
from __future__ import annotations


class PyBlockAllocator:
    def __init__(self, n_blocks: int, n_slots: int):
        self.free = list(range(n_blocks - 1, -1, -1))
        self.owned = [[] for _ in range(n_slots)]
        self.n_blocks = n_blocks

    def n_free(self) -> int:
        return len(self.free)

    def n_blocks_of(self, slot: int) -> int:
        return len(self.owned[slot])

    def blocks_of(self, slot: int) -> list:
        return list(self.owned[slot])

    def allocate(self, slot: int, n: int) -> list:
        if n > len(self.free):
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {len(self.free)} free")
        got = [self.free.pop() for _ in range(n)]
        self.owned[slot].extend(got)
        return got

    def release(self, slot: int) -> int:
        n = len(self.owned[slot])
        self.free.extend(reversed(self.owned[slot]))
        self.owned[slot] = []
        return n

    def truncate(self, slot: int, n_keep: int) -> int:
        """Free the slot's blocks beyond the first n_keep (returns how many were freed)."""
        extra = self.owned[slot][n_keep:]
        self.owned[slot] = self.owned[slot][:n_keep]
        self.free.extend(reversed(extra))
        return len(extra)


def BlockAllocator(n_blocks: int, n_slots: int):
    try:
        from .. import _host
        return _host.BlockAllocator(n_blocks, n_slots)
    except ImportError:
        return PyBlockAllocator(n_blocks, n_slots)

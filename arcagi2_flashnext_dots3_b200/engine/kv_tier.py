"""Pinned-host KV tier: idle sequences' caches move to host memory and come back intact, so a session evicted to
make room resumes without recomputing its context.

The reference keeps most of its D3 latent KV in pinned host memory (dotsnote/engine/arcstats_pkg/arcstats/
sparse_offload.py:1051-1350: a device row cache in front of host rows, filled on demand over PCIe) because an
L4 has 24 GB. A B200's 180 GB holds the benchmarked contexts, so here the host tier serves a different limit:
the number of sessions a solver keeps open between turns. The unit is the whole sequence state:

* its paged attention blocks (FN: ``k`` and ``v``; D3: ``latent``), gathered on the device and copied once
  into free host blocks, and copied back into newly allocated device blocks (the block table is rewritten in the
  same logical order);
* its per-slot state rows (FN: recurrent GDN states, conv windows, compressed-key and ring buffers, PLE and
  token histories; D3: DSA index keys), copied whole.

:class:`..engine.scheduler.Scheduler` offloads an idle session here before dropping it, and restores it into a
free slot when the session is pushed again.
"""
from __future__ import annotations

import dataclasses

import torch

PAGED = ("k", "v", "latent")


class HostKVTier:
    def __init__(self, llm, host_blocks: int, pin: bool = None):
        self.llm = llm
        c = llm.caches
        pin = (llm.device.type == "cuda") if pin is None else pin
        self.pools = [t for name in PAGED for t in (getattr(c, name, None) or []) if t is not None]
        self.host = [torch.empty((host_blocks,) + tuple(t.shape[1:]), dtype=t.dtype, pin_memory=pin)
                     for t in self.pools]
        S = c.block_table.shape[0]
        self.slot_state = []
        for f in dataclasses.fields(c):
            if f.name in PAGED or f.name == "block_table":
                continue
            v = getattr(c, f.name)
            items = v if isinstance(v, list) else [v]
            self.slot_state += [t for t in items if torch.is_tensor(t) and t.dim() >= 1 and t.shape[0] == S]
        self.free = list(range(host_blocks - 1, -1, -1))
        self.saved = {}
        self.stats = {"offloaded": 0, "restored": 0, "bytes_out": 0, "bytes_in": 0}

    @property
    def free_blocks(self) -> int:
        return len(self.free)

    def offload(self, key, slot: int) -> bool:
        """Move slot's blocks and state to host memory under `key` and free its device blocks. False (nothing
        changed) when the host tier lacks room."""
        llm = self.llm
        blocks = llm.alloc.blocks_of(slot)
        if len(blocks) > len(self.free) or key in self.saved:
            return False
        hb = [self.free.pop() for _ in blocks]
        dev_idx = torch.tensor(blocks, dtype=torch.long, device=llm.device)
        host_idx = torch.tensor(hb, dtype=torch.long)
        moved = 0
        for dpool, hpool in zip(self.pools, self.host):
            rows = dpool.index_select(0, dev_idx).cpu()
            hpool.index_copy_(0, host_idx, rows)
            moved += rows.numel() * rows.element_size()
        state = [t[slot].to("cpu", copy=True) for t in self.slot_state]
        moved += sum(s.numel() * s.element_size() for s in state)
        self.saved[key] = (hb, state)
        llm.alloc.release(slot)
        self.stats["offloaded"] += 1
        self.stats["bytes_out"] += moved
        return True

    def restore(self, key, slot: int):
        """Bring `key` back into `slot`: new device blocks in the saved logical order, state rows copied back."""
        llm = self.llm
        hb, state = self.saved.pop(key)
        have = llm.alloc.n_blocks_of(slot)
        if have:
            llm.alloc.release(slot)
        new = llm.alloc.allocate(slot, len(hb))
        llm.caches.block_table[slot, :len(new)] = torch.tensor(new, dtype=torch.int32, device=llm.device)
        dev_idx = torch.tensor(new, dtype=torch.long, device=llm.device)
        host_idx = torch.tensor(hb, dtype=torch.long)
        moved = 0
        for dpool, hpool in zip(self.pools, self.host):
            rows = hpool.index_select(0, host_idx)
            dpool.index_copy_(0, dev_idx, rows.to(llm.device))
            moved += rows.numel() * rows.element_size()
        for t, s in zip(self.slot_state, state):
            t[slot].copy_(s.to(llm.device))
            moved += s.numel() * s.element_size()
        self.free.extend(hb)
        self.stats["restored"] += 1
        self.stats["bytes_in"] += moved

    def drop(self, key):
        if key in self.saved:
            self.free.extend(self.saved.pop(key)[0])

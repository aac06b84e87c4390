"""Single-GPU emulation of one rank of a W-way tensor-parallel D3 deployment (memory studies).

The reference's fake_tp.py (dotsnote/engine/arcstats_pkg/arcstats/fake_tp.py) runs one vLLM worker as rank 0
of a W-way group on one GPU so the memory footprint of a real rank (weights, KV, workspaces, their allocation
order) can be reproduced locally, with local stand-ins for the collectives. Here the same holds for this
framework's TP: :func:`fake_rank_model` builds rank 0's weights and caches at their TP-W shapes
(``tp_config`` + ``random_engine(tp=(0, W))``), and :class:`FakeTPGroup` takes the place of
:class:`.tp.TPGroup`. It allocates buffers of the fused path's size and answers every collective locally: an
all-reduce adds this rank's partial only, and the vocabulary pick sees only rank 0's slice. The model runs at
the right shapes and sizes, so step time and memory are those of a rank; its outputs are not the full model's.
"""
from __future__ import annotations

import torch


class FakeTPGroup:
    """Stand-in for :class:`.tp.TPGroup` as rank 0 of `world` ranks, on one device, with no other process."""
    fake = True

    def __init__(self, world: int, device, max_tokens: int, hidden: int, buffers: bool = True):
        self.rank, self.world = 0, world
        self.device = torch.device(device)
        self.H, self.max_tokens = hidden, max_tokens
        self.slot = max_tokens * hidden
        self.group = None
        self.comm = "fake"
        # the fused path's symmetric buffers (two parity slots x world partials, flags), so the footprint matches
        self.buf = torch.zeros(2, world, self.slot, dtype=torch.float32, device=self.device) if buffers else None
        self.flags = torch.zeros(2, world, dtype=torch.int64, device=self.device) if buffers else None

    def allreduce_add(self, h: torch.Tensor, partial: torch.Tensor):
        if partial.shape[0] > self.max_tokens:
            raise ValueError(f"{partial.shape[0]} rows > TP buffer capacity {self.max_tokens}")
        h += partial

    def linear_allreduce_add(self, model, x16, ws, h):
        self.allreduce_add(h, model._mm(x16, ws))

    def sharded_pick(self, local_logits, v0, temperature=0.0, seed=0, step=0):
        """Greedy pick over this rank's vocabulary slice only (token ids offset by the slice start)."""
        return (local_logits.float().argmax(-1) + v0).to(torch.int32)


def fake_rank_model(cfg, world: int, device, n_slots: int, max_len: int, block_size: int = 64, seed: int = 0,
                    shard_vocab: bool = False, max_tokens: int = 64):
    """Rank 0 of a TP-`world` D3 model on one device: (model, weights, caches, group). Weights are random with
    the shapes of that rank's shard; caches hold the rank's heads for n_slots sequences of max_len tokens."""
    from ..models import d3_weights
    from ..models.d3 import D3Model, allocate_caches
    from .tp import tp_config
    dev = torch.device(device)
    rcfg = tp_config(cfg, world)
    W = d3_weights.random_engine(cfg, dev, seed=seed, tp=(0, world), shard_vocab=shard_vocab)
    caches = allocate_caches(rcfg, dev, n_slots, max_len, block_size=block_size)
    grp = FakeTPGroup(world, dev, max_tokens, cfg.hidden_size)
    return D3Model(rcfg, W, caches, dev, tp=grp), W, caches, grp

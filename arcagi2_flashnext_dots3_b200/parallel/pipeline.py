"""Pipeline parallelism for the repair-training student: contiguous layer ranges on consecutive ranks, GPipe
schedule over micro-batches (one rollout sequence each), activations and their gradients moved by NCCL
point-to-point operations that overlap with the next micro-batch's compute.

The reference trains its students with layers split over GPUs when one replica does not fit
(dotsnote/training/finetune/student.py device maps; the FN RL trainer's model parallel layout,
flashnext/training/rl/train_rl.py:75). Here a stage owns layers [a, b) of :func:`stage_bounds`; stage 0 embeds,
the last stage applies the stream mixer and the objective. One training step:

1. forward, micro-batch by micro-batch: receive the stage input (blocking), run the stage's layers (per-layer
   activation checkpointing), send the output to the next stage asynchronously;
2. backward in reverse micro-batch order: the last stage back-propagates its objective; the others receive the
   gradient of their output and back-propagate it; every stage but the first sends the gradient of its input
   back asynchronously.

Gradients of each stage's trainables are then exactly those of the whole model on the same micro-batches.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch.utils.checkpoint import checkpoint

from ..models import fn_reference as R


def stage_bounds(n_layers: int, world: int) -> list:
    """[(first, end)] contiguous layer ranges, sizes differing by at most one (earlier stages take the extra)."""
    base, extra = divmod(n_layers, world)
    out, a = [], 0
    for r in range(world):
        b = a + base + (1 if r < extra else 0)
        out.append((a, b))
        a = b
    return out


class PipelineStage:
    def __init__(self, cfg, W: dict, device, rank: int, world: int, group=None, train_norms: bool = False):
        from ..training.student import FNStudent
        if world > cfg.num_layers:
            raise ValueError("more pipeline stages than layers")
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.a, self.b = stage_bounds(cfg.num_layers, world)[rank]
        Ws = {k: v for k, v in W.items() if k != "layers"}
        Ws["layers"] = W["layers"][self.a:self.b]
        self.student = FNStudent(cfg, Ws, device, train_norms=train_norms, layer_offset=self.a)
        self.device = self.student.device
        self.first, self.last = rank == 0, rank == world - 1
        self._peer = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)

    def parameters(self):
        return self.student.parameters()

    def forward_stage(self, ids: torch.Tensor, h_in: torch.Tensor = None, ckpt: bool = True) -> torch.Tensor:
        cfg, st = self.cfg, self.student
        W = st.W
        ids = ids.to(self.device)
        T = ids.shape[0]
        cos, sin = R.rope_cos_sin(torch.arange(T), cfg.rope_dim, cfg.rope_theta)
        cos, sin = cos.to(self.device), sin.to(self.device)
        h = W["embed"][ids].float().repeat(1, cfg.hc_count) if self.first else h_in
        emb = R.ple_embed(ids, W, cfg) if cfg.ple_layers else None
        for l in range(self.b - self.a):
            if ckpt and torch.is_grad_enabled():
                h = checkpoint(st._layer, l, h, emb, cos, sin, use_reentrant=False)
            else:
                h = st._layer(l, h, emb, cos, sin)
        if self.last:
            return R.gated_residual(h, W["mixer"], cfg.hc_count, cfg.hidden_size, cfg.rms_eps, combine=False)
        return h

    def step(self, micro_batches: list, objective, ckpt: bool = True) -> list:
        """One GPipe pass. micro_batches: token id tensors [T_m] (the same list on every stage); objective(model,
        final_hidden, m) -> loss tensor on the last stage. Accumulates gradients into the stage's trainables and
        returns the last stage's losses (floats; empty elsewhere)."""
        width = self.cfg.hc_count * self.cfg.hidden_size
        saved, sends, losses = [], [], []
        for m, ids in enumerate(micro_batches):
            h_in = None
            if not self.first:
                h_in = torch.empty(len(ids), width, dtype=torch.float32, device=self.device)
                dist.recv(h_in, src=self._peer(self.rank - 1), group=self.group)
                h_in.requires_grad_(True)
            out = self.forward_stage(ids, h_in, ckpt)
            if self.last:
                loss = objective(self.student, out, m)
                losses.append(float(loss.detach()))
                saved.append((h_in, loss))
            else:
                sends.append(dist.isend(out.detach().contiguous(), dst=self._peer(self.rank + 1), group=self.group))
                saved.append((h_in, out))
        for s in sends:
            s.wait()
        sends = []
        for m in reversed(range(len(micro_batches))):
            h_in, out = saved[m]
            if self.last:
                out.backward()
            else:
                g = torch.empty_like(out)
                dist.recv(g, src=self._peer(self.rank + 1), group=self.group)
                out.backward(g)
            if not self.first:
                sends.append(dist.isend(h_in.grad.contiguous(), dst=self._peer(self.rank - 1), group=self.group))
        for s in sends:
            s.wait()
        return losses

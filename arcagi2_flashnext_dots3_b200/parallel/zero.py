"""Data-parallel training optimizer: gradient reduce-scatter overlapped with backward, sharded Adam.

The reference all-reduces one flat fp32 gradient vector after the whole backward (no overlap,
flashnext/training/rl/train_rl.py:197) and keeps full Adam state on every rank. Here:

* every trainable parameter's ``.grad`` is a view into a flat fp32 bucket (one bucket list per parameter group,
  buckets of at most `bucket_elems`), so autograd accumulates straight into the communication buffer;
* during the LAST backward of an optimizer step, a post-accumulate-grad hook counts the parameters of each
  bucket and launches an async ``reduce_scatter_tensor`` (sum) as soon as the bucket is complete, so the
  reduction of late layers overlaps the backward of early ones;
* each rank keeps fp32 Adam moments only for its 1/world shard of every bucket, updates that shard of the
  parameters and all-gathers the updated values back into the (flat) parameters.

On gloo (CPU tests) there is no reduce-scatter: the bucket is all-reduced and sliced, same result.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


class _Bucket:
    def __init__(self, params, lr, world, device):
        self.params = params
        self.lr = lr
        n = sum(p.numel() for p in params)
        self.n = n
        self.padded = (n + world - 1) // world * world
        self.shard = self.padded // world
        self.grad = torch.zeros(self.padded, dtype=torch.float32, device=device)
        self.flat = torch.zeros(self.padded, dtype=torch.float32, device=device)
        off = 0
        for p in params:
            k = p.numel()
            self.flat[off:off + k].copy_(p.detach().reshape(-1))
            p.data = self.flat[off:off + k].view_as(p)
            p.grad = self.grad[off:off + k].view_as(p)
            off += k
        self.pending = 0
        self.work = None
        self.gshard = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.m = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.v = torch.zeros(self.shard, dtype=torch.float32, device=device)


class ShardedAdam:
    def __init__(self, param_groups, group=None, betas=(0.9, 0.999), eps=1e-8, bucket_elems=1 << 24,
                 overlap: bool = True):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.betas, self.eps = betas, eps
        self.overlap = overlap
        self.step_count = 0
        self.buckets = []
        self.lr_scale = 1.0
        for g in param_groups:
            cur, size = [], 0
            for p in g["params"]:
                if cur and size + p.numel() > bucket_elems:
                    self.buckets.append(_Bucket(cur, g["lr"], self.world, p.device))
                    cur, size = [], 0
                cur.append(p)
                size += p.numel()
            if cur:
                self.buckets.append(_Bucket(cur, g["lr"], self.world, cur[0].device))
        self._owner = {}
        for b in self.buckets:
            for p in b.params:
                self._owner[id(p)] = b
                p.register_post_accumulate_grad_hook(self._hook)
        self.last_backward = False

    # -------------------------------------------------------------------------------------- reduction
    def zero_grad(self):
        for b in self.buckets:
            b.grad.zero_()
            b.pending = 0
            b.work = None

    def _hook(self, p):
        if not (self.overlap and self.last_backward):
            return
        b = self._owner[id(p)]
        b.pending += 1
        if b.pending == len(b.params) and b.work is None:
            self._launch(b, async_op=True)

    def _launch(self, b, async_op):
        if self.world == 1:
            b.gshard.copy_(b.grad[: b.shard])
            b.work = True
            return
        if b.grad.is_cuda:
            b.work = dist.reduce_scatter_tensor(b.gshard, b.grad, group=self.group, async_op=async_op) or True
        else:
            w = dist.all_reduce(b.grad, group=self.group, async_op=async_op)
            b.work = ("slice", w)

    def finish_reduction(self):
        """Wait for (or launch) every bucket's reduction; returns this rank's gradient shards."""
        for b in self.buckets:
            if b.work is None:
                self._launch(b, async_op=False)
        for b in self.buckets:
            w = b.work
            if isinstance(w, tuple):
                if w[1] is not None:
                    w[1].wait()
                b.gshard.copy_(b.grad[self.rank * b.shard:(self.rank + 1) * b.shard])
            elif w is not True and w is not None:
                w.wait()
        return [b.gshard for b in self.buckets]

    def grad_norm(self) -> float:
        sq = sum(float(b.gshard.double().pow(2).sum()) for b in self.buckets)
        if self.world > 1:
            t = torch.tensor([sq], dtype=torch.float64, device=self.buckets[0].flat.device)
            dist.all_reduce(t, group=self.group)
            sq = float(t)
        return math.sqrt(sq)

    # ----------------------------------------------------------------------------------------- update
    @torch.no_grad()
    def step(self, lr_scale: float = 1.0):
        self.finish_reduction()
        self.step_count += 1
        b1, b2 = self.betas
        c1 = 1 - b1 ** self.step_count
        c2 = 1 - b2 ** self.step_count
        for b in self.buckets:
            lo, hi = self.rank * b.shard, (self.rank + 1) * b.shard
            g = b.gshard
            b.m.mul_(b1).add_(g, alpha=1 - b1)
            b.v.mul_(b2).addcmul_(g, g, value=1 - b2)
            upd = (b.m / c1) / ((b.v / c2).sqrt() + self.eps)
            b.flat[lo:hi].add_(upd, alpha=-b.lr * lr_scale)
            if self.world > 1:
                if b.flat.is_cuda:
                    dist.all_gather_into_tensor(b.flat, b.flat[lo:hi].clone(), group=self.group)
                else:
                    parts = list(b.flat.chunk(self.world))
                    dist.all_gather(parts, b.flat[lo:hi].clone(), group=self.group)
        self.last_backward = False

    # ---------------------------------------------------------------------------------------- state
    def state_dict(self):
        return {"step": self.step_count, "rank": self.rank, "world": self.world,
                "m": [b.m.cpu() for b in self.buckets], "v": [b.v.cpu() for b in self.buckets]}

    def load_state_dict(self, sd):
        if sd["world"] != self.world:
            raise ValueError(f"optimizer shard saved for world {sd['world']}, running {self.world}")
        self.step_count = sd["step"]
        for b, m, v in zip(self.buckets, sd["m"], sd["v"]):
            b.m.copy_(m)
            b.v.copy_(v)

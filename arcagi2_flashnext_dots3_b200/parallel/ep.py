"""Expert-parallel MoE across GPUs: in-kernel NVLink dispatch/combine (product path) and an NCCL baseline.

Layout (one process per GPU, `world` ranks): every rank runs its own sequences through the dense parts of the
model (attention, Gated DeltaNet, hyper-connections, shared expert) and owns experts
[rank * E / world, (rank + 1) * E / world). Per MoE layer:

* fused path (``comm="fused"``, csrc/k_ep.cu): route -> stable per-destination plan -> push kernel stores every
  routed token row into its owner's symmetric receive buffer (peer stores) and publishes count + epoch flag ->
  owner waits for all sources, sorts by local expert, runs the grouped gate_up GEMM, and the down GEMM's
  epilogue stores every output row directly into the source's pair buffer on the source GPU -> completion
  flags -> the source waits, then combines locally (weights + shared expert + hyper-connection injection);
* baseline (``comm="nccl"``): the same plan, but rows and outputs move with ``all_to_all_single``.

The reference moves the same data through host memory (EP dispatch = host all-gather with int8 packing,
flashnext/kaggle/code_dataset/fnext/base/q8_dispatch.py:58-86; combine = host reduce-scatter,
fnext/base/q8_rs.py:27) because L4s have no peer-to-peer path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import fn_ops as ops
from ..ops import native, wgemm


class EPGroup:
    """Symmetric buffers, peer address tables and scratch of one rank."""

    def __init__(self, cfg, rank: int, world: int, device, max_tokens: int, group=None, comm: str = "fused",
                 n_tile: int = 16, timeout_ns: int = None):
        if cfg.n_experts % world:
            raise ValueError(f"{cfg.n_experts} experts do not split over {world} ranks")
        self.cfg, self.rank, self.world, self.comm = cfg, rank, world, comm
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.e_loc = cfg.n_experts // world
        self.k = cfg.top_k
        self.H = cfg.hidden_size
        self.max_tokens = max_tokens
        self.cap = max_tokens * self.k            # pairs one source can send to one owner (worst case)
        self.n_tile = n_tile
        self.timeout_ns = timeout_ns or native.DEFAULT_TIMEOUT_NS * 4
        dev, W, H = self.device, world, self.H
        self.max_rows = W * self.cap
        self.max_items = (self.max_rows + n_tile - 1) // n_tile + self.e_loc
        self.dest_slot = torch.zeros(self.cap, dtype=torch.int32, device=dev)
        self.dest_count = torch.zeros(W, dtype=torch.int32, device=dev)
        self.sorted_src = torch.zeros(self.max_rows, dtype=torch.int32, device=dev)
        self.items = torch.zeros(self.max_items, 4, dtype=torch.int32, device=dev)
        self.n_items = torch.zeros(1, dtype=torch.int32, device=dev)
        self.row_dst = torch.zeros(self.max_rows, dtype=torch.int64, device=dev)
        self.n_rows = torch.zeros(1, dtype=torch.int32, device=dev)
        self.xs = torch.zeros(self.max_rows, H, dtype=torch.float16, device=dev)
        self.act = torch.zeros(self.max_rows, cfg.moe_inter, dtype=torch.float16, device=dev)
        self.yout = torch.zeros(self.max_rows, H, dtype=torch.float32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        self.done_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
        if comm == "fused":
            self._alloc_symmetric()
        else:
            self.ybuf = torch.zeros(self.cap, H, dtype=torch.float32, device=dev)

    def _alloc_symmetric(self):
        import torch.distributed._symmetric_memory as symm
        W, H, dev = self.world, self.H, self.device

        def alloc(shape, dtype):
            t = symm.empty(*shape, dtype=dtype, device=dev)
            t.zero_()
            h = symm.rendezvous(t, self.group)
            ptrs = [h.get_buffer(r, tuple(shape), dtype).data_ptr() for r in range(W)]
            return t, torch.tensor(ptrs, dtype=torch.int64, device=dev)

        self.xrecv, self.xrecv_ptrs = alloc((W, self.cap, H), torch.float16)
        self.meta, self.meta_ptrs = alloc((W, self.cap, 2), torch.int32)
        self.counts, self.count_ptrs = alloc((W,), torch.int64)
        self.flags, self.flag_ptrs = alloc((W,), torch.int64)
        self.done, self.done_ptrs = alloc((W,), torch.int64)
        self.ybuf, self.ybuf_ptrs = alloc((self.cap, H), torch.float32)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------------------------ one layer
    def moe(self, model, x, p, h, inj):
        """Expert-parallel MoE of one layer for this rank's tokens x [T, H] (act dtype); updates h in place.
        `p` holds this rank's expert shard (gu, d) plus the replicated router and shared expert."""
        cfg = self.cfg
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > EP capacity {self.max_tokens}")
        E = cfg.n_experts
        logits = model._mm(x, p["router"])
        ids, w = ops.moe_route(logits, E, self.k)
        if self.comm == "fused":
            self._fused_exchange(x, ids, p)
        else:
            self._nccl_exchange(x, ids, p)
        sact = model._mm(x, p["sgu"], epi=wgemm.EPI_SILU_MUL, out_dtype=model.act)
        ysh = model._mm(sact, p["sd"])
        if self.comm == "fused":
            native.C().ep_wait_done(self.done, self.world, self.epoch, native.err_word(self.device), self.timeout_ns)
        pair_pos = torch.arange(T * self.k, dtype=torch.int32, device=x.device).view(T, self.k)
        ops.moe_combine(h, self.ybuf, pair_pos, w, ysh, logits[:, E], inj)

    def _fused_exchange(self, x, ids, p):
        C = native.C()
        err = native.err_word(self.device)
        C.ep_epoch(self.epoch)
        C.ep_plan(ids, self.e_loc, self.world, self.dest_slot, self.dest_count)
        C.ep_push(x, ids, self.dest_slot, self.dest_count, self.k, self.e_loc, self.cap, self.rank, self.world,
                  self.xrecv_ptrs, self.meta_ptrs, self.count_ptrs, self.flag_ptrs, self.epoch, self.done_ctr, err)
        C.ep_gather(self.flags, self.counts, self.meta, self.xrecv.view(-1, self.H), self.cap, self.world, self.e_loc,
                    self.epoch, self.ybuf_ptrs, self.n_tile, self.sorted_src, self.items, self.n_items, self.row_dst,
                    self.n_rows, self.xs, err, self.timeout_ns)
        wgemm.grouped(self.xs, p["gu"], self.items, self.n_items, self.max_items, self.act, epi=wgemm.EPI_SILU_MUL,
                      n_tile=self.n_tile)
        wgemm.grouped(self.act, p["d"], self.items, self.n_items, self.max_items, self.yout, n_tile=self.n_tile,
                      row_dst=self.row_dst)
        C.ep_done(self.done_ptrs, self.rank, self.world, self.epoch)

    def _nccl_exchange(self, x, ids, p):
        """Baseline: rows to owners and outputs back with all_to_all_single (works on gloo CPU ranks too)."""
        W, k, H, dev = self.world, self.k, self.H, x.device
        flat = ids.reshape(-1).long()
        owner = flat // self.e_loc
        order = torch.argsort(owner, stable=True)
        send_counts = torch.bincount(owner, minlength=W)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        xrows = x.repeat_interleave(k, 0)[order]
        meta = (flat[order] - owner[order] * self.e_loc).to(torch.int32)
        xr = torch.empty(sum(rc), H, dtype=x.dtype, device=dev)
        mr = torch.empty(sum(rc), dtype=torch.int32, device=dev)
        dist.all_to_all_single(xr, xrows.contiguous(), rc, sc, group=self.group)
        dist.all_to_all_single(mr, meta, rc, sc, group=self.group)
        n = xr.shape[0]
        yr = torch.zeros(n, H, dtype=torch.float32, device=dev)
        if n:
            lid = mr.view(-1, 1)
            pp, items, n_items = ops.moe_plan(lid, self.e_loc, self.n_tile, (n + self.n_tile - 1) // self.n_tile + self.e_loc)
            xs = ops.moe_scatter(xr, pp)
            act = torch.empty(n, self.cfg.moe_inter, dtype=xs.dtype, device=dev)
            wgemm.grouped(xs, p["gu"], items, n_items, items.shape[0], act, epi=wgemm.EPI_SILU_MUL, n_tile=self.n_tile)
            ys = torch.empty(n, H, dtype=torch.float32, device=dev)
            wgemm.grouped(act, p["d"], items, n_items, items.shape[0], ys, n_tile=self.n_tile)
            yr = ys[pp.view(-1).long()]
        back = torch.empty(sum(sc), H, dtype=torch.float32, device=dev)
        dist.all_to_all_single(back, yr.contiguous(), sc, rc, group=self.group)
        ybuf = torch.empty(flat.numel(), H, dtype=torch.float32, device=dev)
        ybuf[order] = back
        self.ybuf = ybuf


def shard_experts(ws: wgemm.WeightSet, lo: int, hi: int) -> wgemm.WeightSet:
    """Sub-WeightSet of experts [lo, hi) (experts are stored contiguously in order)."""
    offs = ws.exp_off.tolist()
    start = offs[lo]
    end = offs[hi] if hi < len(offs) else ws.blob.numel()
    blob = ws.blob[start:end].clone()
    return wgemm.WeightSet(blob, ws.exp_off[lo:hi] - start, ws.exp_fmt[lo:hi].clone(), ws.rows, ws.K,
                           ws.fmts[lo:hi], ws.silu_pairs)


def shard_model_experts(weights: dict, rank: int, world: int) -> dict:
    """Keep only this rank's experts in every layer (router and shared expert stay replicated)."""
    for L in weights["layers"]:
        m = L["moe"]
        E = m["gu"].n_experts
        lo, hi = rank * E // world, (rank + 1) * E // world
        m["gu"] = shard_experts(m["gu"], lo, hi)
        m["d"] = shard_experts(m["d"], lo, hi)
    return weights

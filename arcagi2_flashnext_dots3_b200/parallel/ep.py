"""Expert-parallel MoE across GPUs: in-kernel NVLink dispatch/combine (product path) and an NCCL baseline.

Layout (one process per GPU, `world` ranks): every rank runs its own sequences through the dense parts of the
model (attention, Gated DeltaNet, hyper-connections, shared expert) and owns experts
[rank * E / world, (rank + 1) * E / world). Per MoE layer:

* fused path (``comm="fused"``, csrc/k_ep.cu): route -> stable per-destination plan -> push kernel stores every
  routed token row into its owner's symmetric receive buffer (peer stores) and publishes count + epoch flag ->
  owner waits for all sources, sorts by local expert, runs the grouped gate_up GEMM, and the down GEMM's
  epilogue stores every output row directly into the source's pair buffer on the source GPU -> completion
  flags -> the source waits, then combines locally (weights + shared expert + hyper-connection injection);
* baseline (``comm="nccl"``): NCCL collectives only, the reference's scheme moved onto the GPU: every rank
  all-gathers the (padded) token rows, routing ids and weights, runs its own experts on the pairs they own and
  computes per-token weighted partial sums, and a reduce-scatter returns each rank its tokens' routed sum.
  Static shapes throughout, so both paths capture into CUDA graphs.

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
                 n_tile: int = 0, timeout_ns: int = None):
        if cfg.n_experts % world:
            raise ValueError(f"{cfg.n_experts} experts do not split over {world} ranks")
        self.cfg, self.rank, self.world, self.comm = cfg, rank, world, comm
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.e_loc = cfg.n_experts // world
        self.lo, self.hi = rank * self.e_loc, (rank + 1) * self.e_loc
        self.k = cfg.top_k
        self.H = cfg.hidden_size
        self.max_tokens = max_tokens
        self.cap = max_tokens * self.k            # pairs one source can send to one owner (worst case)
        # token tile of the expert GEMMs: average pairs per expert over the whole job
        # decode-sized exchanges (few pairs per local expert on average) run the experts on the int8 GEMV, whose
        # plans are built with items of at most GEMV_MAX_TOK rows; larger ones on the tcgen05 grouped GEMM
        pairs_per_expert = world * self.cap / cfg.n_experts
        self.use_gemv = not n_tile and pairs_per_expert <= EP_GEMV_PAIRS and wgemm_gemv_ok(cfg)
        self.n_tile = n_tile or (wgemm.GEMV_MAX_TOK if self.use_gemv else
                                 wgemm.pick_n_tile(max(1, (2 * world * self.cap) // cfg.n_experts)))
        self.timeout_ns = timeout_ns or native.DEFAULT_TIMEOUT_NS * 4
        dev, W, H = self.device, world, self.H
        self.max_rows = W * self.cap
        self.max_items = (self.max_rows + self.n_tile - 1) // self.n_tile + self.e_loc + 1
        self.act = torch.zeros(self.max_rows, cfg.moe_inter, dtype=ops.act_dtype(dev), device=dev)
        self.yout = torch.zeros(self.max_rows, H, dtype=torch.float32, device=dev)
        if comm == "fused":
            self.dest_slot = torch.zeros(self.cap, dtype=torch.int32, device=dev)
            self.dest_count = torch.zeros(W, dtype=torch.int32, device=dev)
            self.sorted_src = torch.zeros(self.max_rows, dtype=torch.int32, device=dev)
            self.items = torch.zeros(self.max_items, 4, dtype=torch.int32, device=dev)
            self.n_items = torch.zeros(1, dtype=torch.int32, device=dev)
            self.row_dst = torch.zeros(self.max_rows, dtype=torch.int64, device=dev)
            self.n_rows = torch.zeros(1, dtype=torch.int32, device=dev)
            self.xs = torch.zeros(self.max_rows, H, dtype=torch.float16, device=dev)
            self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
            self.done_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
            self._alloc_symmetric()
        elif comm == "nccl":
            Tm, k = max_tokens, self.k
            self.xpad = torch.zeros(Tm, H, dtype=ops.act_dtype(dev), device=dev)
            self.idpad = torch.full((Tm, k), -1, dtype=torch.int32, device=dev)
            self.wpad = torch.zeros(Tm, k, dtype=torch.float32, device=dev)
            self.xg = torch.zeros(W * Tm, H, dtype=self.xpad.dtype, device=dev)
            self.idg = torch.zeros(W * Tm, k, dtype=torch.int32, device=dev)
            self.wg = torch.zeros(W * Tm, k, dtype=torch.float32, device=dev)
            self.yr = torch.zeros(Tm, H, dtype=torch.float32, device=dev)
            self.one_pos = torch.arange(Tm, dtype=torch.int32, device=dev).view(Tm, 1).expand(Tm, k).contiguous()
            self.one_w = torch.zeros(Tm, k, dtype=torch.float32, device=dev)
            self.one_w[:, 0] = 1.0
            self.item_idx = torch.arange(self.max_items, dtype=torch.int32, device=dev)
        else:
            raise ValueError(f"unknown EP exchange {comm!r}")

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
        `p` holds this rank's expert shard (gu, d) plus the replicated router and shared expert. Every rank must
        call this the same number of times (ranks without tokens pass T = 0 rows)."""
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
            yr = self._nccl_exchange(x, ids, w, p)
        sact = model._mm(x, p["sgu"], epi=wgemm.EPI_SILU_MUL, out_dtype=model.act)
        ysh = model._mm(sact, p["sd"])
        if self.comm == "fused":
            native.C().ep_wait_done(self.done, self.world, self.epoch, native.err_word(self.device), self.timeout_ns)
            pair_pos = torch.arange(T * self.k, dtype=torch.int32, device=x.device).view(T, self.k)
            ops.moe_combine(h, self.ybuf, pair_pos, w, ysh, logits[:, E], inj)
        else:
            ops.moe_combine(h, yr, self.one_pos[:T], self.one_w[:T], ysh, logits[:, E], inj)

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
        if self.use_gemv:
            wgemm.gemv_grouped(self.xs, p["gu"], self.items, self.n_items, self.max_items, self.act,
                               epi=wgemm.EPI_SILU_MUL)
            wgemm.gemv_grouped(self.act, p["d"], self.items, self.n_items, self.max_items, self.yout,
                               row_dst=self.row_dst)
        else:
            wgemm.grouped(self.xs, p["gu"], self.items, self.n_items, self.max_items, self.act,
                          epi=wgemm.EPI_SILU_MUL, n_tile=self.n_tile)
            wgemm.grouped(self.act, p["d"], self.items, self.n_items, self.max_items, self.yout, n_tile=self.n_tile,
                          row_dst=self.row_dst)
        C.ep_done(self.done_ptrs, self.rank, self.world, self.epoch)

    def _nccl_exchange(self, x, ids, w, p):
        """Baseline: all-gather tokens + routing, local experts on owned pairs, reduce-scatter of the weighted
        per-token partial sums. Returns this rank's routed sum [T, H] fp32 (works on gloo CPU ranks too)."""
        W, k, H, Tm, T = self.world, self.k, self.H, self.max_tokens, x.shape[0]
        self.xpad[:T].copy_(x)
        self.idpad[:T].copy_(ids)
        self.idpad[T:].fill_(-1)
        self.wpad[:T].copy_(w)
        self._all_gather(self.xg, self.xpad)
        self._all_gather(self.idg, self.idpad)
        self._all_gather(self.wg, self.wpad)
        owned = (self.idg >= self.lo) & (self.idg < self.hi)
        lid = torch.where(owned, self.idg - self.lo, self.e_loc).to(torch.int32)
        # non-owned pairs go to a dummy expert e_loc; its items sort last and are cut from the item count
        pp, items, n_items = ops.moe_plan(lid, self.e_loc + 1, self.n_tile, self.max_items)
        n_loc = ((items[:, 0] < self.e_loc) & (self.item_idx < n_items)).sum().to(torch.int32).view(1)
        xs = ops.moe_scatter(self.xg, pp)
        if self.use_gemv and xs.is_cuda:
            wgemm.gemv_grouped(xs, p["gu"], items, n_loc, self.max_items, self.act, epi=wgemm.EPI_SILU_MUL)
            wgemm.gemv_grouped(self.act, p["d"], items, n_loc, self.max_items, self.yout)
        else:
            wgemm.grouped(xs, p["gu"], items, n_loc, self.max_items, self.act, epi=wgemm.EPI_SILU_MUL,
                          n_tile=self.n_tile)
            wgemm.grouped(self.act, p["d"], items, n_loc, self.max_items, self.yout, n_tile=self.n_tile)
        y = self.yout[pp.reshape(-1).long()].view(W * Tm, k, H)
        part = (torch.where(owned[..., None], y, 0.0) * self.wg[..., None]).sum(1)
        if part.is_cuda:
            dist.reduce_scatter_tensor(self.yr, part, group=self.group)
        else:  # gloo has no reduce-scatter
            dist.all_reduce(part, group=self.group)
            self.yr.copy_(part[self.rank * Tm:(self.rank + 1) * Tm])
        return self.yr[:T]

    def _all_gather(self, out, inp):
        if inp.is_cuda:
            dist.all_gather_into_tensor(out, inp, group=self.group)
        else:
            dist.all_gather(list(out.chunk(self.world)), inp, group=self.group)

EP_GEMV_PAIRS = float(__import__("os").environ.get("FW_EP_GEMV_PAIRS", "8"))


def wgemm_gemv_ok(cfg) -> bool:
    """The int8 GEMV serves 2/3/4-bit experts only, and only when the decode-MoE GEMV is switched on."""
    from ..models import fn as fn_model
    return fn_model.GEMV_MOE and all(cfg.bits_of(e) <= 4 for e in range(cfg.n_experts))


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

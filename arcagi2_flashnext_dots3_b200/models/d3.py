"""Dots3-Note-shaped model on the engine path: incremental prefill + decode over paged FP8 latent caches.

Layer (pre-norm, the reference's dotsnote/training/finetune/student.py:353-362 and the served vLLM model
dotsnote/engine/vllm_patch/vllm/models/dots3_note/nvidia/model.py:513):

    x = rms(h, ln1)                                   (fused with the previous residual add)
    P = x @ [q_a | kv_a | g | idx_k | idx_w]^T        one tcgen05 GEMM
    prep: q latent norm, FP8 latent row (kv norm + RoPE'd key) into the paged cache, index key into its cache
    Q = q_latent @ [q_b | idx_q]^T                    one tcgen05 GEMM
    q_lat[h] = q_nope[h] @ W_UK[h]                    per-head absorption (batched GEMM)
    DSA layers: indexer logits -> exact top-2048 key positions; SWA layers: the last `swa_window` positions
    o_lat = latent attention over the selected FP8 rows (shared by all heads)
    o[h] = o_lat[h] @ W_UV[h]^T, times sigmoid(g)     absorption back + gate
    h += o @ W_o^T ; x = rms(h, ln2) ; h += MoE(x) (sigmoid router + bias, 3/2-bit experts, shared expert)

Every projection runs on the tcgen05 weight-dequant GEMM; the two per-head absorption products are batched GEMMs
(cuBLAS by default, faster at decode batch than the grouped tcgen05 form available with FW_D3_ABSORB=grouped);
the rest are the kernels of csrc/k_d3.cu and the FN MoE kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import d3_ops as d3
from ..ops import fn_ops as ops
from ..ops import wgemm


@dataclass
class D3Caches:
    latent: list        # per layer [n_blocks, block_size, kvr + dr]
    idx: list           # per layer [S, max_len, iD] (DSA layers) or None
    block_table: torch.Tensor
    block_size: int
    n_blocks: int
    max_len: int


INDEX_SLACK = 4096   # rows past a sharded index cache's end that prefill chunks of up to this many tokens may read


def allocate_caches(cfg, device, n_slots: int, max_len: int, block_size: int = 64, n_blocks: int = None,
                    kv_dtype: str = "fp8", state_dtype: str = "bf16", index_shards: int = 1) -> D3Caches:
    """``index_shards`` > 1: the DSA index caches hold one TP rank's share of the positions (p = rank mod W)."""
    dev = torch.device(device)
    cpu = dev.type == "cpu"
    max_blocks = (max_len + block_size - 1) // block_size
    n_blocks = n_blocks or n_slots * max_blocks
    idx_len = max_len if index_shards == 1 else -(-max_len // index_shards) + INDEX_SLACK
    latent, idx = [], []
    for l in range(cfg.num_layers):
        D = cfg.latent_of(l) + cfg.qk_rope_dim
        latent.append(torch.zeros(n_blocks, block_size, D, dtype=torch.float32 if cpu else torch.float8_e4m3fn,
                                  device=dev))
        own_index = cfg.layer_kind(l) == "dsa" and l not in cfg.shared_index_layers()
        idx.append(torch.zeros(n_slots, idx_len, cfg.index_dim, dtype=torch.float32 if cpu else torch.bfloat16,
                               device=dev) if own_index else None)
    return D3Caches(latent, idx, torch.zeros(n_slots, max_blocks, dtype=torch.int32, device=dev), block_size,
                    n_blocks, max_len)


class D3Model:
    allocate = staticmethod(allocate_caches)

    def __init__(self, cfg, weights: dict, caches: D3Caches, device, ep=None, tp=None):
        """``tp``: a :class:`..parallel.tp.TPGroup`; then `cfg` is the rank's view (:func:`..parallel.tp.tp_config`)
        and `weights` the rank's shard (:func:`..parallel.tp.shard_d3_weights` + :func:`.d3_weights.to_engine`)."""
        self.cfg, self.W, self.c = cfg, weights, caches
        self.ep = ep
        self.tp = tp
        self.device = torch.device(device)
        self.act = ops.act_dtype(self.device)
        self.rope = d3.rope_table(caches.max_len + 8, cfg.qk_rope_dim, cfg.rope_theta, self.device)
        self.scale = (cfg.qk_nope_dim + cfg.qk_rope_dim) ** -0.5
        self.shared_index = cfg.shared_index_layers()
        self.index_shard = (tp.world, tp.rank) if (tp is not None and cfg.shard_index) else (1, 0)
        self.overlap = None     # utils.observe.TopkOverlap: per-step top-k overlap between DSA layers (eval only)

    def _mm(self, x, ws, epi=wgemm.EPI_STORE, out_dtype=torch.float32, f8=True):
        if not x.is_cuda:
            return wgemm.matmul(x.float(), ws, epi=epi, out_dtype=torch.float32)
        return wgemm.matmul(x, ws, epi=epi, out_dtype=out_dtype, f8=f8)

    def _head_items(self, H: int, T: int, n_tile: int):
        """Grouped-GEMM plan with one expert per head: items (h, first row h*T + s, count, 0) over n_tile chunks."""
        key = (H, T, n_tile)
        cache = self.__dict__.setdefault("_items", {})
        if key not in cache:
            it = [[h, h * T + s, min(n_tile, T - s), 0] for h in range(H) for s in range(0, T, n_tile)]
            cache[key] = (torch.tensor(it, dtype=torch.int32, device=self.device),
                          torch.tensor([len(it)], dtype=torch.int32, device=self.device))
        return cache[key]

    def _absorb(self, x: torch.Tensor, p: dict, which: str) -> torch.Tensor:
        """Per-head latent absorption [H, T, k] -> [H, T, n]: q_lat = q_nope[h] @ uk[h] (which="uk") or
        o[h] = o_lat[h] @ uv[h]^T (which="uv"): a batched GEMM on the dense per-head matrices (cuBLAS on a GPU), or
        with the grouped weight sets (FW_D3_ABSORB=grouped) one tcgen05 grouped GEMM over all heads, every head an
        expert of an fp16 weight set."""
        if not x.is_cuda or which + "_ws" not in p:
            return torch.bmm(x, p["uk"]) if which == "uk" else torch.bmm(x, p["uv"].transpose(1, 2))
        ws = p[which + "_ws"]
        H, T, K = x.shape
        n_tile = wgemm.pick_n_tile(T)
        items, n_items = self._head_items(H, T, n_tile)
        out = torch.empty(H, T, ws.rows, dtype=torch.bfloat16, device=x.device)
        x16 = x.reshape(H * T, K).half()
        if ws.K != K:   # zero-padded K (small head dims)
            x16 = torch.nn.functional.pad(x16, (0, ws.K - K))
        wgemm.grouped(x16, ws, items, n_items, items.shape[0], out.view(H * T, ws.rows), n_tile=n_tile)
        return out

    def _attn(self, x, p, l, slots, positions, n_tok):
        cfg, c = self.cfg, self.c
        P = self._mm(x, p["a"])
        shared = l in self.shared_index
        qc, gate, iw = d3.mla_prep(P, cfg, l, p, self.rope, c.latent[l], c.block_table, c.idx[l], slots, positions,
                                   n_tok, index=not shared, index_shard=self.index_shard)
        Q = self._mm(qc, p["qb"])
        q_nope, q_pe, iq = d3.mla_qsplit(Q, cfg, l, self.rope, positions, n_tok)
        q_lat = self._absorb(q_nope, p, "uk")                   # [H, T, kvr]
        if cfg.layer_kind(l) == "dsa":
            if shared:     # index sharing: the latest indexing layer's selection, no scoring of our own
                sel = self._sel
            elif self.index_shard[0] > 1:
                sel = d3.dsa_select_sharded(iq, iw, c.idx[l], slots, positions, n_tok, cfg.index_topk,
                                            self.index_shard[1], self.index_shard[0], self.tp.group)
                self._sel = sel
            else:
                sel = d3.dsa_select(iq, iw, c.idx[l], slots, positions, n_tok, cfg.index_topk, c.max_len)
                self._sel = sel
            if self.overlap is not None:
                self.overlap.add(l, sel, positions, n_tok)
            window = 0
        else:
            sel, window = None, cfg.swa_window
        o_lat = d3.mla_attn(q_lat, q_pe, c.latent[l], c.block_table, slots, positions, n_tok, sel, window,
                            self.scale)
        o = self._absorb(o_lat, p, "uv")                        # [H, T, dv]
        if self.tp is not None and getattr(self.tp, "sp", False):   # sequence parallel: the partial, scattered later
            return self._mm(d3.mla_out(o, gate), p["o"])
        if self.tp is not None:  # row-parallel o-projection fused with the all-reduce; adds into h itself
            self.tp.linear_allreduce_add(self, d3.mla_out(o, gate), p["o"], self._h)
            return None
        return self._mm(d3.mla_out(o, gate), p["o"])

    def _moe_tp(self, x, p, h):
        """Tensor parallel: global routing, this rank's experts for all tokens, partial sum all-reduced into h.
        The shared expert is added by rank 0 only."""
        cfg, tp = self.cfg, self.tp
        T, E = x.shape[0], cfg.n_experts
        lo, hi = p["expert_range"]
        E_loc = hi - lo
        logits = self._mm(x, p["router"])
        ids, w = d3.route(logits, E, p["bias"], cfg.top_k, cfg.route_scale)
        local = (ids >= lo) & (ids < hi)
        lid = torch.where(local, ids - lo, torch.full_like(ids, E_loc)).to(torch.int32)
        wl = torch.where(local, w, torch.zeros_like(w))
        P = T * cfg.top_k
        gemv = x.is_cuda and P <= 4 * E
        n_tile = wgemm.GEMV_MAX_TOK if gemv else (wgemm.pick_n_tile(max(1, (2 * P) // E)) if x.is_cuda else 16)
        max_items = (P + n_tile - 1) // n_tile + E_loc + 1
        pair_pos, items, n_items = ops.moe_plan(lid, E_loc + 1, n_tile, max_items)
        idx = torch.arange(max_items, dtype=torch.int32, device=x.device)
        n_loc = ((items[:, 0] < E_loc) & (idx < n_items)).sum().to(torch.int32).view(1)
        xs = ops.moe_scatter(x, pair_pos)
        act = torch.empty(P, cfg.moe_inter, dtype=self.act, device=x.device)
        ypair = torch.empty(P + 1, cfg.hidden_size, dtype=torch.float32, device=x.device)
        ypair[P].zero_()
        if gemv:
            wgemm.gemv_grouped(xs, p["gu"], items, n_loc, max_items, act, epi=wgemm.EPI_SILU_MUL)
            wgemm.gemv_grouped(act, p["d"], items, n_loc, max_items, ypair)
        else:
            wgemm.grouped(xs, p["gu"], items, n_loc, max_items, act, epi=wgemm.EPI_SILU_MUL, n_tile=n_tile)
            wgemm.grouped(act, p["d"], items, n_loc, max_items, ypair, n_tile=n_tile)
        pp = torch.where(local, pair_pos, torch.full_like(pair_pos, P))
        sact = self._mm(x, p["sgu"], epi=wgemm.EPI_SILU_MUL, out_dtype=self.act)
        ysh = self._mm(sact, p["sd"])
        sg = torch.full((T,), float("inf") if tp.rank == 0 else float("-inf"), device=x.device)
        part = torch.zeros(T, cfg.hidden_size, dtype=torch.float32, device=x.device)
        ops.moe_combine(part, ypair, pp, wl, ysh, sg, torch.ones(T, 1, dtype=torch.float32, device=x.device))
        if h is None:          # sequence parallel: the caller reduce-scatters the partial
            return part
        tp.allreduce_add(h, part)

    def _moe(self, x, p, h):
        if self.tp is not None:
            return self._moe_tp(x, p, h)
        cfg = self.cfg
        T, E = x.shape[0], cfg.n_experts
        logits = self._mm(x, p["router"])
        ids, w = d3.route(logits, E, p["bias"], cfg.top_k, cfg.route_scale)
        P = T * cfg.top_k
        gemv = x.is_cuda and P <= 4 * E   # decode: a few tokens per expert -> CUDA-core grouped GEMV
        n_tile = wgemm.GEMV_MAX_TOK if gemv else (wgemm.pick_n_tile(max(1, (2 * P) // E)) if x.is_cuda else 16)
        max_items = (P + n_tile - 1) // n_tile + E
        pair_pos, items, n_items = ops.moe_plan(ids, E, n_tile, max_items)
        xs = ops.moe_scatter(x, pair_pos)
        act = torch.empty(P, cfg.moe_inter, dtype=self.act, device=x.device)
        ypair = torch.empty(P, cfg.hidden_size, dtype=torch.float32, device=x.device)
        if gemv:
            wgemm.gemv_grouped(xs, p["gu"], items, n_items, max_items, act, epi=wgemm.EPI_SILU_MUL)
            wgemm.gemv_grouped(act, p["d"], items, n_items, max_items, ypair)
        else:
            wgemm.grouped(xs, p["gu"], items, n_items, max_items, act, epi=wgemm.EPI_SILU_MUL, n_tile=n_tile)
            wgemm.grouped(act, p["d"], items, n_items, max_items, ypair, n_tile=n_tile)
        sact = self._mm(x, p["sgu"], epi=wgemm.EPI_SILU_MUL, out_dtype=self.act)
        ysh = self._mm(sact, p["sd"])
        ones = torch.ones(T, 1, dtype=torch.float32, device=x.device)
        ops.moe_combine(h, ypair, pair_pos, w, ysh, torch.full((T,), float("inf"), device=x.device), ones)

    def step(self, ids: torch.Tensor, slots: torch.Tensor, positions: torch.Tensor, n_tok: int = 1,
             verify: bool = False):
        """Hidden states [T, H] after the final norm. ``verify`` (speculative verification) needs no special
        handling: every cache of this model is position-indexed, so rejected positions are simply rewritten
        when real tokens reach them, and :meth:`commit` has nothing to do."""
        return self.step_from_h(self.W["embed"][ids.long()].float(), slots, positions, n_tok)

    def commit(self, n_commit: torch.Tensor):
        """Speculative commit: nothing to roll forward (no recurrent state)."""

    def step_from_h(self, h: torch.Tensor, slots: torch.Tensor, positions: torch.Tensor, n_tok: int = 1):
        cfg, W = self.cfg, self.W
        if self.tp is not None and getattr(self.tp, "sp", False):
            return self._step_sp(h.float(), slots, positions, n_tok)
        h = h.float().contiguous()
        self._h = h
        if self.tp is not None and hasattr(self.tp, "begin_forward"):
            self.tp.begin_forward()
        y = None
        for l, L in enumerate(W["layers"]):
            x = d3.add_rms(h, y, L["ln1"], cfg.rms_eps, self.act)
            y = self._attn(x, L["attn"], l, slots, positions, n_tok)
            x = d3.add_rms(h, y, L["ln2"], cfg.rms_eps, self.act)
            if cfg.is_moe(l):
                self._moe(x, L["moe"], h)
                y = None
            else:
                sact = self._mm(x, L["mlp"]["gu"], epi=wgemm.EPI_SILU_MUL, out_dtype=self.act)
                y = self._mm(sact, L["mlp"]["d"])
        return d3.add_rms(h, y, W["norm"], cfg.rms_eps, self.act)

    def _step_sp(self, h, slots, positions, n_tok):
        """Sequence-parallel layer loop: this rank keeps T/W rows of the residual stream (zero-padded to a multiple
        of the group size) and normalizes only those; the attention and MoE partials (row-parallel products over
        this rank's heads / experts, all tokens) are reduce-scattered into it, and the normalized rows are
        all-gathered before the next column-parallel GEMM. The dense MLP layers are replicated: their output rows
        are sliced. Returns the final normalized hidden states of all T tokens."""
        cfg, W, tp = self.cfg, self.W, self.tp
        T = h.shape[0]
        Tp, Tl = tp.sp_rows(T)
        if Tp != T:
            h = torch.nn.functional.pad(h, (0, 0, 0, Tp - T))
        h_loc = h[tp.rank * Tl:(tp.rank + 1) * Tl].contiguous()
        if hasattr(tp, "begin_forward"):
            tp.begin_forward()
        y = None
        for l, L in enumerate(W["layers"]):
            x = tp.all_gather(d3.add_rms(h_loc, y, L["ln1"], cfg.rms_eps, self.act), T)
            y = tp.reduce_scatter(self._attn(x, L["attn"], l, slots, positions, n_tok))
            x = tp.all_gather(d3.add_rms(h_loc, y, L["ln2"], cfg.rms_eps, self.act), T)
            if cfg.is_moe(l):
                y = tp.reduce_scatter(self._moe_tp(x, L["moe"], None))
            else:
                sact = self._mm(x, L["mlp"]["gu"], epi=wgemm.EPI_SILU_MUL, out_dtype=self.act)
                full = self._mm(sact, L["mlp"]["d"]).float()
                if Tp != T:
                    full = torch.nn.functional.pad(full, (0, 0, 0, Tp - T))
                y = full[tp.rank * Tl:(tp.rank + 1) * Tl].contiguous()
        return tp.all_gather(d3.add_rms(h_loc, y, W["norm"], cfg.rms_eps, self.act), T)

    @property
    def vocab_sharded(self) -> bool:
        """True when the LM head is split over the TP ranks: each rank holds only its vocabulary slice, so next
        tokens must come from :meth:`pick` (a local argmax would return slice-local indices)."""
        return self.tp is not None and "vocab_range" in self.W

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        """Logits over the whole vocabulary. Refused when the head is split over a TP group, since this rank then
        holds only a slice whose indices are not token ids: use :meth:`pick`."""
        if self.vocab_sharded:
            raise RuntimeError("D3Model.logits: the LM head is vocabulary-sharded; select tokens with pick()")
        return self._mm(x, self.W["lm_head"], f8=False)

    def pick(self, x: torch.Tensor, temperature: float = 0.0, seed: int = 0, step: int = 0, top_k: int = 0,
             top_p: float = 1.0) -> torch.Tensor:
        """Next token per row (int32): greedy, Gumbel-max temperature sampling with the sampler's counter RNG, or
        top-k / top-p sampling (the sampler's candidate rule). With the LM head split over the TP ranks
        (``vocab_range`` in the weights) one (value, index) pair per row crosses the group for greedy and
        full-vocabulary sampling, K pairs per row for top-k / top-p (:func:`..parallel.tp.sharded_sample`)."""
        lg = self._mm(x, self.W["lm_head"], f8=False)
        filtered = temperature > 0 and (top_k > 0 or top_p < 1.0)
        if self.vocab_sharded:
            if getattr(self.tp, "fake", False):
                if filtered:
                    raise NotImplementedError("fake TP emulates the greedy / full-vocabulary pick only")
                return self.tp.sharded_pick(lg, self.W["vocab_range"][0], temperature, seed, step)
            from ..parallel.tp import sharded_pick, sharded_sample
            if filtered:
                return sharded_sample(lg, self.W["vocab_range"][0], self.cfg.vocab_size, self.tp.group, temperature,
                                      top_k, top_p, seed, step)
            return sharded_pick(lg, self.W["vocab_range"][0], self.tp.group, temperature, seed, step)
        if temperature <= 0:
            return ops.argmax(lg)
        from ..ops import sampling
        if filtered:
            B = lg.shape[0]
            dev = lg.device
            ids, _ = sampling.sample(lg.float().contiguous(), torch.full((B,), temperature, device=dev),
                                     torch.full((B,), top_k, dtype=torch.int32, device=dev),
                                     torch.full((B,), top_p, device=dev),
                                     torch.full((B,), seed, dtype=torch.int64, device=dev),
                                     torch.full((B,), step, dtype=torch.int64, device=dev), want_lp=False)
            return ids
        u = sampling.uniform_torch(seed, step, torch.arange(lg.shape[1], device=lg.device))
        return (lg.float() / temperature - torch.log(-torch.log(u))[None, :]).argmax(-1).to(torch.int32)

    # ------------------------------------------------------------------------------------------- engine hooks
    def assign_blocks(self, slot: int, n_tokens: int, allocator):
        bs = self.c.block_size
        need = (n_tokens + bs - 1) // bs
        have = allocator.n_blocks_of(slot)
        if need > have:
            new = allocator.allocate(slot, need - have)
            self.c.block_table[slot, have:need] = torch.tensor(new, dtype=torch.int32, device=self.device)

    def reset_slot(self, slot: int):
        pass  # attention-only state: the block table and positions define what is visible

    def randomize_caches(self, g: torch.Generator):
        for t in self.c.latent:
            t.copy_((torch.randn(t.shape, generator=g, device=self.device)).to(t.dtype))
        for t in self.c.idx:
            if t is not None:
                t.copy_(torch.randn(t.shape, generator=g, device=self.device).to(t.dtype))

"""Flash-Next-shaped model on the engine path: incremental prefill + decode over per-sequence caches.

The layer wiring is the reference's (flashnext/training/student/student_fn.py:578 `Layer.forward`): PLE add,
attention hyper-connection, mixer (Gated DeltaNet or block-sparse attention), residual injection into every
stream, MLP hyper-connection, MoE, residual injection; final hyper-connection mixer and LM head.

Differences from the reference's serving stack (vLLM + the `fnext` overlay) are in HOW each step runs:
every GEMM is the tcgen05 weight-dequant kernel (fused projections: GDN qkv|z|b|a in one launch, attention
q|gate|k|v|indexer in one launch, router + shared-expert gate in one launch), the MoE is one grouped launch per
projection for all experts and bit widths with silu*up fused into the gate_up epilogue, and combine + shared
expert + hyper-connection injection is one kernel.

Caches (per slot = sequence): paged attention KV (fp8 on GPU), per-slot compressed indexer keys and a ring of
the last `ratio` raw indexer keys, GDN conv and recurrent states, PLE conv history and n-gram token history.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from ..ops import fn_ops as ops
from ..ops import wgemm
from .fn_weights import rank_pad

GEMV_MOE = os.environ.get("FW_MOE_GEMV", "1") != "0"   # decode MoE on the CUDA-core grouped GEMV
# the GEMV serves MoE calls with at most this many (token, expert) pairs per expert on average (above: tcgen05)
GEMV_PAIRS_PER_EXPERT = float(os.environ.get("FW_MOE_GEMV_PAIRS", "4"))
SIDE_STREAM = os.environ.get("FW_SIDE_STREAM", "1") != "0"  # shared expert concurrent with the routed experts


# Extra entries of the position-indexed rings (indexer raw keys, PLE values): speculative verification writes up to
# this many rejected positions ahead without overwriting entries that accepted positions still need.
SPEC_SLACK = 8


@dataclass
class FNCaches:
    k: list            # per attention layer [n_blocks, block_size, KV, D]
    v: list
    kr_ring: list      # per attention layer [S, ratio + SPEC_SLACK, iD] raw indexer keys by position mod length
    comp: list         # per attention layer [S, max_comp_blocks, iD]
    conv: list         # per linear layer [S, C, kc-1]
    ssm: list          # per linear layer [S, nv, dk, dv]
    block_table: torch.Tensor  # [S, max_blocks] int32
    block_size: int
    n_blocks: int
    ple_hist: list = None           # per PLE layer [S, (ple_conv-1)*ngram, hc*H] ring of normalized gated values
    tok_hist: torch.Tensor = None   # [S, ngram]: ngram-1 previous tokens (newest first) + tokens since eos


def kv_dtype_for(device, kv_dtype: str):
    if torch.device(device).type == "cpu":
        return torch.float32
    return torch.float8_e4m3fn if kv_dtype == "fp8" else torch.bfloat16


def allocate_caches(cfg, device, n_slots: int, max_len: int, block_size: int = 64, n_blocks: int = None,
                    kv_dtype: str = "fp8", state_dtype: str = "bf16") -> FNCaches:
    dev = torch.device(device)
    kvd = kv_dtype_for(dev, kv_dtype)
    sd = torch.float32 if dev.type == "cpu" or state_dtype == "fp32" else torch.bfloat16
    max_blocks = (max_len + block_size - 1) // block_size
    n_blocks = n_blocks or n_slots * max_blocks
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    C = 2 * nk * dk + nv * dv
    n_attn = sum(cfg.layer_kind(l) == "attention" for l in range(cfg.num_layers))
    n_lin = cfg.num_layers - n_attn
    idx_dt = torch.float32 if dev.type == "cpu" else torch.bfloat16
    c = FNCaches(
        k=[torch.zeros(n_blocks, block_size, cfg.n_kv_heads, cfg.head_dim, dtype=kvd, device=dev) for _ in range(n_attn)],
        v=[torch.zeros(n_blocks, block_size, cfg.n_kv_heads, cfg.head_dim, dtype=kvd, device=dev) for _ in range(n_attn)],
        kr_ring=[torch.zeros(n_slots, cfg.indexer_ratio + SPEC_SLACK, cfg.indexer_dim, dtype=torch.float32, device=dev)
                 for _ in range(n_attn)],
        comp=[torch.zeros(n_slots, max_len // cfg.indexer_ratio + 1, cfg.indexer_dim, dtype=idx_dt, device=dev)
              for _ in range(n_attn)],
        conv=[torch.zeros(n_slots, C, cfg.conv_kernel - 1, dtype=torch.float32, device=dev) for _ in range(n_lin)],
        ssm=[torch.zeros(n_slots, nv, dk, dv, dtype=sd, device=dev) for _ in range(n_lin)],
        block_table=torch.zeros(n_slots, max_blocks, dtype=torch.int32, device=dev),
        block_size=block_size, n_blocks=n_blocks)
    if cfg.ple_layers:
        c.ple_hist = [torch.zeros(n_slots, (cfg.ple_conv - 1) * cfg.ngram_size + SPEC_SLACK, cfg.hc_count * cfg.hidden_size,
                                  dtype=torch.float32, device=dev) for _ in cfg.ple_layers]
        c.tok_hist = torch.full((n_slots, cfg.ngram_size), cfg.eos_token_id, dtype=torch.int64, device=dev)
        c.tok_hist[:, -1] = 0
    return c


class FNModel:
    """Engine model. ``step(ids, slots, positions, n_tok)`` runs rows = len(slots) * n_tok tokens (token j of
    sequence b at positions[b] + j) through all layers, updating the caches of `slots`, and returns the final
    hidden state [rows, H] (act dtype); ``logits`` applies the LM head."""

    def __init__(self, cfg, weights: dict, caches: FNCaches, device, ep=None):
        self.cfg = cfg
        self.ep = ep  # parallel.ep.EPGroup: expert-parallel MoE across GPUs (None = all experts local)
        self.capture = None  # training.capture.RoutingCapture: records MoE inputs / router logits (eager steps)
        self._layer = 0
        self.W = weights
        self.c = caches
        self.device = torch.device(device)
        self.act = ops.act_dtype(self.device)
        self.rope = ops.rope_tables(caches.block_table.shape[1] * caches.block_size + 8, cfg.rope_dim,
                                    cfg.rope_theta, self.device)
        self.rank_pad = rank_pad(cfg)
        self.attn_idx = {}
        self.lin_idx = {}
        for l in range(cfg.num_layers):
            d = self.attn_idx if cfg.layer_kind(l) == "attention" else self.lin_idx
            d[l] = len(d)

    # ------------------------------------------------------------------------------------------ pieces
    def _mm(self, x, ws, epi=wgemm.EPI_STORE, out_dtype=torch.float32, f8=True):
        if not x.is_cuda:
            return wgemm.matmul(x.float(), ws, epi=epi, out_dtype=torch.float32)
        return wgemm.matmul(x, ws, epi=epi, out_dtype=out_dtype, f8=f8)

    def _hc(self, h, p, with_inj=True):
        cfg = self.cfg
        hn = ops.hc_prenorm(h, p["norm"], cfg.hc_count, cfg.hidden_size, cfg.rms_eps)
        z = self._mm(hn, p["w1"])
        a, inj = ops.hc_act(z, self.rank_pad, cfg.hc_count, with_inj)
        u = self._mm(a, p["w2"])
        x = ops.hc_mix(u, hn, cfg.hc_count, cfg.hidden_size)
        return x, inj

    def _gdn(self, x, p, li, slots, n_tok):
        proj = self._mm(x, p["proj"])
        v = getattr(self, "_verify", None)
        ncm = None
        if v is not None:
            v["proj"][li] = (proj, p)
            ncm = v["zeros"]
        o = ops.gdn_step(proj, p["conv"], self.c.conv[li], self.c.ssm[li], p["A_log"], p["dt_bias"], p["norm"],
                         slots, self.cfg, n_tok, n_commit=ncm)
        return self._mm(o, p["out"])

    def commit(self, n_commit: torch.Tensor):
        """After a verify step: advance every recurrent state by the first n_commit[b] tokens of sequence b
        (int32 [B] on the model's device) and restore + replay the PLE token history."""
        v = self._verify
        if v is None:
            raise RuntimeError("commit() without a preceding verify step")
        for li, (proj, p) in v["proj"].items():
            ops.gdn_step(proj, p["conv"], self.c.conv[li], self.c.ssm[li], p["A_log"], p["dt_bias"], p["norm"],
                         v["slots"], self.cfg, v["n_tok"], n_commit=n_commit)
        if "tok_hist" in v:
            self._replay_tok_hist(v, n_commit)
        self._verify = None

    def _replay_tok_hist(self, v, n_commit):
        cfg = self.cfg
        hist = v["tok_hist"].clone()                               # [B, n]: n-1 tokens newest first + since
        toks = v["ids"].long().view(-1, v["n_tok"])
        n = hist.shape[1]
        for j in range(v["n_tok"]):
            take = (n_commit.long() > j)[:, None]
            t = toks[:, j:j + 1]
            shifted = torch.cat([t, hist[:, :n - 2], torch.where(t == cfg.eos_token_id, torch.zeros_like(t),
                                                                 hist[:, -1:] + 1)], 1)
            hist = torch.where(take, shifted, hist)
        self.c.tok_hist[v["slots"].long()] = hist

    def _attn(self, x, p, ai, slots, positions, n_tok):
        cfg, c = self.cfg, self.c
        proj = self._mm(x, p["proj"])
        q, gate, iq = ops.qsa_prep(proj, p["qn"], p["kn"], p["iqn"], p["ikn"], self.rope, c.k[ai], c.v[ai],
                                   c.block_table, slots, positions, c.kr_ring[ai], c.comp[ai], cfg, n_tok)
        sel, sparse = ops.qsa_select(iq, c.comp[ai], slots, positions, cfg, n_tok)
        o = ops.attn_decode(q, gate, c.k[ai], c.v[ai], c.block_table, slots, positions, sel, sparse, cfg, n_tok)
        return self._mm(o, p["o"])

    def _moe(self, x, p, h, inj):
        if self.ep is not None:
            self.ep.moe(self, x, p, h, inj)
            return
        cfg = self.cfg
        T = x.shape[0]
        E = cfg.n_experts
        logits = self._mm(x, p["router"])
        if self.capture is not None:
            self.capture.record(self._layer, x, logits[:, :E])
        side = self._side_stream(x)
        if side is not None:  # the shared expert runs concurrently with the routed experts (graph-capturable)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                sact = self._mm(x, p["sgu"], epi=wgemm.EPI_SILU_MUL, out_dtype=self.act)
                ysh = self._mm(sact, p["sd"])
        ids, w = ops.moe_route(logits, E, cfg.top_k)
        P = T * cfg.top_k
        gemv = x.is_cuda and GEMV_MOE and P <= GEMV_PAIRS_PER_EXPERT * E   # decode-sized: CUDA-core GEMV
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
        if side is not None:
            torch.cuda.current_stream().wait_stream(side)
            ysh.record_stream(torch.cuda.current_stream())
            sact.record_stream(torch.cuda.current_stream())
        else:
            sact = self._mm(x, p["sgu"], epi=wgemm.EPI_SILU_MUL, out_dtype=self.act)
            ysh = self._mm(sact, p["sd"])
        ops.moe_combine(h, ypair, pair_pos, w, ysh, logits[:, E], inj)

    def _side_stream(self, x):
        if not (x.is_cuda and SIDE_STREAM):
            return None
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=x.device)
        return self._side

    # ------------------------------------------------------------------------------------------- step
    def step(self, ids: torch.Tensor, slots: torch.Tensor, positions: torch.Tensor, n_tok: int = 1,
             verify: bool = False):
        """``verify``: speculative verification of n_tok tokens per sequence. Recurrent (GDN) states are not
        written back; the layer inputs are kept so :meth:`commit` can apply exactly the accepted prefix, and the
        PLE token history is snapshotted for the same reason. Attention caches are position-indexed and need no
        rollback (rejected positions are rewritten when real tokens reach them)."""
        h = ops.embed_hc(ids, self.W["embed"], self.cfg.hc_count)
        return self.step_from_h(h, ids, slots, positions, n_tok, verify)

    def step_from_h(self, h, ids, slots, positions, n_tok: int = 1, verify: bool = False):
        cfg, W = self.cfg, self.W
        self._verify = None
        if verify:
            self._verify = {"proj": {}, "slots": slots, "n_tok": n_tok, "ids": ids,
                            "zeros": torch.zeros(slots.shape[0], dtype=torch.int32, device=slots.device)}
            if self.c.tok_hist is not None:
                self._verify["tok_hist"] = self.c.tok_hist[slots.long()].clone()
        if cfg.ple_layers:
            from . import fn_ple
            emb = fn_ple.embed_rows(self, ids, slots, positions, n_tok)
        for l, L in enumerate(W["layers"]):
            if "ple" in L:
                fn_ple.apply(self, h, emb, L["ple"], self.c.ple_hist[cfg.ple_layers.index(l)], slots, positions,
                             n_tok)
            x, inj = self._hc(h, L["ahc"])
            if cfg.layer_kind(l) == "linear":
                y = self._gdn(x, L["mix"], self.lin_idx[l], slots, n_tok)
            else:
                y = self._attn(x, L["mix"], self.attn_idx[l], slots, positions, n_tok)
            ops.hc_residual(h, y, inj)
            x, inj = self._hc(h, L["mhc"])
            self._layer = l
            self._moe(x, L["moe"], h, inj)
        x, _ = self._hc(h, W["mixer"], with_inj=False)
        return x

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return self._mm(x, self.W["lm_head"], f8=False)

    # --------------------------------------------------------------------------------------- helpers
    def assign_blocks(self, slot: int, n_tokens: int, allocator):
        """Make sure slot's block table covers n_tokens positions, taking blocks from `allocator`."""
        bs = self.c.block_size
        need = (n_tokens + bs - 1) // bs
        have = allocator.n_blocks_of(slot)
        if need > have:
            new = allocator.allocate(slot, need - have)
            self.c.block_table[slot, have:need] = torch.tensor(new, dtype=torch.int32, device=self.device)

    def reset_slot(self, slot: int):
        c = self.c
        for t in c.conv + c.ssm + c.kr_ring:
            t[slot].zero_()
        if c.ple_hist is not None:
            for t in c.ple_hist:
                t[slot].zero_()
            c.tok_hist[slot, :-1].fill_(self.cfg.eos_token_id)   # n-gram context before the first token: eos
            c.tok_hist[slot, -1] = 0                              # tokens since the last eos

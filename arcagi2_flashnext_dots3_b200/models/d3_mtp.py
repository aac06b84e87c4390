"""Multi-token-prediction (MTP) draft layer of the D3 model (the reference serves it as its draft model:
dotsnote/engine/vllm_patch/vllm/models/dots3_note/nvidia/mtp.py:34-100 `Dots3NoteMultiTokenPredictorLayer`, the
DeepSeek-V3.2 MTP structure, with its own embedding table, mtp.py:170-185).

At position q the layer reads the main model's final hidden state x_q and the token t_{q+1}:
    u = eh_proj([rms(E_mtp[t_{q+1}], enorm); rms(x_q, hnorm)])          (one tcgen05 GEMM, [H, 2H] FP8)
    x'_q = one D3 decoder layer over u (own latent and index caches), then the shared-head norm
and the main model's LM head on x'_q predicts t_{q+2}. MTP-3 chains the same layer on its own output. Under tensor
parallelism the layer is sharded like the main layers and picks through the main model's (possibly
vocabulary-sharded) head. Weights: :func:`random_d3_mtp` (no trained MTP checkpoint is available offline).
"""
from __future__ import annotations

import dataclasses

import torch

from ..ops import d3_ops as d3
from ..ops import fn_ops as ops
from . import d3_weights
from .d3 import D3Model, allocate_caches


def mtp_config(cfg):
    """The MTP layer's view of a D3 config: one MoE decoder layer with a DSA (indexed) latent attention."""
    return dataclasses.replace(cfg, num_layers=1, n_dsa_layers=1, n_dense_layers=0, index_share=False)


def random_d3_mtp(cfg, device, seed: int = 11, tp=None) -> dict:
    """Random MTP weights: own embedding [V, H], enorm / hnorm, eh_proj [H, 2H], one decoder layer, final norm.
    ``tp=(rank, world)``: the rank's shard of the layer."""
    mc = mtp_config(cfg)
    dev = torch.device(device)
    if dev.type == "cpu" or cfg.hidden_size <= 1024:
        W = d3_weights.to_engine(d3_weights.random_dense(mc, seed=seed), mc, dev)
    else:
        W = d3_weights.random_engine(mc, dev, seed=seed, tp=tp)
    del W["lm_head"]                        # the main model's head is shared
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    H = cfg.hidden_size
    eh = torch.randn(H, 2 * H, generator=g, device=dev) * 0.02
    return {"embed": W["embed"], "norm": W["norm"], "layer": W["layers"][0],
            "enorm": 1.0 + torch.randn(H, generator=g, device=dev) * 0.1,
            "hnorm": 1.0 + torch.randn(H, generator=g, device=dev) * 0.1,
            "eh": d3_weights._ws(eh, mc, dev)}


class D3MTPHead:
    """Serving form of the MTP layer; the interface :class:`..engine.spec.MTPDrafter` drives (``caches``,
    ``step``, ``draft_ids``, ``assign_blocks``, ``reset_slot``)."""

    def __init__(self, cfg, main: D3Model, mtp_W: dict, device, n_slots: int, max_len: int, block_size: int = 64):
        self.cfg, self.main, self.W = cfg, main, mtp_W
        self.mc = mtp_config(cfg)
        if main.tp is not None:            # the layer's heads and experts follow the main model's TP split
            self.mc = dataclasses.replace(self.mc, n_heads=main.cfg.n_heads, swa_n_heads=main.cfg.swa_n_heads)
        self.device = torch.device(device)
        self.caches = allocate_caches(self.mc, device, n_slots, max_len, block_size)
        inner_W = {"embed": mtp_W["embed"], "lm_head": main.W["lm_head"], "norm": mtp_W["norm"],
                   "layers": [mtp_W["layer"]]}
        if "vocab_range" in main.W:
            inner_W["vocab_range"] = main.W["vocab_range"]
        self.inner = D3Model(self.mc, inner_W, self.caches, device, tp=main.tp)

    def step(self, x_prev: torch.Tensor, ids: torch.Tensor, slots, positions, n_tok: int = 1) -> torch.Tensor:
        """x_prev [T, H] (main or previous MTP hidden), ids [T] the next tokens -> MTP hidden [T, H]."""
        cfg, m = self.cfg, self.inner
        e = self.W["embed"][ids.long()].float()
        en = d3.add_rms(e, None, self.W["enorm"], cfg.rms_eps, m.act)
        xn = d3.add_rms(x_prev.float().contiguous(), None, self.W["hnorm"], cfg.rms_eps, m.act)
        u = m._mm(torch.cat([en, xn], 1).contiguous(), self.W["eh"])
        return m.step_from_h(u, slots, positions, n_tok)

    def logits(self, x):
        return self.inner.logits(x)

    def draft_ids(self, x) -> torch.Tensor:
        """Greedy draft per row (int32) through the shared head (cross-rank pick when it is vocabulary-sharded)."""
        if self.inner.vocab_sharded:
            return self.inner.pick(x)
        return ops.argmax(self.inner.logits(x)).to(torch.int32)

    def assign_blocks(self, slot, n_tokens, allocator):
        self.inner.assign_blocks(slot, n_tokens, allocator)

    def reset_slot(self, slot):
        self.inner.reset_slot(slot)

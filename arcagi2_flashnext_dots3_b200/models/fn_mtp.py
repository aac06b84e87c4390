"""Multi-token-prediction (MTP) draft head of the FN-shaped model.

Structure (the reference serves the checkpoint's MTP layer, indexed as layer 48, as its draft model:
flashnext/kaggle/README.md:30, fnext/mtp/fnmtp.py): at position q the head reads the main model's final hidden
state x_q and the embedding of token t_{q+1}, normalizes both, projects [e; x] to the hidden size, runs one
attention + MoE layer with its own KV cache (hyper-connection streams initialised from the projection), mixes the
streams and applies the shared LM head; its output predicts t_{q+2}. Later drafts chain on the head's own hidden
output. Weights: :func:`random_mtp` (no MTP checkpoint is available offline).
"""
from __future__ import annotations

import dataclasses

import torch

from ..ops import fn_ops as ops
from ..ops import wgemm
from . import fn_weights
from .fn import FNModel, allocate_caches


def mtp_config(cfg):
    return dataclasses.replace(cfg, num_layers=1, full_attn_interval=1, ple_layers=())


def random_mtp(cfg, device, seed: int = 7) -> dict:
    """Random MTP weights: fc [H, 2H], two RMSNorm weights, one attention+MoE layer and a stream mixer."""
    mc = mtp_config(cfg)
    if torch.device(device).type == "cpu" or cfg.hidden_size <= 1024:
        W = fn_weights.to_engine(fn_weights.random_dense(mc, seed=seed, symmetric=False), mc, device)
    else:
        W = fn_weights.random_engine(mc, device, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    H = cfg.hidden_size
    fc = torch.randn(H, 2 * H, generator=g) * 0.02
    return {"fc": fn_weights._ws(fc, mc, device), "pe": (torch.randn(H, generator=g) * 0.1).to(device),
            "ph": (torch.randn(H, generator=g) * 0.1).to(device), "layer": W["layers"][0], "mixer": W["mixer"]}


class MTPHead:
    def __init__(self, cfg, main_W: dict, mtp_W: dict, device, n_slots: int, max_len: int, block_size: int = 64,
                 kv_dtype: str = "fp8", hot_ids: torch.Tensor = None):
        """``hot_ids``: token ids of the draft vocabulary (the reference drafts over the 32,768 hottest tokens,
        fnext/mtp/fnmtp.py:46). Their LM-head rows go into a separate fp16 weight set holding the exact operand
        values the tensor core reads for those rows of the full head (``rt.tensor_core_operands``), so on the GPU a
        draft step computes the full head's products restricted to the hot rows while reading only that share of
        the head. The rows are not re-quantized: FP8 would need new 128x128 block scales, and the hot logits
        would then differ from the full head's."""
        self.cfg = cfg
        self.mc = mtp_config(cfg)
        self.W = mtp_W
        self.main_W = main_W
        self.caches = allocate_caches(self.mc, device, n_slots, max_len, block_size, kv_dtype=kv_dtype)
        inner_W = {"embed": main_W["embed"], "lm_head": main_W["lm_head"], "mixer": mtp_W["mixer"],
                   "layers": [mtp_W["layer"]]}
        self.inner = FNModel(self.mc, inner_W, self.caches, device)
        self.device = torch.device(device)
        self.hot = None
        if hot_ids is not None:
            from ..formats import runtime as rt
            ws = main_W["lm_head"]
            f = ws.fmts[0]
            blob = ws.blob[: ws.row_tiles * ws.kg * rt.block_bytes(f)].view(ws.row_tiles, ws.kg, rt.block_bytes(f))
            rows = rt.tensor_core_operands(blob, f, ws.rows, ws.K)[hot_ids.to(blob.device).long()]
            self.hot = hot_ids.to(device=self.device, dtype=torch.int32)
            self.ws_hot = wgemm.dense_f16(rows, device)
            del rows

    def step(self, x_prev: torch.Tensor, ids: torch.Tensor, slots, positions, n_tok: int = 1) -> torch.Tensor:
        """x_prev [T, H] (main or previous MTP hidden), ids [T] next tokens -> MTP hidden [T, H] (act)."""
        cfg, H = self.cfg, self.cfg.hidden_size
        e = ops.embed_hc(ids, self.main_W["embed"], 1)
        en = ops.hc_prenorm(e, self.W["pe"], 1, H, cfg.rms_eps)
        xn = ops.hc_prenorm(x_prev.float().contiguous(), self.W["ph"], 1, H, cfg.rms_eps)
        u = self.inner._mm(torch.cat([en, xn], 1).contiguous(), self.W["fc"])
        h = u.repeat(1, cfg.hc_count).contiguous()
        return self.inner.step_from_h(h, ids, slots, positions, n_tok)

    def logits(self, x):
        return self.inner.logits(x)

    def draft_ids(self, x) -> torch.Tensor:
        """Greedy draft token per row (int32): argmax over the hot vocabulary when one is set, else the full head."""
        if self.hot is None:
            return ops.argmax(self.logits(x)).to(torch.int32)
        return self.hot[ops.argmax(self.inner._mm(x, self.ws_hot)).long()]

    def assign_blocks(self, slot, n_tokens, allocator):
        self.inner.assign_blocks(slot, n_tokens, allocator)

    def reset_slot(self, slot):
        self.inner.reset_slot(slot)


def random_mtp_dense(cfg, seed: int = 7) -> dict:
    """Dense (trainable) form of the MTP weights: fc [H, 2H] rounded to its storage format, the two input-norm
    weights, one attention + MoE layer and the stream mixer in the dense layout of :func:`fn_weights.random_dense`."""
    mc = mtp_config(cfg)
    D = fn_weights.random_dense(mc, seed=seed, symmetric=False)
    g = torch.Generator().manual_seed(seed + 1)
    H = cfg.hidden_size
    return {"fc": fn_weights._round_dense(torch.randn(H, 2 * H, generator=g) * 0.02, mc),
            "pe": torch.randn(H, generator=g) * 0.1, "ph": torch.randn(H, generator=g) * 0.1,
            "layer": D["layers"][0], "mixer": D["mixer"]}


def mtp_to_engine(dense: dict, cfg, main_dense: dict, device) -> dict:
    """Dense MTP weights (e.g. a trained draft head's export) -> the engine form :class:`MTPHead` serves."""
    mc = mtp_config(cfg)
    E = fn_weights.to_engine({"embed": main_dense["embed"], "lm_head": main_dense["lm_head"], "mixer": dense["mixer"],
                              "layers": [dense["layer"]]}, mc, device)
    return {"fc": fn_weights._ws(fn_weights._round_dense(dense["fc"].float(), mc), mc, device),
            "pe": dense["pe"].float().to(device), "ph": dense["ph"].float().to(device), "layer": E["layers"][0],
            "mixer": E["mixer"]}

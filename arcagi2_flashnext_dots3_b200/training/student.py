"""Differentiable Flash-Next-shaped student for repair training.

Mirrors the reference's plain-PyTorch student (flashnext/training/student/student_fn.py:589 `Student`): frozen
dense weights, frozen expert codes, and three trainable groups (`--trainable scales,router[,norms]`,
flashnext/training/rl/train_rl.py:63):

* per-expert log-scale offsets t (s = s0 * exp(t), student_fn.py:492-505), one tensor per projection and layer;
* the router rows (softmax over the kept experts, top-k renormalized, student_fn.py:516-519);
* optionally the hyper-connection RMSNorm weights.

The layer math is the oracle's (:mod:`..models.fn_reference`), with the pieces that loop over time replaced for
training: the gated delta rule runs chunked (:mod:`.gdn_chunk`), the QSA block selection is vectorized (no
gradient flows through the selection, as in the reference) and attention is one masked
``scaled_dot_product_attention``; experts run through :class:`.lowbit.GroupedExperts`.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from ..models import fn_reference as R
from .gdn_chunk import chunk_gated_delta_rule
from .lowbit import ExpertBank, grouped_experts


def _to(obj, device):
    if isinstance(obj, torch.Tensor):
        return obj.to(device)
    if isinstance(obj, dict):
        return {k: (v if k in ("lowbit", "experts_dense") else _to(v, device)) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_to(v, device) for v in obj]
    return obj


def gdn_train(x, p, cfg):
    """fn_reference.gdn with the recurrence computed chunked."""
    T = x.shape[0]
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    qkv = x @ p["qkv"].t()
    C = qkv.shape[1]
    kc = p["conv"].shape[-1]
    qkv = F.silu(F.conv1d(F.pad(qkv.t()[None], (kc - 1, 0)), p["conv"], groups=C)[0].t())
    q, k, v = qkv.split([nk * dk, nk * dk, nv * dv], -1)
    q, k, v = q.view(T, nk, dk), k.view(T, nk, dk), v.view(T, nv, dv)
    z = (x @ p["z"].t()).view(T, nv, dv)
    beta = torch.sigmoid(x @ p["b"].t())
    g = -p["A_log"].float().exp() * F.softplus(x @ p["a"].t() + p["dt_bias"].float())
    r = nv // nk
    q, k = q.repeat_interleave(r, 1), k.repeat_interleave(r, 1)
    q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
    o = chunk_gated_delta_rule(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), g.t(), beta.t())
    o = o.transpose(0, 1)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * p["norm"].float()
    o = o * (torch.sigmoid(z) if cfg.gdn_gate == "sigmoid" else F.silu(z))
    return o.reshape(T, -1) @ p["out"].t()


@torch.no_grad()
def qsa_select_vec(x, p, cfg, cos, sin, q_chunk: int = 1024):
    """Vectorized fn_reference.qsa_select: [T, nb] kept-block mask or None."""
    T, r = x.shape[0], cfg.indexer_ratio
    nblk = cfg.indexer_blocks
    nb = T // r
    ncomp = (torch.arange(T, device=x.device) + 1) // r
    if nb == 0 or int(ncomp.max()) <= nblk:
        return None
    iH, iD = cfg.indexer_heads, cfg.indexer_dim
    qk = x @ p["iqk"].t()
    q, kr = qk.split([iH * iD, iD], -1)
    q = R.rope_part(R.rms1p(q.view(T, iH, iD), p["iqn"], cfg.rms_eps), cos, sin)
    kb = R.rms1p(kr[: nb * r].view(nb, r, iD).mean(1), p["ikn"], cfg.rms_eps)
    bstart = torch.arange(nb, device=x.device) * r
    kb = R.rope_part(kb[:, None], cos[bstart], sin[bstart])[:, 0]
    SB = torch.arange(nb, device=x.device)[None, :] < ncomp[:, None]
    k_sel = min(nblk, nb)
    for a in range(0, T, q_chunk):
        b = min(T, a + q_chunk)
        need = ncomp[a:b] > nblk
        if not bool(need.any()):
            continue
        s = torch.relu(torch.einsum("thd,bd->thb", q[a:b], kb)).sum(1) / math.sqrt(iD)
        s = s.masked_fill(~SB[a:b], float("-inf"))
        top = torch.sort(s, dim=-1, descending=True, stable=True).indices[:, :k_sel]  # ties: lower block first
        picked = torch.zeros(b - a, nb, dtype=torch.bool, device=x.device).scatter_(1, top, True)
        SB[a:b] = torch.where(need[:, None], picked, SB[a:b])
    return SB


def qsa_train(x, p, cfg, cos, sin):
    T = x.shape[0]
    Hq, KV, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    SB = qsa_select_vec(x, p, cfg, cos, sin)
    qg = (x @ p["q"].t()).view(T, Hq, 2 * D)
    q, gate = qg[..., :D], qg[..., D:]
    q = R.rope_part(R.rms1p(q, p["qn"], cfg.rms_eps), cos, sin)
    k = R.rope_part(R.rms1p((x @ p["k"].t()).view(T, KV, D), p["kn"], cfg.rms_eps), cos, sin)
    v = (x @ p["v"].t()).view(T, KV, D)
    qi = torch.arange(T, device=x.device)[:, None]
    ki = torch.arange(T, device=x.device)[None, :]
    allowed = ki <= qi
    if SB is not None:
        r = cfg.indexer_ratio
        sel = torch.gather(SB, 1, (ki // r).expand(T, T).clamp_max(SB.shape[1] - 1))
        allowed = allowed & (sel | (ki >= ((qi + 1) // r) * r))
    rep = Hq // KV
    o = F.scaled_dot_product_attention(q.transpose(0, 1), k.repeat_interleave(rep, 1).transpose(0, 1),
                                       v.repeat_interleave(rep, 1).transpose(0, 1), attn_mask=allowed[None])
    o = o.transpose(0, 1).reshape(T, -1) * torch.sigmoid(gate.reshape(T, -1))
    return o @ p["o"].t()


class MoETrain(nn.Module):
    """One MoE layer: trainable router rows and expert log-scale offsets; frozen codes and shared expert."""

    def __init__(self, moe: dict, cfg, device):
        super().__init__()
        self.cfg = cfg
        self.bank = ExpertBank.from_lowbit(moe["lowbit"], device)
        self.router = nn.Parameter(moe["gate"].float().to(device).clone())
        self.t_gu = nn.Parameter(torch.zeros_like(self.bank.s0["gu"]))
        self.t_d = nn.Parameter(torch.zeros_like(self.bank.s0["d"]))
        self.frozen = {k: moe[k].float().to(device) for k in ("sgu", "sd", "sgate")}

    def scales(self):
        return self.bank.s0["gu"] * self.t_gu.exp(), self.bank.s0["d"] * self.t_d.exp()

    def forward(self, x):
        cfg, k = self.cfg, self.cfg.top_k
        T, H = x.shape
        pr = torch.softmax(x @ self.router.t(), -1)
        w, ids = torch.topk(pr, k, -1)
        w = w / w.sum(-1, keepdim=True)
        flat = ids.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=self.bank.E).tolist()
        xs = x.repeat_interleave(k, 0)[order]
        s_gu, s_d = self.scales()
        ys = grouped_experts(xs, s_gu, s_d, counts, self.bank)
        y = torch.zeros(T * k, H, dtype=ys.dtype, device=x.device).index_copy(0, order, ys)
        out = (y.view(T, k, H) * w[..., None]).sum(1)
        f = self.frozen
        g, u = (x @ f["sgu"].t()).chunk(2, -1)
        return out + torch.sigmoid(x @ f["sgate"].t()) * ((F.silu(g) * u) @ f["sd"].t())


class FNStudent(nn.Module):
    def __init__(self, cfg, W: dict, device, train_norms: bool = False, layer_offset: int = 0):
        """``layer_offset``: W["layers"] holds layers layer_offset.. of the model (a pipeline stage)."""
        super().__init__()
        self.cfg = cfg
        self.l0 = layer_offset
        self.device = torch.device(device)
        Wd = _to({k: v for k, v in W.items() if k != "layers"}, self.device)
        Wd["layers"] = [_to({k: v for k, v in L.items() if k != "moe"}, self.device) for L in W["layers"]]
        self.W = Wd
        self.moe = nn.ModuleList([MoETrain(L["moe"], cfg, self.device) for L in W["layers"]])
        self.norms = nn.ParameterList()
        if train_norms:
            for L in self.W["layers"]:
                for key in ("ahc", "mhc"):
                    prm = nn.Parameter(L[key]["norm"].float().clone())
                    L[key]["norm"] = prm
                    self.norms.append(prm)

    def _layer(self, l, h, emb, cos, sin):
        cfg, L = self.cfg, self.W["layers"][l]
        hc, H = cfg.hc_count, cfg.hidden_size
        if "ple" in L:
            h = h + R.ple(h, emb, L["ple"], cfg)
        x, inj = R.gated_residual(h, L["ahc"], hc, H, cfg.rms_eps)
        if cfg.layer_kind(l + self.l0) == "linear":
            y = gdn_train(x, L["mix"], cfg)
        else:
            y = qsa_train(x, L["mix"], cfg, cos, sin)
        h = h + (y.unsqueeze(-2) * inj.unsqueeze(-1)).flatten(-2)
        x, inj = R.gated_residual(h, L["mhc"], hc, H, cfg.rms_eps)
        y = self.moe[l](x)
        return h + (y.unsqueeze(-2) * inj.unsqueeze(-1)).flatten(-2)

    def hidden(self, ids: torch.Tensor, ckpt: bool = False) -> torch.Tensor:
        """Final mixed hidden state [T, H] of one sequence (input to the LM head)."""
        cfg, W = self.cfg, self.W
        ids = ids.to(self.device)
        T = ids.shape[0]
        cos, sin = R.rope_cos_sin(torch.arange(T), cfg.rope_dim, cfg.rope_theta)
        cos, sin = cos.to(self.device), sin.to(self.device)
        h = W["embed"][ids].float().repeat(1, cfg.hc_count)
        emb = R.ple_embed(ids, W, cfg) if cfg.ple_layers else None
        for l in range(len(W["layers"])):
            if ckpt and torch.is_grad_enabled():
                h = checkpoint(self._layer, l, h, emb, cos, sin, use_reentrant=False)
            else:
                h = self._layer(l, h, emb, cos, sin)
        return R.gated_residual(h, W["mixer"], cfg.hc_count, cfg.hidden_size, cfg.rms_eps, combine=False)

    @property
    def lm_head(self):
        return self.W["lm_head"]

    def logits(self, ids: torch.Tensor) -> torch.Tensor:
        return self.hidden(ids) @ self.lm_head.float().t()

    def param_groups(self, lr_scales=3e-4, lr_router=1.5e-5, lr_norms=1e-5):
        """Adam groups with the reference's learning rates (train_rl.py:64-66)."""
        groups = [{"params": [p for m in self.moe for p in (m.t_gu, m.t_d)], "lr": lr_scales, "name": "scales"},
                  {"params": [m.router for m in self.moe], "lr": lr_router, "name": "router"}]
        if len(self.norms):
            groups.append({"params": list(self.norms), "lr": lr_norms, "name": "norms"})
        return groups

    def export_scales(self) -> list:
        """Per layer {"gu_s", "d_s"} fp16 [E, R, KG] = fp16(s0 * exp(t)) and the fp16 router rows."""
        out = []
        with torch.no_grad():
            for m in self.moe:
                s_gu, s_d = m.scales()
                out.append({"gu_s": s_gu.half().cpu(), "d_s": s_d.half().cpu(), "router": m.router.half().cpu()})
        return out

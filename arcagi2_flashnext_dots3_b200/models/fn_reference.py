"""Dense fp32 reference (oracle) of the Flash-Next-shaped model, full-sequence, one sequence at a time.

This follows the math of the reference's differentiable student (flashnext/training/student/student_fn.py):
``rms1p`` (:58), partial RoPE (:67-80), hyper-connection ``GatedResidual`` (:232), ``GDN`` (:251, the gated delta
rule with L2-normed q/k, decay -exp(A_log)*softplus(a+dt_bias), gated RMSNorm output), ``QSA`` (:295, q/k RMSNorm,
partial RoPE, sigmoid output gate, GQA, and the compressed-block indexer that keeps the top `budget/ratio` blocks per
query once a query has more complete blocks than that), ``PLE`` (:380, xor-hash n-gram embedding, gated and
dilated-conv mixed into every hyper-connection stream), ``MoE`` (:461, softmax router over the kept experts, top-k
renormalized, plus a sigmoid-gated shared expert) and the layer wiring (:578).

Everything is written with explicit loops over time where the reference uses chunked library kernels, so it is a
slow but independent oracle for the engine's incremental (prefill + decode) path.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms1p(x, w, eps, group=None):
    xf = x.float()
    if group is not None:
        xf = xf.view(*xf.shape[:-1], -1, group)
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if group is not None:
        xf = xf.flatten(-2)
    return xf * (1.0 + w.float())


def rope_cos_sin(pos: torch.Tensor, rd: int, theta: float):
    inv = 1.0 / theta ** (torch.arange(0, rd, 2, dtype=torch.float64) / rd)
    f = pos.double()[:, None] * inv[None]
    e = torch.cat([f, f], -1)
    return e.cos().float(), e.sin().float()


def rope_part(x, cos, sin):
    """Rotate the first rd dims of x [T, h, d] (neox half-split)."""
    rd = cos.shape[-1]
    c, s = cos[:, None, :], sin[:, None, :]
    xr, xp = x[..., :rd], x[..., rd:]
    x1, x2 = xr[..., : rd // 2], xr[..., rd // 2:]
    rot = torch.cat([-x2, x1], -1)
    return torch.cat([xr * c + rot * s, xp], -1)


def gated_residual(h, p, hc, H, eps, combine=True):
    hn = rms1p(h, p["norm"], eps, H)
    w = F.silu(hn @ p["down"].t() / hc)
    w = torch.sigmoid(w @ p["up"].t())
    mixed = (w.unflatten(-1, (hc, H)) * hn.unflatten(-1, (hc, H))).mean(-2)
    if not combine:
        return mixed
    return mixed, 2 * torch.sigmoid(hn @ p["inj"].t() / hc)


def gdn(x, p, cfg):
    T = x.shape[0]
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    qkv = x @ p["qkv"].t()
    C = qkv.shape[1]
    kc = p["conv"].shape[-1]
    qkv = F.conv1d(F.pad(qkv.t()[None], (kc - 1, 0)), p["conv"], groups=C)[0].t()
    qkv = F.silu(qkv)
    q, k, v = qkv.split([nk * dk, nk * dk, nv * dv], -1)
    q, k, v = q.view(T, nk, dk), k.view(T, nk, dk), v.view(T, nv, dv)
    z = (x @ p["z"].t()).view(T, nv, dv)
    beta = torch.sigmoid(x @ p["b"].t())
    g = -p["A_log"].float().exp() * F.softplus(x @ p["a"].t() + p["dt_bias"].float())
    r = nv // nk
    q, k = q.repeat_interleave(r, 1), k.repeat_interleave(r, 1)
    q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
    S = torch.zeros(nv, dk, dv)
    o = torch.empty(T, nv, dv)
    for t in range(T):
        S = S * g[t].exp()[:, None, None]
        kv = torch.einsum("hkv,hk->hv", S, k[t])
        u = beta[t][:, None] * (v[t] - kv)
        S = S + k[t][:, :, None] * u[:, None, :]
        o[t] = torch.einsum("hkv,hk->hv", S, q[t])
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * p["norm"].float()
    o = o * (torch.sigmoid(z) if cfg.gdn_gate == "sigmoid" else F.silu(z))
    return o.reshape(T, -1) @ p["out"].t()


def qsa_select(x, p, cfg, cos, sin):
    """Block-selection mask SB [T, nb] (True = block kept) or None when no query exceeds the budget."""
    T, r = x.shape[0], cfg.indexer_ratio
    nblk = cfg.indexer_blocks
    nb = T // r
    ar = torch.arange(T)
    ncomp = (ar + 1) // r
    if int(ncomp.max()) <= nblk:
        return None
    iH, iD = cfg.indexer_heads, cfg.indexer_dim
    qk = x @ p["iqk"].t()
    q, kr = qk.split([iH * iD, iD], -1)
    q = rope_part(rms1p(q.view(T, iH, iD), p["iqn"], cfg.rms_eps), cos, sin)
    kb = kr[: nb * r].view(nb, r, iD).mean(1)
    kb = rms1p(kb, p["ikn"], cfg.rms_eps)
    bstart = torch.arange(nb) * r
    kb = rope_part(kb[:, None], cos[bstart], sin[bstart])[:, 0]
    SB = torch.zeros(T, nb, dtype=torch.bool)
    for i in range(T):
        nc = int(ncomp[i])
        if nc <= nblk:
            SB[i, :nc] = True
            continue
        s = torch.relu(torch.einsum("hd,bd->hb", q[i], kb[:nc])).sum(0) / math.sqrt(iD)
        SB[i, s.topk(nblk).indices] = True
    return SB


def qsa(x, p, cfg, cos, sin):
    T = x.shape[0]
    Hq, KV, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    SB = qsa_select(x, p, cfg, cos, sin)
    qg = (x @ p["q"].t()).view(T, Hq, 2 * D)
    q, gate = qg[..., :D], qg[..., D:]
    q = rope_part(rms1p(q, p["qn"], cfg.rms_eps), cos, sin)
    k = rope_part(rms1p((x @ p["k"].t()).view(T, KV, D), p["kn"], cfg.rms_eps), cos, sin)
    v = (x @ p["v"].t()).view(T, KV, D)
    qi = torch.arange(T)[:, None]
    ki = torch.arange(T)[None, :]
    allowed = ki <= qi
    if SB is not None:
        r = cfg.indexer_ratio
        blk = (ki // r).expand(T, T)
        sel = torch.gather(SB, 1, blk.clamp_max(SB.shape[1] - 1))
        tail = ki >= ((qi + 1) // r) * r
        allowed = allowed & (sel | tail)
    rep = Hq // KV
    k = k.repeat_interleave(rep, 1)
    v = v.repeat_interleave(rep, 1)
    s = torch.einsum("qhd,khd->hqk", q, k) * D ** -0.5
    s = s.masked_fill(~allowed[None], float("-inf"))
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)
    o = o.reshape(T, -1) * torch.sigmoid(gate.reshape(T, -1))
    return o @ p["o"].t()


def moe(x, p, cfg):
    logits = x @ p["gate"].float().t()
    pr = torch.softmax(logits, -1)
    w, ids = torch.topk(pr, cfg.top_k, -1)
    w = w / w.sum(-1, keepdim=True)
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(cfg.top_k):
            e = int(ids[t, j])
            wgu, wd = p["experts_dense"][e]
            g, u = (x[t] @ wgu.t()).chunk(2, -1)
            out[t] += w[t, j] * ((F.silu(g) * u) @ wd.t())
    g, u = (x @ p["sgu"].t()).chunk(2, -1)
    sh = torch.sigmoid(x @ p["sgate"].t()) * ((F.silu(g) * u) @ p["sd"].t())
    return out + sh


def ngram_ids(ids: torch.Tensor, cfg, mult, offs, sizes):
    """xor-hash n-gram row ids [T, heads] (student_fn.py:413-433); n-grams restart after each eos."""
    n, hpn, eos = cfg.ngram_size, cfg.heads_per_ngram, cfg.eos_token_id
    ctx = n - 1
    dev = ids.device
    hist = torch.cat([torch.full((ctx,), eos, dtype=torch.long, device=dev), ids.long()])
    L = hist.shape[0]
    pos = torch.arange(L, device=dev)
    eosp = torch.where(hist == eos, pos, -1)
    prev = torch.cat([torch.tensor([-1], device=dev), torch.cummax(eosp, 0).values[:-1]])
    pis = pos - (prev + 1)
    sh = []
    for s in range(n):
        src = pos - s
        v = hist[src.clamp_min(0)]
        ok = (pis >= s) & (src >= 0)
        sh.append(torch.where(ok, v, torch.full_like(v, eos)))
    blocks = []
    for ng in range(2, n + 1):
        a, b = (ng - 2) * hpn, (ng - 1) * hpn
        mixed = sh[0] * mult[0]
        for q in range(1, ng):
            mixed = torch.bitwise_xor(mixed, sh[q] * mult[q])
        blocks.append(torch.remainder(mixed[:, None], sizes[a:b][None]) + offs[a:b][None])
    return torch.cat(blocks, -1)[ctx:]


def ple(h, emb, p, cfg):
    hc, H = cfg.hc_count, cfg.hidden_size
    T = h.shape[0]
    key = rms1p(emb @ p["kp"].t(), p["nk"], cfg.rms_eps, H).unflatten(-1, (hc, H))
    val = emb @ p["vp"].t()
    qn = rms1p(h, p["nq"], cfg.rms_eps, H).unflatten(-1, (hc, H))
    gate = (key * qn).sum(-1, keepdim=True) / math.sqrt(H)
    gate = gate.abs().clamp_min(1e-6).sqrt() * gate.sign()
    gv = torch.sigmoid(gate) * val[:, None, :]
    gvn = rms1p(gv.flatten(-2), p["nc"], cfg.rms_eps, H)
    gv = gv.flatten(-2)
    dil = cfg.ngram_size
    pad = (p["conv"].shape[-1] - 1) * dil
    c = F.conv1d(F.pad(gvn.t()[None], (pad, 0)), p["conv"], groups=gvn.shape[1], dilation=dil)[0].t()
    return gv + F.silu(c)


def ple_embed(ids, W, cfg):
    rows = ngram_ids(ids, cfg, W["ple_mult"], W["ple_offs"], W["ple_sizes"])
    emb = W["ple_table"][rows.clamp_max(W["ple_table"].shape[0] - 1)].float() * W["ple_scale"]
    return emb.reshape(ids.shape[0], -1)


@torch.no_grad()
def forward(W: dict, cfg, ids: torch.Tensor) -> torch.Tensor:
    """Logits [T, V] (fp32) of one sequence."""
    T = ids.shape[0]
    hc, H = cfg.hc_count, cfg.hidden_size
    cos, sin = rope_cos_sin(torch.arange(T), cfg.rope_dim, cfg.rope_theta)
    h = W["embed"][ids].float().repeat(1, hc)
    emb = ple_embed(ids, W, cfg) if cfg.ple_layers else None
    for l, L in enumerate(W["layers"]):
        if "ple" in L:
            h = h + ple(h, emb, L["ple"], cfg)
        x, inj = gated_residual(h, L["ahc"], hc, H, cfg.rms_eps)
        y = gdn(x, L["mix"], cfg) if cfg.layer_kind(l) == "linear" else qsa(x, L["mix"], cfg, cos, sin)
        h = h + (y.unsqueeze(-2) * inj.unsqueeze(-1)).flatten(-2)
        x, inj = gated_residual(h, L["mhc"], hc, H, cfg.rms_eps)
        y = moe(x, L["moe"], cfg)
        h = h + (y.unsqueeze(-2) * inj.unsqueeze(-1)).flatten(-2)
    x = gated_residual(h, W["mixer"], hc, H, cfg.rms_eps, combine=False)
    return x @ W["lm_head"].float().t()


@torch.no_grad()
def greedy(W, cfg, prompt: torch.Tensor, n_new: int) -> list:
    """Greedy continuation by full recomputation (slow oracle)."""
    ids = prompt.clone()
    out = []
    for _ in range(n_new):
        nxt = int(forward(W, cfg, ids)[-1].argmax())
        out.append(nxt)
        ids = torch.cat([ids, torch.tensor([nxt])])
    return out

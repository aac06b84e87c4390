"""Dense fp32 reference (oracle) of the Dots3-Note-shaped model, full sequence, one sequence at a time.

Math of the reference's D3 student (dotsnote/training/finetune/student.py): ``rms`` (:58, weight w not 1+w),
interleaved RoPE ``rope_inter`` (:66), the FP8 round trip of the cached latent ``kvq`` (:103), MLA attention
``Attn.forward`` (:231-259: q/kv LoRA with RMSNorm and sqrt(hidden/rank) rescale, decoupled RoPE key shared by
all heads, headwise sigmoid gate ``g_proj``), the DSA indexer mask ``Attn.dsa_mask`` (:209-229: ReLU scores of
``index_heads`` query heads against one LayerNorm'd key per token, weighted by ``weights_proj``, top-`index_topk`
causal positions, full causal attention while a query has no more than `index_topk` predecessors), sliding-window
layers (window `swa_window` including the query), ``MoE.forward`` (:322-343: sigmoid scores, top-k by score +
correction bias, weights = renormalized scores, times the routed scaling factor, plus the shared expert) and the
pre-norm layer (:353-362).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def rope_tab(pos: torch.Tensor, dim: int, theta: float):
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, dtype=torch.float64, device=pos.device) / dim)
    f = pos.double()[:, None] * inv[None]
    return f.cos().float(), f.sin().float()


def rope_inter(x, cos, sin):
    """x [T, h, d] with d = 2 * cos.shape[-1]; pairs (2i, 2i+1) rotate together."""
    c, s = cos[:, None, :], sin[:, None, :]
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x1 * c - x2 * s, x2 * c + x1 * s], -1).flatten(-2)


def kvq(t):
    return t.to(torch.float8_e4m3fn).float()


def dsa_mask(x, qc, p, cfg, cos, sin):
    T = x.shape[0]
    if T <= cfg.index_topk:
        return None
    iH, iD, dr = cfg.index_heads, cfg.index_dim, cfg.qk_rope_dim
    q = (qc @ p["iq"].t()).view(T, iH, iD)
    k = F.layer_norm(x @ p["ik"].t(), (iD,), p["ik_w"], p["ik_b"], 1e-6)
    q = torch.cat([rope_inter(q[..., :dr], cos, sin), q[..., dr:]], -1)
    k = torch.cat([rope_inter(k[:, None, :dr], cos, sin)[:, 0], k[:, dr:]], -1)
    w = (x @ p["iw"].t()) * iD ** -0.5 * iH ** -0.5
    s = torch.relu(torch.einsum("qhd,kd->qhk", q, k))
    lg = torch.einsum("qhk,qh->qk", s, w)
    ar = torch.arange(T, device=x.device)
    lg = lg.masked_fill(ar[None, :] > ar[:, None], float("-inf"))
    M = torch.zeros(T, T, dtype=torch.bool, device=x.device)
    # ties (ReLU makes exact zeros common) resolve to the lower position, the rule of the engine's radix select
    idx = torch.sort(lg, dim=-1, descending=True, stable=True).indices[:, : cfg.index_topk]
    M.scatter_(1, idx, True)
    causal = ar[None, :] <= ar[:, None]
    M = M & causal
    M[: cfg.index_topk] = causal[: cfg.index_topk]
    return M


def mla(x, p, cfg, l, cos, sin):
    T = x.shape[0]
    H, kvr = cfg.heads_of(l), cfg.latent_of(l)
    dn, dr, dv, qr = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.q_lora_rank
    qs = (cfg.hidden_size / qr) ** 0.5 if cfg.kv_rescale else 1.0
    kvs = (cfg.hidden_size / kvr) ** 0.5 if cfg.kv_rescale else 1.0
    qc = rms(x @ p["q_a"].t(), p["q_ln"], cfg.rms_eps) * qs
    kvc, kpe = (x @ p["kv_a"].t()).split([kvr, dr], -1)
    kvc = kvq(rms(kvc, p["kv_ln"], cfg.rms_eps) * kvs)
    kpe = rms(kpe, p["kr_ln"], cfg.rms_eps)
    q = (qc @ p["q_b"].t()).view(T, H, dn + dr)
    q = torch.cat([q[..., :dn], rope_inter(q[..., dn:], cos, sin)], -1)
    kpe = kvq(rope_inter(kpe[:, None, :], cos, sin))
    kv = (kvc @ p["kv_b"].t()).view(T, H, dn + dv)
    k = torch.cat([kv[..., :dn], kpe.expand(T, H, dr)], -1)
    v = kv[..., dn:]
    ar = torch.arange(T)
    allowed = ar[None, :] <= ar[:, None]
    if cfg.layer_kind(l) == "swa":
        allowed = allowed & (ar[:, None] - ar[None, :] < cfg.swa_window)
    else:
        M = dsa_mask(x, qc, p, cfg, cos, sin)
        if M is not None:
            allowed = M
    s = torch.einsum("qhd,khd->hqk", q, k) * (dn + dr) ** -0.5
    s = s.masked_fill(~allowed[None], float("-inf"))
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)
    gate = torch.sigmoid(x @ p["g"].t())
    return (o * gate[..., None]).reshape(T, H * dv) @ p["o"].t()


def mlp(x, p):
    g, u = (x @ p["gu"].t()).chunk(2, -1)
    return (F.silu(g) * u) @ p["d"].t()


def moe(x, p, cfg):
    sc = torch.sigmoid(x @ p["gate"].t())
    ids = torch.topk(sc + p["bias"], cfg.top_k, -1).indices
    w = sc.gather(1, ids)
    w = w / w.sum(-1, keepdim=True) * cfg.route_scale
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(cfg.top_k):
            wgu, wd = p["experts_dense"][int(ids[t, j])]
            g, u = (x[t] @ wgu.t()).chunk(2, -1)
            out[t] += w[t, j] * ((F.silu(g) * u) @ wd.t())
    return out + mlp(x, p["shared"])


@torch.no_grad()
def forward(W: dict, cfg, ids: torch.Tensor) -> torch.Tensor:
    T = ids.shape[0]
    cos, sin = rope_tab(torch.arange(T), cfg.qk_rope_dim, cfg.rope_theta)
    h = W["embed"][ids].float()
    for l, L in enumerate(W["layers"]):
        h = h + mla(rms(h, L["ln1"], cfg.rms_eps), L["attn"], cfg, l, cos, sin)
        x = rms(h, L["ln2"], cfg.rms_eps)
        h = h + (moe(x, L["moe"], cfg) if cfg.is_moe(l) else mlp(x, L["mlp"]))
    return rms(h, W["norm"], cfg.rms_eps) @ W["lm_head"].t()


@torch.no_grad()
def greedy(W, cfg, prompt: torch.Tensor, n_new: int) -> list:
    ids = prompt.clone()
    out = []
    for _ in range(n_new):
        nxt = int(forward(W, cfg, ids)[-1].argmax())
        out.append(nxt)
        ids = torch.cat([ids, torch.tensor([nxt])])
    return out

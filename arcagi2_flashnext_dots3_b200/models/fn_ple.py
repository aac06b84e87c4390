"""PLE (per-layer n-gram embedding) on the engine path: incremental over per-slot token history and a ring of the
last (ple_conv - 1) * ngram_size normalized gated values per PLE layer.

Same math as the oracle (:func:`.fn_reference.ple`, :func:`.fn_reference.ngram_ids`; the reference's
flashnext/training/student/student_fn.py:380-459): the embedding rows of one step are gathered once and shared by
all PLE layers; each PLE layer runs one fused key|value GEMM and the gate / norm / dilated-conv kernel. GPU:
csrc/k_ple.cu; CPU: torch below.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import native


def _rms1p(x, w, eps, group):
    xf = x.view(*x.shape[:-1], -1, group)
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf.flatten(-2) * (1.0 + w)


def _ids_cpu(ids, slots, n_tok, hist, W, cfg):
    n, hpn, eos = cfg.ngram_size, cfg.heads_per_ngram, cfg.eos_token_id
    mult, offs, sizes = W["ple_mult"].tolist(), W["ple_offs"].tolist(), W["ple_sizes"].tolist()
    nh = (n - 1) * hpn
    rows = torch.empty(len(slots) * n_tok, nh, dtype=torch.int64)
    M64 = (1 << 64) - 1

    def wrap(v):
        v &= M64
        return v - (1 << 64) if v >= (1 << 63) else v
    for b, s in enumerate(slots.tolist()):
        hs = hist[s].tolist()
        since = hs[-1]
        for j in range(n_tok):
            t = int(ids[b * n_tok + j])
            for ng in range(2, n + 1):
                m = wrap(t * mult[0])
                for q in range(1, ng):
                    sq = hs[q - 1] if since >= q else eos
                    m = wrap(m ^ wrap(sq * mult[q]))
                for h in range((ng - 2) * hpn, (ng - 1) * hpn):
                    rows[b * n_tok + j, h] = m % sizes[h] + offs[h]
            hs[1:n - 1] = hs[0:n - 2]
            if n > 1:
                hs[0] = t
            since = 0 if t == eos else since + 1
        hs[-1] = since
        hist[s] = torch.tensor(hs, dtype=torch.int64)
    return rows


def embed_rows(model, ids, slots, positions, n_tok):
    """Scaled embedding rows [T, heads * ple_dim] of this step's tokens (updates the token history)."""
    cfg, W, c = model.cfg, model.W, model.c
    nh = (cfg.ngram_size - 1) * cfg.heads_per_ngram
    T = ids.shape[0]
    if ids.is_cuda:
        rows = torch.empty(T, nh, dtype=torch.int64, device=ids.device)
        native.C().ple_ids(ids.to(torch.int32), slots, n_tok, c.tok_hist, W["ple_mult"], W["ple_offs"],
                           W["ple_sizes"], cfg.heads_per_ngram, cfg.eos_token_id, rows)
        emb = torch.empty(T, nh * cfg.ple_dim, dtype=torch.float16, device=ids.device)
        native.C().ple_gather(W["ple_table"], rows, float(W["ple_scale"]), emb)
        return emb
    rows = _ids_cpu(ids, slots, n_tok, c.tok_hist, W, cfg)
    table = W["ple_table"]
    return (table[rows.clamp_max(table.shape[0] - 1)].float() * W["ple_scale"]).reshape(T, -1)


def apply(model, h, emb, p, ring, slots, positions, n_tok):
    """h += PLE(h, emb) in place for the rows of this step."""
    cfg = model.cfg
    hc, H, d = cfg.hc_count, cfg.hidden_size, cfg.ngram_size
    P = model._mm(emb, p["kv"])                       # [T, hc*H + H] fp32
    if h.is_cuda:
        native.C().ple_mix(h, P, p["nk"], p["nq"], p["nc"], p["conv"], ring, slots, positions, n_tok, hc, d,
                           cfg.rms_eps)
        return
    T = h.shape[0]
    key = _rms1p(P[:, :hc * H], p["nk"], cfg.rms_eps, H).view(T, hc, H)
    val = P[:, hc * H:]
    qn = _rms1p(h, p["nq"], cfg.rms_eps, H).view(T, hc, H)
    gate = (key * qn).sum(-1, keepdim=True) / H ** 0.5
    gate = gate.abs().clamp_min(1e-6).sqrt() * gate.sign()
    gv = (torch.sigmoid(gate) * val[:, None, :]).reshape(T, hc * H)
    gvn = _rms1p(gv, p["nc"], cfg.rms_eps, H)
    kc = p["conv"].shape[1]
    R = ring.shape[1]
    pos = positions.long()
    for t in range(T):
        b, j = divmod(t, n_tok)
        pt = int(pos[b]) + j
        acc = torch.zeros(hc * H)
        for k in range(kc):
            back = (kc - 1 - k) * d
            pp = pt - back
            if pp < 0:
                continue
            x = gvn[t - back] if back <= j else ring[int(slots[b]), pp % R]
            acc += p["conv"][:, k] * x
        h[t] += gv[t] + F.silu(acc)
    for t in range(T):
        b, j = divmod(t, n_tok)
        if n_tok - 1 - j < R:
            ring[int(slots[b]), (int(pos[b]) + j) % R] = gvn[t]

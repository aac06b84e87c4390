"""Engine ops of the Flash-Next-shaped model (decode and prefill), each with a torch implementation.

Every function takes and returns plain tensors. On CUDA tensors it calls the sm_100a kernel of the same name in
the `_C` extension (which must be built: there is no silent eager fallback on a GPU); on CPU tensors it runs the
torch code below, which is also the numerics reference of the kernels' GPU tests.

Shapes: T = tokens in the step, H = hidden, hc = hyper-connection streams, S = cache slots (sequences).
"act" tensors (GEMM inputs) are fp16 on GPU and fp32 on CPU.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import native


def _cuda(t):
    return t.is_cuda


def act_dtype(device) -> torch.dtype:
    return torch.float16 if torch.device(device).type == "cuda" else torch.float32


# --------------------------------------------------------------------------------------------- embedding
def embed_hc(ids: torch.Tensor, table: torch.Tensor, hc: int) -> torch.Tensor:
    """h [T, hc*H] fp32 = embedding row repeated over the hc streams (student_fn.py:646)."""
    if _cuda(ids):
        out = torch.empty(ids.shape[0], hc * table.shape[1], dtype=torch.float32, device=ids.device)
        native.C().embed_hc(ids, table, out, hc)
        return out
    return table[ids.long()].float().repeat(1, hc)


# ------------------------------------------------------------------------------------- hyper-connections
def hc_prenorm(h: torch.Tensor, w: torch.Tensor, hc: int, H: int, eps: float) -> torch.Tensor:
    """Per-stream RMSNorm with (1 + w) weight: hn [T, hc*H] (act dtype)."""
    if _cuda(h):
        out = torch.empty(h.shape, dtype=torch.float16, device=h.device)
        native.C().hc_prenorm(h, w, out, H, eps)
        return out
    xf = h.float().view(h.shape[0], hc, H)
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf.view(h.shape) * (1.0 + w.float())


def hc_act(z: torch.Tensor, rank_pad: int, hc: int, with_inj: bool = True):
    """z [T, rank_pad (+hc)] -> a = silu(z/hc) [T, rank_pad] (act), inj = 2*sigmoid(z_inj/hc) [T, hc] fp32."""
    if _cuda(z):
        a = torch.empty(z.shape[0], rank_pad, dtype=torch.float16, device=z.device)
        inj = torch.empty(z.shape[0], hc if with_inj else 1, dtype=torch.float32, device=z.device)
        native.C().hc_act(z, a, inj, rank_pad, hc, with_inj)
        return a, (inj if with_inj else None)
    a = F.silu(z[:, :rank_pad].float() / hc)
    inj = 2 * torch.sigmoid(z[:, rank_pad: rank_pad + hc].float() / hc) if with_inj else None
    return a, inj


def hc_mix(u: torch.Tensor, hn: torch.Tensor, hc: int, H: int) -> torch.Tensor:
    """x [T, H] (act) = mean over streams of sigmoid(u) * hn."""
    if _cuda(u):
        out = torch.empty(u.shape[0], H, dtype=torch.float16, device=u.device)
        native.C().hc_mix(u, hn, out, hc, H)
        return out
    T = u.shape[0]
    return (torch.sigmoid(u.float()).view(T, hc, H) * hn.float().view(T, hc, H)).mean(1)


def hc_residual(h: torch.Tensor, y: torch.Tensor, inj: torch.Tensor) -> None:
    """h[t, s*H + i] += y[t, i] * inj[t, s] (in place)."""
    if _cuda(h):
        native.C().hc_residual(h, y, inj)
        return
    T, hc = inj.shape
    h.view(T, hc, -1).add_(y.float()[:, None, :] * inj.float()[:, :, None])


# --------------------------------------------------------------------------------------- Gated DeltaNet
GDN_CHUNK = __import__("os").environ.get("FW_GDN_CHUNK", "1") != "0"   # chunked tcgen05 prefill (k_gdn_chunk.cu)
GDN_CHUNK_MIN = 64        # tokens per sequence from which a step runs the chunked form


def gdn_step(proj: torch.Tensor, conv_w: torch.Tensor, conv_state: torch.Tensor, ssm: torch.Tensor,
             A_log: torch.Tensor, dt_bias: torch.Tensor, norm_w: torch.Tensor, slots: torch.Tensor, cfg,
             n_tok: int = 1, n_commit: torch.Tensor = None) -> torch.Tensor:
    """Gated DeltaNet over `n_tok` consecutive tokens of each sequence (rows of proj are grouped per sequence:
    row = seq * n_tok + j). proj [rows, C + nv*dv + 2*nv] fp32 holds [qkv | z | b | a]. Updates conv_state
    [S, C, kc-1] and ssm [S, nv, dk, dv] (fp32 or bf16) of `slots` in place and returns the gated-normed output
    [rows, nv*dv] (act). Math: student_fn.py:251-293 (fla gated delta rule, qk l2norm, scale dk^-0.5).
    ``n_commit`` (int32 [B]): write back only the states after the first n_commit[b] tokens (speculative verify)."""
    if _cuda(proj):
        out = torch.empty(proj.shape[0], cfg.lin_v_heads * cfg.lin_v_dim, dtype=torch.float16, device=proj.device)
        gate = 1 if cfg.gdn_gate == "sigmoid" else 0
        if (GDN_CHUNK and n_commit is None and n_tok >= GDN_CHUNK_MIN and ssm.dtype == torch.bfloat16
                and cfg.lin_k_dim == 128 and cfg.lin_v_dim == 128):
            # prefill: every token's convolution in parallel, then the chunked delta rule on tcgen05
            native.C().gdn_prefill(proj, conv_w, conv_state, ssm, A_log, dt_bias, norm_w, slots, out,
                                   cfg.lin_k_heads, cfg.lin_v_heads, n_tok, cfg.rms_eps, gate,
                                   native.err_word(proj.device), native.DEFAULT_TIMEOUT_NS)
            return out
        native.C().gdn_step(proj, conv_w, conv_state, ssm, A_log, dt_bias, norm_w, slots, out, cfg.lin_k_heads,
                            cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim, n_tok, cfg.rms_eps, gate, n_commit,
                            native.err_word(proj.device), native.DEFAULT_TIMEOUT_NS)
        return out
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    C = 2 * nk * dk + nv * dv
    rows = proj.shape[0]
    B = rows // n_tok
    kc = conv_w.shape[-1]
    out = torch.empty(rows, nv * dv, dtype=torch.float32)
    r = nv // nk
    for b in range(B):
        s = int(slots[b])
        P = proj[b * n_tok:(b + 1) * n_tok].float()
        qkv, z, bb, aa = P.split([C, nv * dv, nv, nv], -1)
        hist = torch.cat([conv_state[s].float(), qkv.t()], 1)              # [C, kc-1+n]
        conv = torch.stack([(hist[:, j:j + kc] * conv_w.view(C, kc)).sum(-1) for j in range(n_tok)], 0)
        m = n_tok if n_commit is None else int(n_commit[b])
        if m > 0:
            conv_state[s] = hist[:, m:m + kc - 1].to(conv_state.dtype)
        x = F.silu(conv)
        q, k, v = x.split([nk * dk, nk * dk, nv * dv], -1)
        q = q.view(n_tok, nk, dk).repeat_interleave(r, 1)
        k = k.view(n_tok, nk, dk).repeat_interleave(r, 1)
        v = v.view(n_tok, nv, dv)
        q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
        k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
        beta = torch.sigmoid(bb)
        g = -A_log.float().exp() * F.softplus(aa + dt_bias.float())
        S = ssm[s].float()
        o = torch.empty(n_tok, nv, dv)
        for j in range(n_tok):
            S = S * g[j].exp()[:, None, None]
            kv = torch.einsum("hkv,hk->hv", S, k[j])
            u = beta[j][:, None] * (v[j] - kv)
            S = S + k[j][:, :, None] * u[:, None, :]
            o[j] = torch.einsum("hkv,hk->hv", S, q[j])
            if j + 1 == m:
                ssm[s] = S.to(ssm.dtype)
        o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * norm_w.float()
        zz = z.view(n_tok, nv, dv)
        o = o * (torch.sigmoid(zz) if cfg.gdn_gate == "sigmoid" else F.silu(zz))
        out[b * n_tok:(b + 1) * n_tok] = o.reshape(n_tok, -1)
    return out


# --------------------------------------------------------------------------------------------- attention
def rope_tables(max_pos: int, rd: int, theta: float, device) -> torch.Tensor:
    """cos/sin table [max_pos, rd] each, stacked -> [2, max_pos, rd] fp32 (computed in fp64)."""
    inv = 1.0 / theta ** (torch.arange(0, rd, 2, dtype=torch.float64) / rd)
    f = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    e = torch.cat([f, f], -1)
    return torch.stack([e.cos(), e.sin()]).float().to(device)


def _rope(x, cs):
    """x [..., d] rotated on its first rd dims with cs = (cos [rd], sin [rd]) broadcastable."""
    c, s = cs
    rd = c.shape[-1]
    xr, xp = x[..., :rd], x[..., rd:]
    x1, x2 = xr[..., : rd // 2], xr[..., rd // 2:]
    return torch.cat([xr * c + torch.cat([-x2, x1], -1) * s, xp], -1)


def _rms1p(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def qsa_prep(proj, qn, kn, iqn, ikn, rope, k_cache, v_cache, block_table, slots, positions, kr_ring, comp_cache,
             cfg, n_tok: int = 1):
    """Split the fused projection, normalize + rotate q/k, append k/v (and the indexer key) to the caches.

    proj rows = seq * n_tok + j (token j of sequence seq at position positions[seq] + j). Returns (q [rows, Hq, D]
    fp32, gate [rows, Hq*D] fp32, iq [rows, iH, iD] fp32). Complete indexer blocks (every `ratio` tokens) are
    compressed into comp_cache [S, max_blocks, iD] (mean of the block's keys, RMSNorm, RoPE at the block start;
    student_fn.py:313-322)."""
    if _cuda(proj):
        rows = proj.shape[0]
        q = torch.empty(rows, cfg.n_heads, cfg.head_dim, dtype=torch.float32, device=proj.device)
        gate = torch.empty(rows, cfg.n_heads * cfg.head_dim, dtype=torch.float32, device=proj.device)
        iq = torch.empty(rows, cfg.indexer_heads, cfg.indexer_dim, dtype=torch.float32, device=proj.device)
        native.C().qsa_prep(proj, qn, kn, iqn, ikn, rope, k_cache, v_cache, block_table, slots, positions,
                            kr_ring, comp_cache, q, gate, iq, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                            cfg.indexer_heads, cfg.indexer_dim, cfg.indexer_ratio, n_tok, cfg.rms_eps)
        return q, gate, iq
    Hq, KV, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    iH, iD, r = cfg.indexer_heads, cfg.indexer_dim, cfg.indexer_ratio
    rows = proj.shape[0]
    P = proj.float()
    qg, k, v, iqk = P.split([Hq * 2 * D, KV * D, KV * D, iH * iD + iD], -1)
    qg = qg.view(rows, Hq, 2 * D)
    q, gate = qg[..., :D], qg[..., D:].reshape(rows, Hq * D)
    bs = k_cache.shape[1]
    pos = (positions.long()[:, None] + torch.arange(n_tok)[None]).reshape(-1)
    cs = (rope[0][pos][:, None, :], rope[1][pos][:, None, :])
    q = _rope(_rms1p(q, qn, cfg.rms_eps), cs)
    k = _rope(_rms1p(k.view(rows, KV, D), kn, cfg.rms_eps), cs)
    v = v.view(rows, KV, D)
    iq_, kr = iqk.split([iH * iD, iD], -1)
    iq = _rope(_rms1p(iq_.view(rows, iH, iD), iqn, cfg.rms_eps), (rope[0][pos][:, None, :], rope[1][pos][:, None, :]))
    for row in range(rows):
        b, p = row // n_tok, int(pos[row])
        s = int(slots[b])
        blk = int(block_table[s, p // bs])
        k_cache[blk, p % bs] = k[row].to(k_cache.dtype)
        v_cache[blk, p % bs] = v[row].to(v_cache.dtype)
        RL = kr_ring.shape[1]
        kr_ring[s, p % RL] = kr[row].to(kr_ring.dtype)
        if (p + 1) % r == 0:
            cb = (p + 1) // r - 1
            st = cb * r
            kb = _rms1p(kr_ring[s, [q % RL for q in range(st, p + 1)]].float().mean(0), ikn, cfg.rms_eps)
            comp_cache[s, cb] = _rope(kb, (rope[0][st], rope[1][st])).to(comp_cache.dtype)
    return q, gate, iq


def qsa_select(iq, comp_cache, slots, positions, cfg, n_tok: int = 1):
    """Indexer top-k over complete compressed blocks. Returns sel [rows, nblk] int32 block ids (-1 padded) and
    a flag per row (1 = sparse, 0 = all blocks allowed because ncomp <= nblk)."""
    nblk, r = min(cfg.indexer_blocks, comp_cache.shape[1]), cfg.indexer_ratio
    rows = iq.shape[0]
    if _cuda(iq):
        sel = torch.empty(rows, nblk, dtype=torch.int32, device=iq.device)
        sparse = torch.empty(rows, dtype=torch.int32, device=iq.device)
        native.C().qsa_select(iq, comp_cache, slots, positions, sel, sparse, nblk, r, n_tok)
        return sel, sparse
    sel = torch.full((rows, nblk), -1, dtype=torch.int32)
    sparse = torch.zeros(rows, dtype=torch.int32)
    for row in range(rows):
        b = row // n_tok
        p = int(positions[b]) + row % n_tok
        nc = (p + 1) // r
        if nc <= nblk:
            continue
        kb = comp_cache[int(slots[b]), :nc].float()
        sc = torch.relu(iq[row].float() @ kb.t()).sum(0) / math.sqrt(cfg.indexer_dim)
        sel[row] = sc.topk(nblk).indices.to(torch.int32)
        sparse[row] = 1
    return sel, sparse


def attn_decode(q, gate, k_cache, v_cache, block_table, slots, positions, sel, sparse, cfg, n_tok: int = 1):
    """Sparse (or full causal) GQA attention of each row's query over its sequence's cached keys, times the
    sigmoid output gate: out [rows, Hq*D] (act). Allowed keys of a query at position p: k <= p and (k's indexer
    block is selected, or k >= ((p+1)//r)*r); all k <= p when the row is not sparse."""
    if _cuda(q):
        out = torch.empty(q.shape[0], q.shape[1] * q.shape[2], dtype=torch.float16, device=q.device)
        native.C().attn_decode(q, gate, k_cache, v_cache, block_table, slots, positions, sel, sparse, out,
                               cfg.n_kv_heads, cfg.indexer_ratio, n_tok)
        return out
    Hq, KV, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    r = cfg.indexer_ratio
    bs = k_cache.shape[1]
    rows = q.shape[0]
    out = torch.empty(rows, Hq * D)
    for row in range(rows):
        b = row // n_tok
        p = int(positions[b]) + row % n_tok
        s = int(slots[b])
        L = p + 1
        nb = (L + bs - 1) // bs
        blks = block_table[s, :nb].long()
        K = k_cache[blks].float().reshape(nb * bs, KV, D)[:L]
        V = v_cache[blks].float().reshape(nb * bs, KV, D)[:L]
        keep = torch.ones(L, dtype=torch.bool)
        if int(sparse[row]):
            blk_ok = torch.zeros((L + r - 1) // r + 1, dtype=torch.bool)
            ids = sel[row][sel[row] >= 0].long()
            blk_ok[ids] = True
            kk = torch.arange(L)
            keep = blk_ok[kk // r] | (kk >= ((p + 1) // r) * r)
        Kr = K[keep].repeat_interleave(Hq // KV, 1)
        Vr = V[keep].repeat_interleave(Hq // KV, 1)
        s_ = torch.einsum("hd,khd->hk", q[row].float(), Kr) * D ** -0.5
        o = torch.einsum("hk,khd->hd", torch.softmax(s_, -1), Vr)
        out[row] = o.reshape(-1) * torch.sigmoid(gate[row].float())
    return out


# ------------------------------------------------------------------------------------------------- MoE
def moe_route(logits: torch.Tensor, E: int, top_k: int):
    """Softmax over the first E logits, top-k, renormalize (student_fn.py:516-519). ids [T, k] int32,
    w [T, k] fp32. Ties resolve to the lower expert id."""
    if _cuda(logits):
        T = logits.shape[0]
        ids = torch.empty(T, top_k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, top_k, dtype=torch.float32, device=logits.device)
        native.C().moe_route(logits, ids, w, E, top_k)
        return ids, w
    pr = torch.softmax(logits[:, :E].float(), -1)
    w, ids = torch.topk(pr, top_k, -1)
    return ids.to(torch.int32), w / w.sum(-1, keepdim=True)


def moe_plan(ids: torch.Tensor, E: int, n_tile: int, max_items: int):
    """Sort the T*k (token, expert) pairs by expert. Returns pair_pos [T, k] int32 (row of each pair in the
    expert-sorted order), items [max_items, 4] int32 ({expert, first row, count, 0}, one per n_tile chunk) and
    n_items [1] int32."""
    T, k = ids.shape
    if _cuda(ids):
        pair_pos = torch.empty(T, k, dtype=torch.int32, device=ids.device)
        items = torch.empty(max_items, 4, dtype=torch.int32, device=ids.device)
        n_items = torch.empty(1, dtype=torch.int32, device=ids.device)
        native.C().moe_plan(ids, pair_pos, items, n_items, E, n_tile)
        return pair_pos, items, n_items
    flat = ids.reshape(-1).long()
    order = torch.argsort(flat, stable=True)
    pos = torch.empty_like(order)
    pos[order] = torch.arange(flat.numel())
    counts = torch.bincount(flat, minlength=E)
    items, start = [], 0
    for e in range(E):
        c = int(counts[e])
        for s0 in range(0, c, n_tile):
            items.append([e, start + s0, min(n_tile, c - s0), 0])
        start += c
    it = torch.zeros(max(max_items, 1), 4, dtype=torch.int32)
    if items:
        it[: len(items)] = torch.tensor(items, dtype=torch.int32)
    return pos.view(T, k).to(torch.int32), it, torch.tensor([len(items)], dtype=torch.int32)


def moe_scatter(x: torch.Tensor, pair_pos: torch.Tensor) -> torch.Tensor:
    """xs [T*k, H] with xs[pair_pos[t, j]] = x[t]."""
    T, k = pair_pos.shape
    if _cuda(x):
        xs = torch.empty(T * k, x.shape[1], dtype=x.dtype, device=x.device)
        native.C().moe_scatter(x, pair_pos, xs)
        return xs
    xs = torch.empty(T * k, x.shape[1], dtype=x.dtype)
    xs[pair_pos.reshape(-1).long()] = x.repeat_interleave(k, 0)
    return xs


def moe_combine(h, ypair, pair_pos, w, ysh, sg_logit, inj) -> None:
    """h += (sum_j w[t, j] * ypair[pair_pos[t, j]] + sigmoid(sg_logit[t]) * ysh[t]) (x) inj[t] (in place)."""
    if _cuda(h):
        native.C().moe_combine(h, ypair, pair_pos, w, ysh, sg_logit, inj)
        return
    T, k = pair_pos.shape
    y = (ypair[pair_pos.long()].float() * w[..., None].float()).sum(1)
    y = y + torch.sigmoid(sg_logit.float().reshape(T, 1)) * ysh.float()
    hc_residual(h, y, inj)


# ---------------------------------------------------------------------------------------------- sampling
def argmax(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token per row (int32); ties resolve to the lowest id like torch.argmax."""
    if _cuda(logits):
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
        native.C().argmax_rows(logits, out)
        return out
    return logits.float().argmax(-1).to(torch.int32)

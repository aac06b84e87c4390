"""Dots3-shaped model ops: CUDA tensors go to the `_C` kernels (csrc/k_d3.cu), CPU tensors to torch code with
the same math and the same selection rules (the CPU path is the engine-level oracle in tests).

Latent cache: [n_blocks, block_size, kv_lora_rank + rope_dim] FP8 e4m3 on GPU (the reference's 576/1088-byte
rows); on CPU fp32 rows holding the FP8-rounded values. Index-key cache: [slots, max_len, index_dim].
DSA selection: all keys above the k-th largest score plus the lowest-index keys among those equal to it (a
stable descending sort), full causal attention while a query has at most `index_topk` predecessors.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from . import native


def _cuda(t):
    return t.is_cuda


def rope_table(max_pos: int, dr: int, theta: float, device) -> torch.Tensor:
    """[max_pos, dr/2, 2] (cos, sin) for interleaved RoPE."""
    inv = 1.0 / theta ** (torch.arange(0, dr, 2, dtype=torch.float64) / dr)
    f = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    return torch.stack([f.cos(), f.sin()], -1).float().to(device)


def _rope_inter(x, cs):
    """x [..., T, h, d] rotated with cs [T, d/2, 2]."""
    c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x1 * c - x2 * s, x2 * c + x1 * s], -1).flatten(-2)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _pos(positions, n_tok):
    return (positions.long()[:, None] + torch.arange(n_tok, device=positions.device)[None]).reshape(-1)


def add_rms(h, y, w, eps, out_dtype=torch.float16):
    """h += y (if given, in place); returns rms(h) * w in out_dtype."""
    out = torch.empty(h.shape, dtype=out_dtype if h.is_cuda else torch.float32, device=h.device)
    if _cuda(h):
        native.C().d3_add_rms(h, y, w, eps, out)
        return out
    if y is not None:
        h += y
    out.copy_(_rms(h, w, eps))
    return out


def mla_prep(P, cfg, l, p, rope, cache, block_table, idx_cache, slots, positions, n_tok, index: bool = True,
             index_shard=(1, 0)):
    """Returns (qc [T, qr] act, gate logits [T, H], index weights [T, iH] or None); writes the cache rows.
    ``index=False`` (a DSA layer that shares another layer's top-k) skips the index key and weights.
    ``index_shard=(W, r)``: the index cache holds only positions p = r (mod W), position p at row (p - r) / W."""
    T = P.shape[0]
    qr, kvr, dr, H = cfg.q_lora_rank, cfg.latent_of(l), cfg.qk_rope_dim, cfg.heads_of(l)
    dsa = cfg.layer_kind(l) == "dsa" and index
    iD, iH = (cfg.index_dim, cfg.index_heads) if dsa else (0, 0)
    off_g = qr + kvr + dr
    off_ik, off_iw = off_g + H, off_g + H + iD
    qs = (cfg.hidden_size / qr) ** 0.5 if cfg.kv_rescale else 1.0
    kvs = (cfg.hidden_size / kvr) ** 0.5 if cfg.kv_rescale else 1.0
    dev = P.device
    if _cuda(P):
        qc = torch.empty(T, qr, dtype=torch.float16, device=dev)
        gate = torch.empty(T, H, dtype=torch.float32, device=dev)
        iw = torch.empty(T, iH, dtype=torch.float32, device=dev) if dsa else None
        offs = [off_g, off_ik, off_iw] + ([index_shard[0], index_shard[1]] if index_shard[0] > 1 else [])
        native.C().d3_mla_prep(P, [qr, kvr, dr, H, iD, iH], offs, p["q_ln"], p["kv_ln"], p["kr_ln"],
                               p.get("ik_w"), p.get("ik_b"), [qs, kvs, cfg.rms_eps], rope, cache, block_table,
                               idx_cache, slots, positions, n_tok, qc, gate, iw)
        return qc, gate, iw
    pos = _pos(positions, n_tok)
    sl = slots.long().repeat_interleave(n_tok)
    cs = rope[pos]
    qc = _rms(P[:, :qr], p["q_ln"], cfg.rms_eps) * qs
    kvc = (_rms(P[:, qr:qr + kvr], p["kv_ln"], cfg.rms_eps) * kvs).to(torch.float8_e4m3fn).float()
    kpe = _rope_inter(_rms(P[:, qr + kvr:off_g], p["kr_ln"], cfg.rms_eps)[:, None, :], cs)[:, 0]
    kpe = kpe.to(torch.float8_e4m3fn).float()
    bs = cache.shape[1]
    blk = block_table[sl, pos // bs].long()
    cache[blk, pos % bs] = torch.cat([kvc, kpe], -1)
    gate = P[:, off_g:off_g + H].clone()
    iw = None
    if dsa:
        ik = F.layer_norm(P[:, off_ik:off_ik + iD], (iD,), p["ik_w"], p["ik_b"], 1e-6)
        ik = torch.cat([_rope_inter(ik[:, None, :dr], cs)[:, 0], ik[:, dr:]], -1)
        Wsh, r = index_shard
        keep = ((pos - r) % Wsh == 0) & (pos >= r)
        idx_cache[sl[keep], (pos[keep] - r) // Wsh] = ik[keep].to(idx_cache.dtype)
        iw = P[:, off_iw:off_iw + iH] * iD ** -0.5 * iH ** -0.5
    return qc, gate, iw


def mla_qsplit(Q, cfg, l, rope, positions, n_tok):
    """Returns (q_nope [H, T, dn], q_pe [T, H, dr] fp32, iq [T, iH, iD] fp32 or None)."""
    T = Q.shape[0]
    H, dn, dr = cfg.heads_of(l), cfg.qk_nope_dim, cfg.qk_rope_dim
    dsa = cfg.layer_kind(l) == "dsa"
    iH, iD = (cfg.index_heads, cfg.index_dim) if dsa else (0, 0)
    if _cuda(Q):
        q_nope = torch.empty(H, T, dn, dtype=torch.bfloat16, device=Q.device)
        q_pe = torch.empty(T, H, dr, dtype=torch.float32, device=Q.device)
        iq = torch.empty(T, iH, iD, dtype=torch.float32, device=Q.device) if dsa else None
        native.C().d3_mla_qsplit(Q, H, dn, dr, iH, iD, rope, positions, n_tok, q_nope, q_pe, iq)
        return q_nope, q_pe, iq
    cs = rope[_pos(positions, n_tok)]
    q = Q[:, :H * (dn + dr)].view(T, H, dn + dr)
    q_nope = q[..., :dn].transpose(0, 1).contiguous()
    q_pe = _rope_inter(q[..., dn:], cs)
    iq = None
    if dsa:
        iq = Q[:, H * (dn + dr):H * (dn + dr) + iH * iD].view(T, iH, iD)
        iq = torch.cat([_rope_inter(iq[..., :dr], cs), iq[..., dr:]], -1)
    return q_nope, q_pe, iq


_DSA_CUDA_CORE = os.environ.get("FW_DSA_CUDA_CORE", "0") == "1"   # force the CUDA-core indexer logits


def dsa_select(iq, iw, idx_cache, slots, positions, n_tok, topk: int, max_len: int):
    """[T, topk] int32 selected key positions; a row whose first entry is -1 attends to all causal keys."""
    T = iq.shape[0]
    ld = (max_len + 255) // 256 * 256
    if _cuda(iq):
        scores = torch.empty(T, ld, dtype=torch.float32, device=iq.device)
        C = native.C()
        if (not _DSA_CUDA_CORE and idx_cache.dtype == torch.bfloat16
                and C.d3_dsa_tc_supported(iq.shape[1], iq.shape[2])):
            # tcgen05 path (csrc/k_dsa.cu): keys as the MMA's M, one key per epilogue thread
            C.d3_dsa_scores_tc(iq, iw, idx_cache, slots, positions, n_tok, scores, native.err_word(iq.device),
                               native.DEFAULT_TIMEOUT_NS)
        else:
            C.d3_dsa_scores(iq, iw, idx_cache, slots, positions, n_tok, scores)
        sel = torch.empty(T, topk, dtype=torch.int32, device=iq.device)
        n_valid = (_pos(positions, n_tok) + 1).to(torch.int32)
        native.C().topk_rows(scores, n_valid, topk, sel)
        return sel
    pos = _pos(positions, n_tok)
    sl = slots.long().repeat_interleave(n_tok)
    sel = torch.full((T, topk), -1, dtype=torch.int32)
    for t in range(T):
        p = int(pos[t])
        if p + 1 <= topk:
            continue
        k = idx_cache[sl[t], : p + 1].float()
        s = (torch.relu(torch.einsum("hd,kd->hk", iq[t], k)) * iw[t][:, None]).sum(0)
        sel[t] = torch.sort(s, descending=True, stable=True).indices[:topk].to(torch.int32)
    return sel


def dsa_select_sharded(iq, iw, idx_cache, slots, positions, n_tok, topk: int, rank: int, world: int, group=None):
    """:func:`dsa_select` with the index keys sharded over a TP group by position mod world (the reference's
    shard_indexer.py:1-15, 42-145 with the local select / all-gather / merge of topk_select.cu:77, 204): this rank
    scores only its own keys (position p = rank + world * i at row i), takes its local top-k (lowest position
    first among equal scores), all-gathers (score, position) candidates and merges them into the global top-k by
    (score descending, position ascending). Each rank's share of the global top-k is inside its local top-k, so
    the merge selects the same key set as the unsharded indexer."""
    import torch.distributed as dist
    T = iq.shape[0]
    dev = iq.device
    pos = _pos(positions, n_tok).long()
    n_loc = torch.where(pos >= rank, (pos - rank) // world + 1, torch.zeros_like(pos))
    if _cuda(iq):
        L = idx_cache.shape[1]
        ld = (L + 255) // 256 * 256
        scores = torch.full((T, ld), float("-inf"), dtype=torch.float32, device=dev)
        # every row of a sequence scores up to the sequence's last local key plus its row offset (masked below);
        # the local cache keeps n_tok rows of slack past max_len / world for these reads
        last = n_loc.view(-1, n_tok)[:, -1] - 1                 # last local key of each sequence
        p_kern = last.clamp_min(0).to(torch.int32)              # row j scores local keys <= last + j
        C = native.C()
        if (not _DSA_CUDA_CORE and idx_cache.dtype == torch.bfloat16
                and C.d3_dsa_tc_supported(iq.shape[1], iq.shape[2])):
            C.d3_dsa_scores_tc(iq, iw, idx_cache, slots, p_kern, n_tok, scores, native.err_word(dev),
                               native.DEFAULT_TIMEOUT_NS)
        else:
            C.d3_dsa_scores(iq, iw, idx_cache, slots, p_kern, n_tok, scores)
        loc = torch.empty(T, topk, dtype=torch.int32, device=dev)
        C.topk_rows(scores, n_loc.to(torch.int32), topk, loc)
    else:
        sl = slots.long().repeat_interleave(n_tok)
        scores = torch.full((T, max(1, int(n_loc.max()))), float("-inf"))
        for t in range(T):
            n = int(n_loc[t])
            if n:
                k = idx_cache[sl[t], :n].float()
                scores[t, :n] = (torch.relu(torch.einsum("hd,kd->hk", iq[t], k)) * iw[t][:, None]).sum(0)
        loc = torch.full((T, topk), -1, dtype=torch.int32)
        for t in range(T):
            n = int(n_loc[t])
            if n > topk:
                loc[t] = torch.sort(scores[t, :n], descending=True, stable=True).indices[:topk].to(torch.int32)
    # rows with at most topk local keys: every local key is a candidate
    ar = torch.arange(topk, device=dev)[None, :]
    all_local = (loc[:, :1] < 0)
    loc = torch.where(all_local, torch.where(ar < n_loc[:, None], ar, -1).to(torch.int32), loc)
    valid = loc >= 0
    cand_s = torch.where(valid, scores.gather(1, loc.clamp_min(0).long()), torch.full_like(loc, float("-inf"),
                                                                                          dtype=torch.float32))
    cand_p = torch.where(valid, rank + world * loc.long(), torch.full_like(loc, -1, dtype=torch.long))
    pack = torch.stack([cand_s, cand_p.float()], -1).contiguous()            # positions < 2^24: exact in fp32
    parts = [torch.empty_like(pack) for _ in range(world)]
    dist.all_gather(parts, pack, group=group)
    allc = torch.cat(parts, 1)                                               # [T, world * topk, 2]
    s_all, p_all = allc[..., 0], allc[..., 1]
    p_key = torch.where(p_all < 0, torch.full_like(p_all, float(1 << 30)), p_all)
    o1 = torch.sort(p_key, dim=1, stable=True).indices                       # position ascending
    s1 = s_all.gather(1, o1)
    o2 = torch.sort(s1, dim=1, descending=True, stable=True).indices         # then score descending
    order = o1.gather(1, o2)
    sel = p_all.gather(1, order[:, :topk]).to(torch.int32)
    dense = (pos + 1 <= topk)[:, None]                                       # short rows attend to every key
    return torch.where(dense, torch.full_like(sel, -1), sel)


_MLA_CUDA_CORE = os.environ.get("FW_MLA_CUDA_CORE", "0") == "1"   # force the CUDA-core latent attention
_MLA_SPLITS = int(os.environ.get("FW_MLA_SPLITS", "0"))              # > 0: fixed key-split count (tests)
_MLA_TRACE = None   # int64 [64 * 8] device tensor: per-chunk phase timestamps of the first CTA (profiling)


def mla_attn(q_lat, q_pe, cache, block_table, slots, positions, n_tok, sel, window: int, scale: float):
    """o_lat [H, T, kvr]: softmax over rows of (q_lat . c + q_pe . r) * scale, times the latent c."""
    H, T, kvr = q_lat.shape
    if _cuda(q_lat):
        o = torch.empty_like(q_lat)
        C = native.C()
        if not _MLA_CUDA_CORE and C.d3_mla_tc_supported(kvr, q_pe.shape[2]):
            # tcgen05 path (csrc/k_mla.cu); the CUDA-core kernel stays for shapes it does not cover
            C.d3_mla_attn_tc(q_lat, q_pe, cache, block_table, slots, positions, n_tok, sel, window, scale, o,
                             native.err_word(q_lat.device), native.DEFAULT_TIMEOUT_NS, _MLA_SPLITS, _MLA_TRACE)
        else:
            C.d3_mla_attn(q_lat, q_pe, cache, block_table, slots, positions, n_tok, sel, window, scale, o)
        return o
    pos = _pos(positions, n_tok)
    sl = slots.long().repeat_interleave(n_tok)
    bs = cache.shape[1]
    o = torch.zeros(H, T, kvr)
    for t in range(T):
        p = int(pos[t])
        if sel is not None and int(sel[t, 0]) >= 0:
            rows = sel[t].long()
        else:
            lo = max(0, p - window + 1) if window > 0 else 0
            rows = torch.arange(lo, p + 1)
        c = cache[block_table[sl[t], rows // bs].long(), rows % bs]
        s = (q_lat[:, t] @ c[:, :kvr].t() + q_pe[t] @ c[:, kvr:].t()) * scale
        o[:, t] = torch.softmax(s, -1) @ c[:, :kvr]
    return o


def mla_out(o, gate):
    """o [H, T, dv] * sigmoid(gate [T, H]) -> [T, H * dv] (fp16 on GPU)."""
    H, T, dv = o.shape
    if _cuda(o):
        out = torch.empty(T, H * dv, dtype=torch.float16, device=o.device)
        native.C().d3_mla_out(o, gate, out)
        return out
    return (o.transpose(0, 1) * torch.sigmoid(gate)[..., None]).reshape(T, H * dv)


def route(logits, E: int, bias, k: int, scale: float):
    """Sigmoid scores, top-k by score + bias (ties: lower id), weights renormalized * scale."""
    T = logits.shape[0]
    if _cuda(logits):
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        native.C().d3_route(logits, E, bias, k, scale, ids, w)
        return ids, w
    sc = torch.sigmoid(torch.nan_to_num(logits[:, :E].float()))
    ids = torch.sort(sc + bias, dim=-1, descending=True, stable=True).indices[:, :k]
    w = sc.gather(1, ids)
    return ids.to(torch.int32), w / w.sum(-1, keepdim=True) * scale

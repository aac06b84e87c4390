"""Random-init weights of the Flash-Next-shaped model, in reference (dense) form and engine (runtime) form.

``random_dense(cfg, seed)`` returns the dict consumed by :mod:`.fn_reference`: every dense tensor is already
rounded to its storage format (fp16, or FP8 128x128 block-scaled when ``cfg.dense_fp8``) so the oracle and the
engine see bit-identical weights; experts are N(0, std) weights quantized per expert to ``cfg.bits_of(e)`` bits
(symmetric or asymmetric RTN, group 128) and kept both as planar checkpoint blobs and dequantized copies.

``to_engine(W, cfg, device)`` converts that dict to the engine form (WeightSets in the tile-block layout,
fused projection matrices, padded hyper-connection ranks). ``random_engine(cfg, device, seed)`` builds engine
weights directly on the device without dense copies (used for the full-size model: 320 experts x 48 layers).
"""
from __future__ import annotations

import torch

from ..formats import lowbit_file, planar
from ..formats import runtime as rt
from ..ops import wgemm

STD = 0.02


def _round_dense(w: torch.Tensor, cfg) -> torch.Tensor:
    if getattr(cfg, "dense_fp8", False) and w.shape[1] % 128 == 0:
        w8, sc = rt.quantize_fp8_blocks(w)
        return rt.dequant_fp8_blocks(w8, sc)
    return w.half().float()


def _round_permuted(w_gu: torch.Tensor, cfg) -> torch.Tensor:
    """Round a [gate; up] weight in the silu-epilogue row order (where its FP8 blocks live), return it unpermuted."""
    perm = rt.gate_up_perm(w_gu.shape[0] // 2)
    out = torch.empty_like(w_gu)
    out[perm] = _round_dense(w_gu[perm], cfg)
    return out


def rank_pad(cfg) -> int:
    return (cfg.hc_rank + 127) // 128 * 128


def _hc_params(cfg, g, combine=True):
    hc, H, R = cfg.hc_count, cfg.hidden_size, cfg.hc_rank
    up = torch.randn(hc * H, R, generator=g) * (1.0 / R ** 0.5)
    p = {"norm": torch.randn(hc * H, generator=g) * 0.1,
         "down": _round_dense(torch.randn(R, hc * H, generator=g) * STD, cfg),
         "up": _round_dense(_pad_cols(up, rank_pad(cfg)), cfg)[:, :R]}
    if combine:
        p["inj"] = _round_dense(torch.randn(hc, hc * H, generator=g) * STD, cfg)
    return p


def random_dense(cfg, seed: int = 0, symmetric: bool = True) -> dict:
    g = torch.Generator().manual_seed(seed)
    H, hc = cfg.hidden_size, cfg.hc_count
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    Hq, KV, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    iH, iD = cfg.indexer_heads, cfg.indexer_dim
    rd = lambda *s, std=STD: torch.randn(*s, generator=g) * std  # noqa: E731
    W = {"embed": rd(cfg.vocab_size, H, std=1.0).bfloat16().float(),
         "lm_head": _round_dense(rd(cfg.vocab_size, H), cfg),
         "mixer": _hc_params(cfg, g, combine=False), "layers": []}
    if cfg.ple_layers:
        nh = (cfg.ngram_size - 1) * cfg.heads_per_ngram
        W["ple_table"] = (torch.randn(cfg.ple_rows, cfg.ple_dim, generator=g)).to(torch.float8_e4m3fn)
        W["ple_scale"] = 0.05
        W["ple_mult"] = torch.randint(1, 1 << 20, (cfg.ngram_size,), generator=g).long() * 2 + 1
        sizes = torch.randint(cfg.ple_rows // (2 * nh), cfg.ple_rows // nh, (nh,), generator=g).long()
        W["ple_sizes"] = sizes
        W["ple_offs"] = torch.cumsum(torch.cat([torch.zeros(1, dtype=torch.long), sizes[:-1]]), 0)
    for l in range(cfg.num_layers):
        L = {"ahc": _hc_params(cfg, g), "mhc": _hc_params(cfg, g)}
        if l in cfg.ple_layers:
            nh = (cfg.ngram_size - 1) * cfg.heads_per_ngram
            L["ple"] = {"kp": _round_dense(rd(hc * H, nh * cfg.ple_dim), cfg),
                        "vp": _round_dense(rd(H, nh * cfg.ple_dim), cfg),
                        "nk": rd(hc * H, std=0.1), "nq": rd(hc * H, std=0.1), "nc": rd(hc * H, std=0.1),
                        "conv": rd(hc * H, 1, cfg.ple_conv, std=0.3)}
        if cfg.layer_kind(l) == "linear":
            C = 2 * nk * dk + nv * dv
            ba = _round_dense(rd(2 * nv, H), cfg)
            L["mix"] = {"qkv": _round_dense(rd(C, H), cfg), "z": _round_dense(rd(nv * dv, H), cfg),
                        "b": ba[:nv], "a": ba[nv:],
                        "conv": rd(C, 1, cfg.conv_kernel, std=0.3),
                        "A_log": torch.log(torch.rand(nv, generator=g) * 15 + 1),
                        "dt_bias": rd(nv, std=0.5), "norm": 1.0 + rd(dv, std=0.1),
                        "out": _round_dense(rd(H, nv * dv), cfg)}
        else:
            L["mix"] = {"q": _round_dense(rd(Hq * 2 * D, H), cfg), "k": _round_dense(rd(KV * D, H), cfg),
                        "v": _round_dense(rd(KV * D, H), cfg), "o": _round_dense(rd(H, Hq * D), cfg),
                        "qn": rd(D, std=0.1), "kn": rd(D, std=0.1),
                        "iqk": _round_dense(rd(iH * iD + iD, H), cfg), "iqn": rd(iD, std=0.1),
                        "ikn": rd(iD, std=0.1)}
        lay = lowbit_file.random_layer(cfg.n_experts, H, cfg.moe_inter, [cfg.bits_of(e) for e in range(cfg.n_experts)],
                                       g, std=STD, symmetric=symmetric, n_orig=cfg.n_experts_orig)
        L["moe"] = {"gate": lay.router.float().half().float(), "lowbit": lay,
                    "experts_dense": [b.dense() for b in lay.blobs],
                    "sgu": _round_permuted(rd(2 * cfg.shared_inter, H), cfg),
                    "sd": _round_dense(rd(H, cfg.shared_inter), cfg),
                    "sgate": rd(1, H).half().float()}
        W["layers"].append(L)
    return W


# ----------------------------------------------------------------------------------------- engine form
def _ws(w: torch.Tensor, cfg, device, silu_pairs=False):
    """Dense weight -> WeightSet (fp16 format, or FP8 when the config stores dense weights in FP8)."""
    if getattr(cfg, "dense_fp8", False) and w.shape[1] % 128 == 0 and not silu_pairs:
        w8, sc = rt.quantize_fp8_blocks(w)
        return wgemm.build_weight_set([rt.pack_fp8(w8, sc)], [8], w.shape[0], w.shape[1], device=device)
    if getattr(cfg, "dense_fp8", False) and silu_pairs:
        w8, sc = rt.quantize_fp8_blocks(w)
        return wgemm.build_weight_set([rt.pack_fp8(w8, sc)], [8], w.shape[0], w.shape[1], silu_pairs=True,
                                      device=device)
    return wgemm.build_weight_set([rt.pack_f16(w)], [16], w.shape[0], w.shape[1], silu_pairs=silu_pairs,
                                  device=device)


def _pad_cols(w, n):
    if w.shape[1] == n:
        return w
    return torch.cat([w, torch.zeros(w.shape[0], n - w.shape[1])], 1)


def _pad_rows(w, n):
    if w.shape[0] == n:
        return w
    return torch.cat([w, torch.zeros(n - w.shape[0], w.shape[1])], 0)


def _hc_engine(p, cfg, device):
    R = rank_pad(cfg)
    down = _pad_rows(p["down"], R)
    w1 = torch.cat([down, p["inj"]], 0) if "inj" in p else down
    return {"norm": p["norm"].float().to(device), "w1": _ws(w1, cfg, device),
            "w2": _ws(_pad_cols(p["up"], R), cfg, device)}


def _silu_perm_rows(w_gu, inter):
    """[gate I; up I] rows -> the silu-epilogue tile order."""
    return w_gu[rt.gate_up_perm(inter)]


def to_engine(W: dict, cfg, device) -> dict:
    """Engine weights from the dense dict (small models; the full-size model uses random_engine)."""
    H = cfg.hidden_size
    E = {"embed": W["embed"].to(device, torch.float32 if torch.device(device).type == "cpu" else torch.bfloat16),
         "lm_head": _ws(W["lm_head"], cfg, device), "mixer": _hc_engine(W["mixer"], cfg, device), "layers": []}
    for k in ("ple_table", "ple_mult", "ple_offs", "ple_sizes"):
        if k in W:
            E[k] = W[k].to(device)
    if "ple_scale" in W:
        E["ple_scale"] = W["ple_scale"]
    for l, L in enumerate(W["layers"]):
        M = {"ahc": _hc_engine(L["ahc"], cfg, device), "mhc": _hc_engine(L["mhc"], cfg, device)}
        m = L["mix"]
        if cfg.layer_kind(l) == "linear":
            proj = torch.cat([m["qkv"], m["z"], m["b"], m["a"]], 0)
            M["mix"] = {"proj": _ws(proj, cfg, device), "out": _ws(m["out"], cfg, device),
                        "conv": m["conv"].reshape(m["conv"].shape[0], -1).float().to(device),
                        "A_log": m["A_log"].float().to(device), "dt_bias": m["dt_bias"].float().to(device),
                        "norm": m["norm"].float().to(device)}
        else:
            proj = torch.cat([m["q"], m["k"], m["v"], m["iqk"]], 0)
            M["mix"] = {"proj": _ws(proj, cfg, device), "o": _ws(m["o"], cfg, device),
                        **{k: m[k].float().to(device) for k in ("qn", "kn", "iqn", "ikn")}}
        mo = L["moe"]
        lay = mo["lowbit"]
        perm = rt.gate_up_perm(cfg.moe_inter)
        gu_blobs, d_blobs, fmts = [], [], []
        for b in lay.blobs:
            gu_blobs.append(rt.pack_planar_blob(b.gu, b.gu_s, b.gu_z, b.bits, row_perm=perm))
            d_blobs.append(rt.pack_planar_blob(b.d, b.d_s, b.d_z, b.bits))
            fmts.append(b.bits)
        router = torch.cat([mo["gate"].float(), mo["sgate"].float()], 0)
        M["moe"] = {"router": wgemm.build_weight_set([rt.pack_f16(router)], [16], router.shape[0], H, device=device),
                    "gu": wgemm.build_weight_set(gu_blobs, fmts, 2 * cfg.moe_inter, H, silu_pairs=True, device=device),
                    "d": wgemm.build_weight_set(d_blobs, fmts, H, cfg.moe_inter, device=device),
                    "sgu": _ws(_silu_perm_rows(mo["sgu"], cfg.shared_inter), cfg, device, silu_pairs=True),
                    "sd": _ws(mo["sd"], cfg, device)}
        if "ple" in L:
            P = L["ple"]
            M["ple"] = {"kv": _ws(torch.cat([P["kp"], P["vp"]], 0), cfg, device),
                        **{k: P[k].float().to(device) for k in ("nk", "nq", "nc")},
                        "conv": P["conv"].reshape(P["conv"].shape[0], -1).float().to(device)}
        E["layers"].append(M)
    return E


# ------------------------------------------------------------------------- full-size, built on the device
def _ws_chunks(chunks: list, fmts: list, rows: int, K: int, silu_pairs: bool, device) -> wgemm.WeightSet:
    """WeightSet from per-chunk runtime blocks ([n_e * tiles, KG, bb] each, experts consecutive in a chunk)."""
    tiles = (rows + 127) // 128
    total = sum(c.numel() for c in chunks)
    blob = torch.empty(total, dtype=torch.uint8, device=device)
    offs, o = [], 0
    fi = 0
    for c in chunks:
        n_e = c.shape[0] // tiles
        per = c.numel() // n_e
        blob[o: o + c.numel()] = c.reshape(-1)
        for e in range(n_e):
            offs.append(o + e * per)
        o += c.numel()
        fi += n_e
    return wgemm.WeightSet(blob, torch.tensor(offs, dtype=torch.int64, device=device),
                           torch.tensor(fmts, dtype=torch.int8, device=device), rows, K,
                           tuple(int(f) for f in fmts), silu_pairs)


def _random_experts(cfg, g, device, chunk=32, symmetric=False, lo=0, hi=None):
    """Experts [lo, hi) (default: all) of one layer, random N(0, STD) weights quantized to each expert's bits."""
    H, I = cfg.hidden_size, cfg.moe_inter
    E = cfg.n_experts if hi is None else hi
    perm = rt.gate_up_perm(I, device=device)
    gu_chunks, d_chunks, fmts = [], [], []
    e = lo
    while e < E:
        bits = cfg.bits_of(e)
        n = 1
        while e + n < E and n < chunk and cfg.bits_of(e + n) == bits:
            n += 1
        wgu = torch.randn(n, 2 * I, H, generator=g, device=device) * STD
        wgu = wgu[:, perm].reshape(n * 2 * I, H)
        q, s, z = planar.quantize_rtn(wgu, bits, symmetric)
        gu_chunks.append(rt.pack_q(q, s, z, bits))
        del wgu, q, s, z
        wd = (torch.randn(n * H, I, generator=g, device=device) * STD)
        q, s, z = planar.quantize_rtn(wd, bits, symmetric)
        d_chunks.append(rt.pack_q(q, s, z, bits))
        del wd, q, s, z
        fmts += [bits] * n
        e += n
    return (_ws_chunks(gu_chunks, fmts, 2 * I, H, True, device), _ws_chunks(d_chunks, fmts, H, I, False, device))


def random_engine(cfg, device, seed: int = 0, symmetric: bool = False, expert_shard=None) -> dict:
    """Engine weights of the configured size, generated and packed on `device` (N(0, 0.02) dense weights stored
    FP8 128x128 block-scaled, experts N(0, 0.02) RTN-quantized to their bit widths with group-128 scales).
    ``expert_shard=(rank, world)`` builds only that rank's experts (expert parallelism)."""
    e_lo, e_hi = 0, cfg.n_experts
    if expert_shard is not None:
        r, w = expert_shard
        e_lo, e_hi = r * cfg.n_experts // w, (r + 1) * cfg.n_experts // w
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    H, hc = cfg.hidden_size, cfg.hc_count
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    Hq, KV, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    iH, iD = cfg.indexer_heads, cfg.indexer_dim
    R = rank_pad(cfg)

    def rn(*s, std=STD):
        return torch.randn(*s, generator=g, device=dev) * std

    def dense(rows, K, silu=False, std=STD):
        w = rn(rows, K, std=std)
        if silu:
            w = w[rt.gate_up_perm(rows // 2, device=dev)]
        return _ws(w, cfg, dev, silu_pairs=silu)

    def hc_params(combine=True):
        w1 = torch.cat([rn(cfg.hc_rank, hc * H), torch.zeros(R - cfg.hc_rank, hc * H, device=dev)] +
                       ([rn(hc, hc * H)] if combine else []), 0)
        up = torch.cat([rn(hc * H, cfg.hc_rank, std=cfg.hc_rank ** -0.5),
                        torch.zeros(hc * H, R - cfg.hc_rank, device=dev)], 1)
        return {"norm": rn(hc * H, std=0.1), "w1": _ws(w1, cfg, dev), "w2": _ws(up, cfg, dev)}

    E = {"embed": rn(cfg.vocab_size, H, std=1.0).to(torch.bfloat16),
         "lm_head": dense(cfg.vocab_size, H), "mixer": hc_params(False), "layers": []}
    if cfg.ple_layers:
        nh = (cfg.ngram_size - 1) * cfg.heads_per_ngram
        E["ple_table"] = torch.empty(cfg.ple_rows, cfg.ple_dim, dtype=torch.uint8, device=dev)
        for a in range(0, cfg.ple_rows, 1 << 24):
            b = min(cfg.ple_rows, a + (1 << 24))
            E["ple_table"][a:b] = rn(b - a, cfg.ple_dim, std=1.0).to(torch.float8_e4m3fn).view(torch.uint8)
        E["ple_table"] = E["ple_table"].view(torch.float8_e4m3fn)
        E["ple_scale"] = 0.05
        E["ple_mult"] = (torch.randint(1, 1 << 20, (cfg.ngram_size,), generator=g, device=dev) * 2 + 1).long()
        sizes = torch.randint(cfg.ple_rows // (2 * nh), cfg.ple_rows // nh, (nh,), generator=g, device=dev).long()
        E["ple_sizes"] = sizes
        E["ple_offs"] = torch.cumsum(torch.cat([torch.zeros(1, dtype=torch.long, device=dev), sizes[:-1]]), 0)
    for l in range(cfg.num_layers):
        M = {"ahc": hc_params(), "mhc": hc_params()}
        if l in cfg.ple_layers:
            M["ple"] = {"kv": dense(hc * H + H, nh * cfg.ple_dim),
                        "nk": rn(hc * H, std=0.1), "nq": rn(hc * H, std=0.1), "nc": rn(hc * H, std=0.1),
                        "conv": rn(hc * H, cfg.ple_conv, std=0.3)}
        if cfg.layer_kind(l) == "linear":
            C = 2 * nk * dk + nv * dv
            M["mix"] = {"proj": dense(C + nv * dv + 2 * nv, H), "out": dense(H, nv * dv),
                        "conv": rn(C, cfg.conv_kernel, std=0.3),
                        "A_log": torch.log(torch.rand(nv, generator=g, device=dev) * 15 + 1),
                        "dt_bias": rn(nv, std=0.5), "norm": 1.0 + rn(dv, std=0.1)}
        else:
            M["mix"] = {"proj": dense(Hq * 2 * D + 2 * KV * D + iH * iD + iD, H), "o": dense(H, Hq * D),
                        "qn": rn(D, std=0.1), "kn": rn(D, std=0.1), "iqn": rn(iD, std=0.1), "ikn": rn(iD, std=0.1)}
        gu, d = _random_experts(cfg, g, dev, symmetric=symmetric, lo=e_lo, hi=e_hi)
        router = rn(cfg.n_experts + 1, H)
        M["moe"] = {"router": wgemm.build_weight_set([rt.pack_f16(router)], [16], router.shape[0], H, device=dev),
                    "gu": gu, "d": d, "sgu": dense(2 * cfg.shared_inter, H, silu=True),
                    "sd": dense(H, cfg.shared_inter)}
        E["layers"].append(M)
    return E


def engine_bytes(E: dict) -> dict:
    """Bytes of the engine weights by kind (expert / dense / embedding)."""
    out = {"experts": 0, "dense": 0, "embed": 0}

    def walk(x, key):
        if isinstance(x, wgemm.WeightSet):
            out["experts" if key in ("gu", "d") else "dense"] += x.nbytes()
        elif isinstance(x, dict):
            for k, v in x.items():
                walk(v, k)
        elif isinstance(x, list):
            for v in x:
                walk(v, key)
        elif torch.is_tensor(x):
            out["embed" if key in ("embed", "ple_table") else "dense"] += x.numel() * x.element_size()
    walk(E, "")
    return out

"""Random-init weights of the Dots3-Note-shaped model in oracle (dense) form and engine form.

Dense weights are rounded to their storage format first (block FP8 when ``cfg.dense_fp8``), so the oracle and
the engine multiply the same values; experts are RTN-quantized to ``cfg.bits_of(e)`` bits (3/2 in the shipped
build, dotsnote/training/README.md:218-224) and kept as planar checkpoint blobs plus dequantized copies.

Engine form: the MLA down projections, the gate projection and (DSA layers) the indexer key/weight
projections fuse into one GEMM ``a`` (the reference merges ``g_proj`` into the q/kv-a GEMM,
dotsnote/engine/arcstats_pkg/arcstats/gmerge.py:1-20); ``q_b`` and the indexer query projection (both read the
normalized q latent) fuse into ``qb``; ``kv_b`` is split into the per-head absorption matrices ``uk`` [H, dn, r]
and ``uv`` [H, dv, r] of latent-space decode attention.
"""
from __future__ import annotations

import torch

from ..formats import lowbit_file
from ..formats import runtime as rt
from ..ops import wgemm
from .fn_weights import STD, _round_dense, _round_permuted, _silu_perm_rows, _ws


def random_dense(cfg, seed: int = 0, symmetric: bool = False) -> dict:
    g = torch.Generator().manual_seed(seed)
    Hd = cfg.hidden_size
    rd = lambda *s, std=STD: torch.randn(*s, generator=g) * std  # noqa: E731
    dn, dr, dv, qr = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.q_lora_rank
    W = {"embed": rd(cfg.vocab_size, Hd, std=1.0).bfloat16().float(),
         "lm_head": _round_dense(rd(cfg.vocab_size, Hd), cfg), "norm": 1.0 + rd(Hd, std=0.1), "layers": []}
    for l in range(cfg.num_layers):
        H, kvr = cfg.heads_of(l), cfg.latent_of(l)
        # q_a / kv_a / g / indexer k,w fuse into one fp16 GEMM (fp16-rounded); the rest is block FP8
        a = {"q_a": rd(qr, Hd).half().float(), "kv_a": rd(kvr + dr, Hd).half().float(),
             "q_ln": 1.0 + rd(qr, std=0.1), "kv_ln": 1.0 + rd(kvr, std=0.1), "kr_ln": 1.0 + rd(dr, std=0.1),
             "q_b": _round_dense(rd(H * (dn + dr), qr), cfg),
             "kv_b": rd(H * (dn + dv), kvr, std=0.05).bfloat16().float(),
             "o": _round_dense(rd(Hd, H * dv), cfg), "g": rd(H, Hd).half().float()}
        if cfg.layer_kind(l) == "dsa":
            iH, iD = cfg.index_heads, cfg.index_dim
            a.update({"iq": _round_dense(rd(iH * iD, qr), cfg), "ik": rd(iD, Hd).half().float(),
                      "ik_w": 1.0 + rd(iD, std=0.1), "ik_b": rd(iD, std=0.1), "iw": rd(iH, Hd).half().float()})
        L = {"ln1": 1.0 + rd(Hd, std=0.1), "ln2": 1.0 + rd(Hd, std=0.1), "attn": a}
        if cfg.is_moe(l):
            lay = lowbit_file.random_layer(cfg.n_experts, Hd, cfg.moe_inter,
                                           [cfg.bits_of(e) for e in range(cfg.n_experts)], g, std=STD,
                                           symmetric=symmetric, n_orig=cfg.n_experts_orig)
            L["moe"] = {"gate": lay.router.float().half().float(), "bias": rd(cfg.n_experts, std=0.1),
                        "lowbit": lay, "experts_dense": [b.dense() for b in lay.blobs],
                        "shared": {"gu": _round_permuted(rd(2 * cfg.shared_inter, Hd), cfg),
                                   "d": _round_dense(rd(Hd, cfg.shared_inter), cfg)}}
        else:
            L["mlp"] = {"gu": _round_permuted(rd(2 * cfg.dense_inter, Hd), cfg),
                        "d": _round_dense(rd(Hd, cfg.dense_inter), cfg)}
        W["layers"].append(L)
    return W


def _f32(t, device):
    return t.float().to(device)


def absorb_sets(uk: torch.Tensor, uv: torch.Tensor, device) -> dict:
    """The per-head absorption matrices as two grouped fp16 weight sets, one "expert" per head, for the tcgen05
    grouped GEMM: ``uk_ws`` rows = latent r, K = dn (head h holds uk[h]^T), ``uv_ws`` rows = dv, K = r (uv[h])."""
    H, dn, r = uk.shape
    dv = uv.shape[1]
    kp = (dn + 127) // 128 * 128      # the GEMM's K is whole 128-column groups: zero columns pad a small dn
    wk = [rt.pack_f16(torch.nn.functional.pad(uk[h].t().float(), (0, kp - dn))) for h in range(H)]
    wv = [rt.pack_f16(uv[h].float()) for h in range(H)]
    return {"uk_ws": wgemm.build_weight_set(wk, [16] * H, r, kp, device=device),
            "uv_ws": wgemm.build_weight_set(wv, [16] * H, dv, r, device=device)}


ABSORB_GROUPED = __import__("os").environ.get("FW_D3_ABSORB", "bmm") == "grouped"


def _absorb_entries(uk, uv, dev, low) -> dict:
    """The dense per-head matrices (batched GEMM), or with FW_D3_ABSORB=grouped on a GPU the grouped weight sets
    of this framework's tcgen05 GEMM instead. At decode batch the batched GEMM is faster: 6 / 4 us per call
    against 34 / 22 us on a B200 (uk / uv, 128 heads, 32 tokens), because each 128-row tile of uk has a single
    128-column K group and the weight-streaming pipeline's per-tile latency dominates."""
    if dev.type == "cpu" or not ABSORB_GROUPED:
        return {"uk": uk.to(dev, low), "uv": uv.to(dev, low)}
    return absorb_sets(uk.to(dev), uv.to(dev), dev)


def to_engine(W: dict, cfg, device) -> dict:
    dev = torch.device(device)
    dn, dr, dv = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
    low = torch.float32 if dev.type == "cpu" else torch.bfloat16
    E = {"embed": W["embed"].to(dev, torch.float32 if dev.type == "cpu" else torch.bfloat16),
         "lm_head": _ws(W["lm_head"], cfg, dev), "norm": _f32(W["norm"], dev), "layers": []}
    if "vocab_range" in W:
        E["vocab_range"] = W["vocab_range"]
    for l, L in enumerate(W["layers"]):
        a = L["attn"]
        H, kvr = cfg.heads_of(l), cfg.latent_of(l)
        dsa = cfg.layer_kind(l) == "dsa"
        rows_a = [a["q_a"], a["kv_a"], a["g"]] + ([a["ik"], a["iw"]] if dsa else [])
        rows_b = [a["q_b"]] + ([a["iq"]] if dsa else [])
        kvb = a["kv_b"].view(H, dn + dv, kvr)
        M = {"ln1": _f32(L["ln1"], dev), "ln2": _f32(L["ln2"], dev),
             "attn": {"a": wgemm.build_weight_set([rt.pack_f16(torch.cat(rows_a, 0))], [16],
                                                  sum(r.shape[0] for r in rows_a), cfg.hidden_size, device=dev),
                      "qb": _ws(torch.cat(rows_b, 0), cfg, dev),
                      **_absorb_entries(kvb[:, :dn, :].contiguous(), kvb[:, dn:, :].contiguous(), dev, low),
                      "o": _ws(a["o"], cfg, dev),
                      **{k: _f32(a[k], dev) for k in ("q_ln", "kv_ln", "kr_ln")}}}
        if dsa:
            M["attn"].update({"ik_w": _f32(a["ik_w"], dev), "ik_b": _f32(a["ik_b"], dev)})
        if cfg.is_moe(l):
            mo = L["moe"]
            perm = rt.gate_up_perm(cfg.moe_inter)
            gu, d, fmts = [], [], []
            for b in mo["lowbit"].blobs:
                gu.append(rt.pack_planar_blob(b.gu, b.gu_s, b.gu_z, b.bits, row_perm=perm))
                d.append(rt.pack_planar_blob(b.d, b.d_s, b.d_z, b.bits))
                fmts.append(b.bits)
            M["moe"] = {"router": wgemm.build_weight_set([rt.pack_f16(mo["gate"].float())], [16], cfg.n_experts,
                                                         cfg.hidden_size, device=dev),
                        "bias": _f32(mo["bias"], dev),
                        "gu": wgemm.build_weight_set(gu, fmts, 2 * cfg.moe_inter, cfg.hidden_size, silu_pairs=True,
                                                     device=dev),
                        "d": wgemm.build_weight_set(d, fmts, cfg.hidden_size, cfg.moe_inter, device=dev),
                        "sgu": _ws(_silu_perm_rows(mo["shared"]["gu"], cfg.shared_inter), cfg, dev, silu_pairs=True),
                        "sd": _ws(mo["shared"]["d"], cfg, dev),
                        "expert_range": mo.get("expert_range", (0, cfg.n_experts))}
        else:
            M["mlp"] = {"gu": _ws(_silu_perm_rows(L["mlp"]["gu"], cfg.dense_inter), cfg, dev, silu_pairs=True),
                        "d": _ws(L["mlp"]["d"], cfg, dev)}
        E["layers"].append(M)
    return E


def random_engine(cfg, device, seed: int = 0, tp=None, shard_vocab: bool = False) -> dict:
    """Engine-form weights of the configured size generated and packed on `device`, without the dense fp32 copies
    of :func:`random_dense` (the full 144-expert model would need ~0.6 TB of them): dense weights N(0, 0.02) in
    their storage formats (fp16 fused down projection, block-FP8 elsewhere), experts N(0, 0.02) RTN-quantized to
    ``cfg.bits_of(e)`` bits with group-128 scales. ``tp=(rank, world)`` builds one tensor-parallel rank's shard
    (its heads, its contiguous expert range); pass the matching :func:`..parallel.tp.tp_config` view to the model.
    ``shard_vocab``: the rank keeps only its slice of the LM head (next tokens via ``D3Model.pick``)."""
    from .fn_weights import _random_experts
    dev = torch.device(device)
    rank, world = tp if tp is not None else (0, 1)
    g = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
    Hd, dn, dr, dv, qr = cfg.hidden_size, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.q_lora_rank

    def rn(*s, std=STD):
        return torch.randn(*s, generator=g, device=dev) * std

    def ws16(rows, K):
        return wgemm.build_weight_set([rt.pack_f16(rn(rows, K))], [16], rows, K, device=dev)

    low = torch.float32 if dev.type == "cpu" else torch.bfloat16
    v0, v1 = (rank * cfg.vocab_size // world, (rank + 1) * cfg.vocab_size // world) if shard_vocab else \
        (0, cfg.vocab_size)
    E = {"embed": rn(cfg.vocab_size, Hd, std=1.0).to(low), "lm_head": _ws(rn(v1 - v0, Hd), cfg, dev),
         "norm": 1.0 + rn(Hd, std=0.1), "layers": []}
    if shard_vocab:
        E["vocab_range"] = (v0, v1)
    for l in range(cfg.num_layers):
        H = cfg.heads_of(l) // world
        kvr = cfg.latent_of(l)
        dsa = cfg.layer_kind(l) == "dsa"
        iH, iD = (cfg.index_heads, cfg.index_dim) if dsa else (0, 0)
        rows_a = qr + kvr + dr + H + iD + iH
        M = {"ln1": 1.0 + rn(Hd, std=0.1), "ln2": 1.0 + rn(Hd, std=0.1),
             "attn": {"a": ws16(rows_a, Hd), "qb": _ws(rn(H * (dn + dr) + iH * iD, qr), cfg, dev),
                      **_absorb_entries(rn(H, dn, kvr, std=0.05).to(low), rn(H, dv, kvr, std=0.05).to(low),
                                        dev, low),
                      "o": _ws(rn(Hd, H * dv), cfg, dev),
                      "q_ln": 1.0 + rn(qr, std=0.1), "kv_ln": 1.0 + rn(kvr, std=0.1), "kr_ln": 1.0 + rn(dr, std=0.1)}}
        if dsa:
            M["attn"].update({"ik_w": 1.0 + rn(iD, std=0.1), "ik_b": rn(iD, std=0.1)})
        if cfg.is_moe(l):
            e0, e1 = rank * cfg.n_experts // world, (rank + 1) * cfg.n_experts // world
            gu, d = _random_experts(cfg, g, dev, lo=e0, hi=e1)
            M["moe"] = {"router": ws16(cfg.n_experts, Hd), "bias": rn(cfg.n_experts, std=0.1), "gu": gu, "d": d,
                        "sgu": _ws(rn(2 * cfg.shared_inter, Hd), cfg, dev, silu_pairs=True),
                        "sd": _ws(rn(Hd, cfg.shared_inter), cfg, dev), "expert_range": (e0, e1)}
        else:
            M["mlp"] = {"gu": _ws(rn(2 * cfg.dense_inter, Hd), cfg, dev, silu_pairs=True),
                        "d": _ws(rn(Hd, cfg.dense_inter), cfg, dev)}
        E["layers"].append(M)
    return E

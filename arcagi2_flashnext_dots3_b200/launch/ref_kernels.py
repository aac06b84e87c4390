"""Same-box comparison of the reference's own kernels with this framework's, on identical shapes and inputs.

The reference's serving engine cannot run on this image (its FN and D3 model classes live in a vLLM 0.30/0.32
overlay; the image has vLLM 0.22), but its hot kernels are plain Triton + torch. Its only installable package,
``arcstats`` (dotsnote/engine/arcstats_pkg, installed unmodified into ``baseline/_ref`` by pip), carries them:

* ``moe``: ``arcstats.lowbit_moe.LowbitMoE`` (dotsnote/engine/arcstats_pkg/arcstats/lowbit_moe.py:336-437), the
  reference's mixed 2/3/4-bit grouped MoE with planar codes, group-128 fp16 scales and uint8 zeros, routing
  aligned by vLLM's ``moe_align_block_size``, silu*up by ``torch.ops._C.silu_and_mul``; its stock entry point,
  called on the FN decode layer (320 experts, hidden 2560, expert FFN 640, top-10, 4/3-bit) and on the D3 layer
  (144 experts, 3/2-bit). Ours: routing plan + scatter + two grouped GEMV launches + combine
  (``ops.fn_ops`` / ``ops.wgemm``), the same sequence ``models.fn`` runs.
* ``dense``: ``arcstats.w8a8_ws.ws_mm`` (w8a8_ws.py:149), the reference's block-FP8 decode GEMM, on the FN dense
  projection shapes at the decode batch, fed bf16 activations with its fused per-128 FP8 quantization; the best of
  a small config grid per shape (the reference tunes per shape at start-up). Ours: ``wgemm.matmul`` (FP8
  128x128 blocks, tcgen05).

Timing: each arm's op sequence is captured R times into one CUDA graph (both engines decode under CUDA graphs),
rotating over enough weight copies that the bytes read per replay exceed the 126 MB L2; time = replay / R
(CUDA events, after warm-up). Each line also reports the max relative difference between the two outputs.

    python -m arcagi2_flashnext_dots3_b200.launch.ref_kernels [--tokens 64] [--reps 20] [--which moe,dense]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "baseline", "_ref")
L2_BYTES = 126 << 20


def _import_reference():
    if not os.path.isdir(os.path.join(REF, "arcstats")):
        raise RuntimeError("reference package not installed in baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import arcstats.lowbit_moe as lm
    import arcstats.w8a8_ws as ws
    return lm, ws


def _graph_time(fn, reps: int, warmup: int = 3) -> float:
    """ms per call of fn() (fn(i) takes the repetition index) from one CUDA graph of `reps` calls."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(warmup):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(3):
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / reps)
    del g
    return best


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-12))


# --------------------------------------------------------------------------------------------------- MoE
def _layer_codes(E, N, K, bits_of, g, dev):
    """Random codes, fp16 scales and uint8 zeros per expert (shared by both arms)."""
    codes, scales, zeros = [], [], []
    for e in range(E):
        b = bits_of(e)
        codes.append(torch.randint(0, 1 << b, (N, K), generator=g, device=dev, dtype=torch.int32).to(torch.uint8))
        scales.append((torch.rand(N, K // 128, generator=g, device=dev) * 0.004 + 0.002).half())
        zeros.append(torch.randint(0, 1 << b, (N, K // 128), generator=g, device=dev, dtype=torch.int32)
                     .to(torch.uint8))
    return codes, scales, zeros


def _our_expert_set(codes, scales, zeros, bits, silu: bool, dev):
    from ..formats import runtime as rt
    from ..ops import wgemm
    blobs = []
    N, K = codes[0].shape
    perm = rt.gate_up_perm(N // 2, device=dev) if silu else None
    for q, s, z, b in zip(codes, scales, zeros, bits):
        if perm is not None:   # the silu epilogue wants gate/up rows interleaved; same weights, permuted rows
            q, s, z = q[perm], s[perm], z[perm]
        blobs.append(rt.pack_q(q.int(), s, z, b))
    return wgemm.build_weight_set(blobs, bits, N, K, silu_pairs=silu, device=dev)


def bench_moe(name, E, H, I, top_k, bits_of, T, reps, lm, dev, seed=0):
    from ..ops import fn_ops as ops
    from ..ops import wgemm
    g = torch.Generator(device=dev).manual_seed(seed)
    bits = [bits_of(e) for e in range(E)]
    gu = _layer_codes(E, 2 * I, H, bits_of, g, dev)
    dn = _layer_codes(E, H, I, bits_of, g, dev)
    layer_bytes = sum(c.numel() * b / 8 + s.numel() * 3 for c, s, b in zip(gu[0] + dn[0], gu[1] + dn[1], bits + bits))
    n_copies = max(1, min(4, int(2 * L2_BYTES // layer_bytes) + 1))
    ref_layers = [lm.LowbitMoE(lm.LowbitProj(bits, *gu, dev), lm.LowbitProj(bits, *dn, dev), E)
                  for _ in range(n_copies)]
    our = [(_our_expert_set(*gu, bits, True, dev), _our_expert_set(*dn, bits, False, dev)) for _ in range(n_copies)]
    x = (torch.randn(T, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev)
    topk_w, topk_ids = torch.softmax(logits, -1).topk(top_k, -1)
    topk_w = (topk_w / topk_w.sum(-1, keepdim=True)).float()
    ids32 = topk_ids.to(torch.int32).contiguous()
    x16 = x.half()
    P = T * top_k
    n_tile = wgemm.GEMV_MAX_TOK
    max_items = (P + n_tile - 1) // n_tile + E
    h = torch.zeros(T, H, dtype=torch.float32, device=dev)
    zero_sh = torch.zeros(T, H, dtype=torch.float32, device=dev)
    no_gate = torch.full((T,), float("-inf"), device=dev)
    ones = torch.ones(T, 1, dtype=torch.float32, device=dev)
    act = torch.empty(P, I, dtype=torch.float16, device=dev)
    ypair = torch.empty(P, H, dtype=torch.float32, device=dev)

    def ours(i):
        gu_ws, d_ws = our[i % n_copies]
        pair_pos, items, n_items = ops.moe_plan(ids32, E, n_tile, max_items)
        xs = ops.moe_scatter(x16, pair_pos)
        wgemm.gemv_grouped(xs, gu_ws, items, n_items, max_items, act, epi=wgemm.EPI_SILU_MUL)
        wgemm.gemv_grouped(act, d_ws, items, n_items, max_items, ypair)
        h.zero_()
        ops.moe_combine(h, ypair, pair_pos, topk_w, zero_sh, no_gate, ones)

    out_ref = {}

    def ref(i):
        out_ref["y"] = ref_layers[i % n_copies](x, topk_w, ids32)

    t_ours = _graph_time(ours, reps)
    t_ref = _graph_time(ref, reps)
    ours(0)
    ref(0)
    torch.cuda.synchronize()
    return {"op": f"moe {name}", "shape": f"E{E} H{H} I{I} top{top_k} T{T}", "bits": sorted(set(bits)),
            "ref_us": round(t_ref * 1e3, 1), "ours_us": round(t_ours * 1e3, 1),
            "speedup": round(t_ref / t_ours, 2), "max_rel_diff": round(_rel(h, out_ref["y"]), 4),
            "weight_mb": round(layer_bytes / 2**20, 1),
            "ours_gbs": round(layer_bytes / (t_ours * 1e-3) / 1e9, 0)}


# ------------------------------------------------------------------------------------------------- dense
REF_DENSE_CFGS = [{"BM": 64, "NSUB": 1, "BN": bn, "SPLIT_K": sk, "FUSE_Q": 1, "num_warps": 4, "num_stages": 3}
                  for bn in (32, 64, 128) for sk in (1, 2, 4, 8)]


def bench_dense(N, K, T, reps, wsm, dev, seed=0):
    from ..formats import runtime as rt
    from ..ops import wgemm
    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randn(N, K, generator=g, device=dev) * 0.02
    w8, sc = rt.quantize_fp8_blocks(w)
    n_copies = max(1, min(16, int(2 * L2_BYTES // (N * K)) + 1))
    ref_w = [(w8.clone(), sc.clone()) for _ in range(n_copies)]
    our_w = [wgemm.build_weight_set([rt.pack_fp8(w8, sc)], [8], N, K, device=dev) for _ in range(n_copies)]
    x = (torch.randn(T, K, generator=g, device=dev)).to(torch.bfloat16)
    x16 = x.half()
    y = torch.empty(T, N, dtype=torch.float32, device=dev)

    def ours(i):
        wgemm.matmul(x16, our_w[i % n_copies], out=y)

    best = (float("inf"), None)
    out_ref = {}
    for cfg in REF_DENSE_CFGS:
        if cfg["SPLIT_K"] > K // 128:
            continue

        def ref(i, cfg=cfg):
            a, s = ref_w[i % n_copies]
            out_ref["y"] = wsm.ws_mm(x, None, a, s, cfg)
        try:
            t = _graph_time(ref, reps)
        except Exception:
            continue
        if t < best[0]:
            best = (t, cfg)
    t_ours = _graph_time(ours, reps)
    a, s = ref_w[0]
    yr = wsm.ws_mm(x, None, a, s, best[1])
    ours(0)
    torch.cuda.synchronize()
    return {"op": "dense fp8", "shape": f"N{N} K{K} T{T}", "ref_us": round(best[0] * 1e3, 1),
            "ours_us": round(t_ours * 1e3, 1), "speedup": round(best[0] / t_ours, 2),
            "ref_cfg": {k: best[1][k] for k in ("BN", "SPLIT_K")}, "max_rel_diff": round(_rel(y, yr), 4),
            "ours_gbs": round(N * K / (t_ours * 1e-3) / 1e9, 0)}


def fn_dense_shapes(cfg):
    H, hc = cfg.hidden_size, cfg.hc_count
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    C = 2 * nk * dk + nv * dv
    from ..models.fn_weights import rank_pad
    R = rank_pad(cfg)
    return [("gdn proj", C + nv * dv + 2 * nv, H), ("gdn out", H, nv * dv), ("shared gate_up", 2 * cfg.shared_inter, H),
            ("shared down", H, cfg.shared_inter), ("hc down", R + hc, hc * H), ("hc up", hc * H, R)]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--which", default="moe,dense")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    from ..config import d3_config, fn_config
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    try:
        lm, wsm = _import_reference()
    except Exception as e:   # the reference package or one of its imports is missing
        print(json.dumps({"impl": "reference-kernels", "unavailable": f"{type(e).__name__}: {e}"}))
        return
    rows = []
    fc, dc = fn_config(), d3_config()
    if "moe" in a.which:
        rows.append(bench_moe("fn", fc.n_experts, fc.hidden_size, fc.moe_inter, fc.top_k, fc.bits_of, a.tokens,
                              a.reps, lm, dev))
        rows.append(bench_moe("d3", dc.n_experts, dc.hidden_size, dc.moe_inter, dc.top_k, dc.bits_of, a.tokens,
                              a.reps, lm, dev))
    if "dense" in a.which:
        for name, N, K in fn_dense_shapes(fc):
            r = bench_dense(N, K, a.tokens, a.reps, wsm, dev)
            r["op"] = f"dense fp8 ({name})"
            rows.append(r)
    for r in rows:
        print(json.dumps(r), flush=True)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()

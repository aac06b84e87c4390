"""Kernel microbenchmarks (CUDA-event timed, warm-up, max over repetitions reported as median).

    python -m arcagi2_flashnext_dots3_b200.launch.kbench moe   [--tokens 64] [--experts 320] [--reps 20]
    python -m arcagi2_flashnext_dots3_b200.launch.kbench dense [--tokens 64] [--reps 20]
    python -m arcagi2_flashnext_dots3_b200.launch.kbench attn  [--tokens 64] [--ctx 9000] [--reps 20]
    python -m arcagi2_flashnext_dots3_b200.launch.kbench gdn   [--tokens 64] [--reps 20]
    python -m arcagi2_flashnext_dots3_b200.launch.kbench mla   [--tokens 64] [--ctx 9000] [--reps 20]
    python -m arcagi2_flashnext_dots3_b200.launch.kbench absorb [--tokens 32] [--reps 20]

Counterpart of the reference's micro-benchmarks and startup gates (dotsnote/kaggle/runtime_dataset/bench_*.py,
run_l4.py:435 `run_bench`): each case prints one JSON line with the median device time and the achieved
bandwidth against the bytes the kernel must move. Inputs are larger than L2 where the case streams weights.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch


def _time(fn, reps, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def bench_moe(args):
    from ..config import fn_config
    from ..models.fn_weights import _random_experts
    from ..ops import fn_ops as ops
    from ..ops import native, wgemm
    cfg = fn_config(n_experts=args.experts)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    gu, d = _random_experts(cfg, g, dev)
    T, E, k = args.tokens, cfg.n_experts, cfg.top_k
    logits = torch.randn(T, E + 1, device=dev, generator=g)
    ids, w = ops.moe_route(logits, E, k)
    P = T * k
    n_tile = wgemm.pick_n_tile(max(1, 2 * P // E))
    max_items = (P + n_tile - 1) // n_tile + E
    pp, items, n_items = ops.moe_plan(ids, E, n_tile, max_items)
    x = torch.randn(T, cfg.hidden_size, device=dev, generator=g).half()
    xs = ops.moe_scatter(x, pp)
    act = torch.empty(P, cfg.moe_inter, dtype=torch.float16, device=dev)
    yp = torch.empty(P, cfg.hidden_size, dtype=torch.float32, device=dev)
    touched = torch.unique(ids).tolist()
    bytes_gu = sum(gu.row_tiles * gu.kg * (8576 if cfg.bits_of(e) == 4 else 7040) for e in touched)
    bytes_d = sum(d.row_tiles * d.kg * (8576 if cfg.bits_of(e) == 4 else 7040) for e in touched)
    t_gu = _time(lambda: wgemm.grouped(xs, gu, items, n_items, max_items, act, epi=wgemm.EPI_SILU_MUL,
                                       n_tile=n_tile), args.reps)
    t_d = _time(lambda: wgemm.grouped(act, d, items, n_items, max_items, yp, n_tile=n_tile), args.reps)
    # CUDA-core grouped GEMV on a plan of <= 8 tokens per item
    mi8 = (P + 7) // 8 + E
    pp8, items8, n8 = ops.moe_plan(ids, E, 8, mi8)
    xs8 = ops.moe_scatter(x, pp8)
    t_gu8 = _time(lambda: wgemm.gemv_grouped(xs8, gu, items8, n8, mi8, act, epi=wgemm.EPI_SILU_MUL, kernel="dp4a"),
                  args.reps)
    t_d8 = _time(lambda: wgemm.gemv_grouped(act, d, items8, n8, mi8, yp, kernel="dp4a"), args.reps)
    # tcgen05 kind::i8 on the same plan
    t_gui = _time(lambda: wgemm.gemv_grouped(xs8, gu, items8, n8, mi8, act, epi=wgemm.EPI_SILU_MUL, kernel="i8"),
                  args.reps)
    t_di = _time(lambda: wgemm.gemv_grouped(act, d, items8, n8, mi8, yp, kernel="i8"), args.reps)
    native.check_error()
    for name, t, b in (("moe_gate_up", t_gu, bytes_gu), ("moe_down", t_d, bytes_d),
                       ("moe_gate_up_gemv", t_gu8, bytes_gu), ("moe_down_gemv", t_d8, bytes_d),
                       ("moe_gate_up_i8", t_gui, bytes_gu), ("moe_down_i8", t_di, bytes_d)):
        print(json.dumps({"case": name, "tokens": T, "experts": E, "touched": len(touched), "n_tile": n_tile,
                          "ms": round(t, 4), "MB": round(b / 1e6, 1), "GBps": round(b / t / 1e6, 1)}))


def bench_route(args):
    """Router top-k (softmax over the experts, top-k, renormalize) at the decode batch, graph-timed."""
    from ..config import fn_config
    from ..ops import fn_ops as ops
    cfg = fn_config()
    dev = torch.device("cuda")
    logits = torch.randn(args.tokens, cfg.n_experts + 1, device=dev)
    ops.moe_route(logits, cfg.n_experts, cfg.top_k)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(10):
            ops.moe_route(logits, cfg.n_experts, cfg.top_k)
    t = _time(g.replay, args.reps) / 10
    print(json.dumps({"case": "moe_route", "tokens": args.tokens, "experts": cfg.n_experts, "k": cfg.top_k,
                      "us": round(t * 1e3, 2)}))


def bench_dense(args):
    """Dense FP8 projections at decode batch: the tcgen05 kind::f8f6f4 GEMM (per-group FP8 activations, the
    default) against the weight-dequant kind::f16 GEMM. Each arm rotates over enough weight copies that every
    replay streams more than the 126 MB L2 from HBM; 10 launches per CUDA graph."""
    from ..ops import native, wgemm
    dev = torch.device("cuda")
    T = args.tokens
    shapes = [("hc_down", 388, 10240), ("hc_up", 10240, 384), ("gdn_proj", 16480, 2560), ("gdn_out", 2560, 6144),
              ("attn_proj", 11904, 2560), ("attn_o", 2560, 4096), ("router", 321, 2560),
              ("shared_gu", 1280, 2560), ("shared_d", 2560, 640)]

    def graph_us(fn, copies):
        fn(copies[0])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(10):
                fn(copies[i % len(copies)])
        t = _time(g.replay, args.reps) / 10
        del g
        return t * 1e3

    for name, R, K in shapes:
        if args.only and name not in args.only.split(","):
            continue
        ws0 = wgemm.dense_fp8(torch.randn(R, K, device=dev) * 0.02)
        n = max(1, min(10, -(-(256 << 20) // ws0.nbytes())))
        copies = [ws0] + [wgemm.WeightSet(ws0.blob.clone(), ws0.exp_off, ws0.exp_fmt, R, K, ws0.fmts)
                          for _ in range(n - 1)]
        for c in copies:
            c.f8_operands()
        x = torch.randn(T, K, device=dev).half()
        out = torch.empty(T, R, device=dev)
        nt_old, ks_old = wgemm.dense_plan(T, ws0)
        t_old = graph_us(lambda w: wgemm.matmul(x, w, out=out, n_tile=nt_old, k_splits=ks_old), copies)
        t_f8 = graph_us(lambda w: wgemm.f8_linear(x, w, out), copies)
        nt, s = wgemm.f8_plan(T, ws0)
        b = R * K
        sweep = {}
        if args.sweep:
            for ss in range(1, 9):
                if ss <= K // 128:
                    sweep[f"s{ss}"] = round(graph_us(lambda w: wgemm.f8_linear(x, w, out, nt=nt, splits=ss),
                                                     copies), 1)
        print(json.dumps({"case": name, "rows": R, "K": K, "tokens": T, "weight_MB": round(b / 1e6, 2),
                          "f16_dequant_us": round(t_old, 1), "f8_us": round(t_f8, 1), "f8_plan": [nt, s],
                          "f8_GBps": round(b / t_f8 / 1e3, 1), "f8_sweep_us": sweep}))
    native.check_error()


def bench_attn(args):
    from ..config import fn_config
    from ..models.fn import allocate_caches
    from ..ops import fn_ops as ops
    from ..ops import native
    cfg = fn_config()
    dev = torch.device("cuda")
    B = args.tokens
    one_attn = fn_config(num_layers=cfg.full_attn_interval)  # exactly one attention layer's caches
    c = allocate_caches(one_attn, dev, B, args.ctx + 64, block_size=64)
    nb = c.block_table.shape[1]
    c.block_table.copy_(torch.arange(B * nb, dtype=torch.int32, device=dev).view(B, nb))
    for t in (c.k[0], c.v[0]):
        t.copy_(torch.randn(t.shape, device=dev).to(t.dtype))
    c.comp[0].copy_(torch.randn(c.comp[0].shape, device=dev).to(c.comp[0].dtype))
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    pos = torch.full((B,), args.ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, cfg.n_heads, cfg.head_dim, device=dev)
    gate = torch.randn(B, cfg.n_heads * cfg.head_dim, device=dev)
    iq = torch.randn(B, cfg.indexer_heads, cfg.indexer_dim, device=dev)
    sel, sp = ops.qsa_select(iq, c.comp[0], slots, pos, cfg)
    t_sel = _time(lambda: ops.qsa_select(iq, c.comp[0], slots, pos, cfg), args.reps)
    t_att = _time(lambda: ops.attn_decode(q, gate, c.k[0], c.v[0], c.block_table, slots, pos, sel, sp, cfg),
                  args.reps)
    native.check_error()
    keys = cfg.indexer_budget + cfg.indexer_ratio
    kv_bytes = B * cfg.n_kv_heads * keys * cfg.head_dim * 2
    comp_bytes = B * (args.ctx // cfg.indexer_ratio) * cfg.indexer_dim * 2
    print(json.dumps({"case": "indexer_select", "rows": B, "ctx": args.ctx, "ms": round(t_sel, 4),
                      "GBps": round(comp_bytes / t_sel / 1e6, 1)}))
    print(json.dumps({"case": "sparse_attn_decode", "rows": B, "ctx": args.ctx, "ms": round(t_att, 4),
                      "GBps": round(kv_bytes / t_att / 1e6, 1)}))


def bench_gdn(args):
    from ..config import fn_config
    from ..ops import fn_ops as ops
    from ..ops import native
    cfg = fn_config()
    dev = torch.device("cuda")
    B = args.tokens
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    C = 2 * nk * dk + nv * dv
    proj = torch.randn(B, C + nv * dv + 2 * nv, device=dev)
    conv_w = torch.randn(C, cfg.conv_kernel, device=dev) * 0.3
    conv_state = torch.randn(B, C, cfg.conv_kernel - 1, device=dev)
    ssm = (torch.randn(B, nv, dk, dv, device=dev) * 0.05).bfloat16()
    A_log = torch.randn(nv, device=dev)
    dt = torch.randn(nv, device=dev)
    nw = torch.randn(dv, device=dev)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    t = _time(lambda: ops.gdn_step(proj, conv_w, conv_state, ssm, A_log, dt, nw, slots, cfg), args.reps)
    native.check_error()
    b = 2 * ssm.numel() * 2
    print(json.dumps({"case": "gdn_decode", "rows": B, "ms": round(t, 4), "state_MB": round(b / 1e6, 1),
                      "GBps": round(b / t / 1e6, 1)}))


def bench_gdn_prefill(args):
    """GDN prefill of one sequence of --ctx tokens at FN size (48 value heads, 16 key heads, 128 x 128 states):
    the chunked tcgen05 delta rule against the sequential recurrence, plus the chunk kernel's per-phase times
    (%globaltimer of one CTA, averaged over its chunks)."""
    from ..config import fn_config
    from ..ops import native
    cfg = fn_config()
    dev = torch.device("cuda")
    n = args.ctx
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    Cq = 2 * nk * dk + nv * dv
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(n, Cq, device=dev, generator=g)
    proj = torch.randn(n, Cq + nv * dv + 2 * nv, device=dev, generator=g)
    ssm = (torch.randn(2, nv, dk, dv, device=dev, generator=g) * 0.05).bfloat16()
    A_log = torch.log(torch.rand(nv, device=dev, generator=g) * 0.2 + 0.01)
    dt = torch.randn(nv, device=dev, generator=g) * 0.3
    nw = torch.rand(dv, device=dev, generator=g) + 0.5
    slots = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty(n, nv * dv, dtype=torch.float16, device=dev)
    err = native.err_word(dev)
    C = native.C()
    trace = torch.zeros((n + 63) // 64 * 16, dtype=torch.int64, device=dev)

    def chunked(tr=None):
        C.gdn_chunk(qkv, proj, ssm, A_log, dt, nw, slots, out, nk, nv, n, cfg.rms_eps, 0, err,
                    native.DEFAULT_TIMEOUT_NS, tr)
    t = _time(chunked, args.reps)
    chunked(trace)
    torch.cuda.synchronize()
    native.check_error()
    tr = trace.view(-1, 16).double().cpu()
    marks = torch.cat([tr[:-1, :10], tr[1:, :1]], 1)            # phase starts P0..P9, next chunk's P0
    steps = (marks[:, 1:] - marks[:, :-1]).mean(0) / 1e3
    per_chunk = ((tr[1:, 0] - tr[:-1, 0]).mean() / 1e3).item() if tr.shape[0] > 1 else 0.0
    sub = {"p0_rows_us": round(((tr[:, 10] - tr[:, 0]).mean() / 1e3).item(), 2),
           "p9_out_us": round(((tr[:, 11] - tr[:, 9]).mean() / 1e3).item(), 2),
           "p9_state_us": round(((tr[:, 12] - tr[:, 11]).mean() / 1e3).item(), 2)}
    print(json.dumps({"case": "gdn_prefill_chunked", "tokens": n, "heads": nv, "ms": round(t, 4),
                      "tok_per_s_layer": round(n / t * 1e3, 1), "chunk_us": round(per_chunk, 2),
                      "phase_us": [round(x, 2) for x in steps.tolist()], **sub}))


def bench_mla(args):
    """D3 latent attention: tcgen05 kernel vs the CUDA-core kernel, DSA (128 heads, 512+64, top-2048) and SWA
    (64 heads, 1024+64, window 513) decode rows."""
    from ..ops import d3_ops
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    T, ctx, bs = args.tokens, args.ctx, 64
    for kind, H, kvr, topk, window in (("dsa", 128, 512, 2048, 0), ("swa", 64, 1024, 0, 513)):
        D = kvr + 64
        mb = (ctx + bs) // bs + 1
        cache = (torch.randn(T * mb, bs, D, device=dev, generator=g) * 0.5).to(torch.float8_e4m3fn)
        bt = torch.randperm(T * mb, device=dev, generator=g).to(torch.int32).view(T, mb).contiguous()
        slots = torch.arange(T, dtype=torch.int32, device=dev)
        pos = torch.full((T,), ctx - 1, dtype=torch.int32, device=dev)
        q_lat = (torch.randn(H, T, kvr, device=dev, generator=g) * 0.3).bfloat16()
        q_pe = torch.randn(T, H, 64, device=dev, generator=g) * 0.3
        sel = None
        if topk:
            sel = torch.stack([torch.randperm(ctx, device=dev, generator=g)[:topk] for _ in range(T)]).to(torch.int32)
        n = topk if topk else min(window, ctx)
        flops = 2 * T * H * n * (D + kvr)
        byts = T * n * D
        row = {"case": f"mla_{kind}", "rows": T, "heads": H, "keys": n}
        for impl, cc in (("tc", False), ("cuda_core", True)):
            d3_ops._MLA_CUDA_CORE = cc
            t = _time(lambda: d3_ops.mla_attn(q_lat, q_pe, cache, bt, slots, pos, 1, sel, window, 0.07), args.reps)
            row[impl + "_us"] = round(t * 1e3, 1)
            row[impl + "_TFLOPs"] = round(flops / t / 1e9, 1)
        row["row_GBps_tc"] = round(byts / (row["tc_us"] * 1e-6) / 1e9, 1)
        d3_ops._MLA_CUDA_CORE = False
        print(json.dumps(row), flush=True)


def bench_absorb(args):
    """D3 per-head latent absorption (q_lat = q_nope[h] @ uk[h], o[h] = o_lat[h] @ uv[h]^T): this framework's
    grouped tcgen05 GEMM (one expert per head) against torch.bmm (cuBLAS), CUDA-graph timed over weight copies
    larger than L2."""
    from ..models import d3_weights
    from ..models.d3 import D3Model
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    T = args.tokens
    for kind, H, r in (("dsa", 128, 512), ("swa", 64, 1024)):
        copies = 4
        uk = [(torch.randn(H, 128, r, device=dev, generator=g) * 0.05).bfloat16() for _ in range(copies)]
        uv = [(torch.randn(H, 128, r, device=dev, generator=g) * 0.05).bfloat16() for _ in range(copies)]
        sets = [d3_weights.absorb_sets(a, b, dev) for a, b in zip(uk, uv)]
        m = D3Model.__new__(D3Model)
        m.device = dev
        qn = (torch.randn(H, T, 128, device=dev, generator=g)).bfloat16()
        ol = (torch.randn(H, T, r, device=dev, generator=g)).bfloat16()
        row = {"case": f"absorb_{kind}", "heads": H, "latent": r, "tokens": T,
               "weight_MB_per_call": round(H * 128 * r * 2 / 2**20, 1)}
        for which, x in (("uk", qn), ("uv", ol)):
            def ours(i, which=which, x=x):
                m._absorb(x, sets[i % copies], which)

            def ref(i, which=which, x=x):
                if which == "uk":
                    torch.bmm(x, uk[i % copies])
                else:
                    torch.bmm(x, uv[i % copies].transpose(1, 2))
            for name, fn in (("ours", ours), ("cublas", ref)):
                from .ref_kernels import _graph_time
                row[f"{which}_{name}_us"] = round(_graph_time(fn, args.reps) * 1e3, 1)
        print(json.dumps(row), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["moe", "dense", "attn", "gdn", "mla", "absorb", "route", "gdn_prefill",
                                     "all"])
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--experts", type=int, default=320)
    ap.add_argument("--ctx", type=int, default=9000)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--sweep", action="store_true", help="dense: time every n_tile x split-K combination")
    ap.add_argument("--only", default="", help="dense: comma-separated case names")
    args = ap.parse_args()
    cases = {"moe": bench_moe, "dense": bench_dense, "attn": bench_attn, "gdn": bench_gdn, "mla": bench_mla,
             "route": bench_route, "gdn_prefill": bench_gdn_prefill,
             "absorb": bench_absorb}
    for name, fn in cases.items():
        if args.case in (name, "all"):
            fn(args)


if __name__ == "__main__":
    main()

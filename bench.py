#!/usr/bin/env python
"""Headline benchmark: generated tokens/s of Flash-Next-shaped 3/4-bit MoE decode on N B200s (max over ranks).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--global-batch B]

For N > 1 launch with torchrun (one rank per GPU). Each rank serves `--batch` concurrent sequences whose caches
hold synthetic 6k-12k-token contexts (random-init weights of the full architecture, random cache state of those
lengths: prefill is outside the measured decode metric). Rank 0 prints one JSON line. `--global-batch B` switches
to strong scaling: B sequences in total (B / N per rank), e.g. 64 over 8 GPUs for the TPxEP-8 serving config.

* value: device time of K decode steps (CUDA events around K replays of the captured decode graph = all 48
  layers + LM head + argmax), max over ranks; tokens/s = N * batch / step time.
* e2e: the same decode through the public API (`LLM.step()`): every step copies the input ids host->device from
  pinned memory, replays the graph and reads the new tokens back device->host; wall time, max over ranks.
* The ~35 GB of weights streamed per step are far larger than L2 (126 MB), so no L2 flush is needed.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_TOKS = 1120.0  # the reference's published FN generated tok/s (4x L4, RC9 Kaggle run)
METRIC = "generated tok/s (box, max over ranks) 3/4-bit MoE decode @1/2/4/8 B200; p50 TPOT"


def reference_arm(args):
    reason = ("the reference serves Qwen3.8-Flash-Next only through vLLM 0.32 with its `fnext` overlay patches "
              "(model class qwen4_exp); this image has vLLM 0.22, which has no qwen4_exp model, and the reference "
              "ships no engine of its own. Its installable `arcstats` package (baseline/_ref) carries its MoE and "
              "FP8 GEMM kernels, which launch/ref_kernels.py times against ours on identical decode shapes")
    print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": reason, "n_gpus": args.gpus}))


class ClockSampler:
    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) > 8 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 8 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) > 8:
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def count_launches(model, step_fn):
    """Run one eager step with counting wrappers around the extension's entry points; returns kernel launches
    of this repository's kernels per step."""
    from arcagi2_flashnext_dots3_b200.ops import native
    C = native.C()
    per_call = {"gdn_step": 2, "qsa_prep": 2, "qsa_select": 2, "attn_decode": 2, "ep_gather": 2, "ple_mix": 3}
    names = [n for n in dir(C) if not n.startswith("_") and callable(getattr(C, n)) and n != "sm_count"]
    counts = {}
    orig = {}
    for n in names:
        f = getattr(C, n)
        orig[n] = f

        def wrap(*a, _f=f, _n=n, **k):
            r = _f(*a, **k)
            # wgemm and f8_linear report how many kernels they launched (a split-K reduce, the activation quantizer)
            counts[_n] = counts.get(_n, 0) + (r if _n in ("wgemm", "f8_linear") and isinstance(r, int) else 1)
            return r
        setattr(C, n, wrap)
    try:
        step_fn()
    finally:
        for n, f in orig.items():
            setattr(C, n, f)
    return sum(per_call.get(n, 1) * c for n, c in counts.items()), counts


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="sequences per rank (weak scaling)")
    ap.add_argument("--global-batch", type=int, default=0,
                    help="strong scaling: this many sequences in total, split evenly over the ranks (overrides --batch)")
    ap.add_argument("--ctx-min", type=int, default=6144)
    ap.add_argument("--ctx-max", type=int, default=12288)
    ap.add_argument("--e2e-steps", type=int, default=0, help="0 = same as --steps")
    ap.add_argument("--layers", type=int, default=0, help="debug only: fewer layers (result marked invalid)")
    ap.add_argument("--ep", default="auto", choices=["auto", "on", "off"],
                    help="expert parallelism across the GPUs (auto: on when more than one GPU)")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"], help="EP exchange: in-kernel NVLink or NCCL")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    import torch.distributed as dist
    from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_config
    from arcagi2_flashnext_dots3_b200.engine.llm import LLM, DecodeGraph
    from arcagi2_flashnext_dots3_b200.models.fn_weights import engine_bytes, random_engine
    from arcagi2_flashnext_dots3_b200.ops import native, wgemm
    from arcagi2_flashnext_dots3_b200.parallel.ep import EPGroup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    scaling = "weak"
    if args.global_batch:
        if args.global_batch % world:
            raise SystemExit(f"--global-batch {args.global_batch} is not a multiple of {world} ranks")
        args.batch, scaling = args.global_batch // world, "strong"
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    kw = {}
    if args.layers:
        kw["num_layers"] = args.layers
    cfg = fn_config(**kw)
    use_ep = world > 1 and args.ep != "off" or args.ep == "on"
    t0 = time.time()
    W = random_engine(cfg, dev, seed=1234 + rank, expert_shard=(rank, world) if use_ep else None)
    torch.cuda.synchronize()
    t_w = time.time() - t0
    nbytes = engine_bytes(W)
    K, Wm = args.steps, args.warmup
    E2E = args.e2e_steps or K
    max_new = Wm + K + E2E + 8
    ec = EngineConfig(max_seqs=args.batch, max_model_len=args.ctx_max + max_new + 64, block_size=64,
                      kv_dtype="fp8", graph_batch_sizes=(args.batch,))
    ep = EPGroup(cfg, rank, world, dev, max_tokens=args.batch, comm=args.comm,
                 timeout_ns=int(20e9)) if use_ep else None
    llm = LLM(cfg, W, dev, ec, ep=ep)
    g = torch.Generator().manual_seed(100 + rank)
    lengths = torch.randint(args.ctx_min, args.ctx_max + 1, (args.batch,), generator=g).tolist()
    seqs = llm.synthesize_context(lengths, max_new)

    # ---------------------------------------------------------------- device-timed decode (graph replay)
    dg = DecodeGraph(llm.model, args.batch, advance=True, scratch_slot=llm.scratch)
    dg.ids.copy_(torch.tensor([s.out[-1] for s in seqs], dtype=torch.int32))
    dg.slots.copy_(torch.tensor([s.slot for s in seqs], dtype=torch.int32))
    dg.positions.copy_(torch.tensor([s.pos for s in seqs], dtype=torch.int32))
    launches, launch_detail = count_launches(llm.model, dg._body)   # one eager step (also a warm-up)
    dg.capture()
    for _ in range(Wm):
        dg.run()
    torch.cuda.synchronize()
    native.check_error(dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(K):
        dg.run()
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    native.check_error(dev)
    ms = ev0.elapsed_time(ev1) / K
    # per-step distribution (p50 TPOT): time a few steps individually
    per = []
    for _ in range(min(10, K)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dg.run()
        b.record()
        torch.cuda.synchronize()
        per.append(a.elapsed_time(b))
    # positions advanced inside the graph; bring the host view in sync for the e2e phase
    pos_now = dg.positions.cpu().tolist()
    ids_now = dg.ids.cpu().tolist()
    for s, p, t in zip(seqs, pos_now, ids_now):
        s.pos, s.out[-1] = p, t
    del dg
    # ---------------------------------------------------------------- end-to-end through the public API
    llm.step()  # captures the bucket graph (warm-up)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t1 = time.perf_counter()
    toks = 0
    for _ in range(E2E):
        toks += len(llm.step())
    t2 = time.perf_counter()
    e2e_ms = (t2 - t1) * 1000 / E2E
    e2e_tok_step = toks / E2E
    native.check_error(dev)

    vals = torch.tensor([ms, e2e_ms, statistics.median(per)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms, p50 = vals.tolist()
    total_batch = args.batch * world
    value = total_batch / (ms / 1000)
    e2e_value = e2e_tok_step * world / (e2e_ms / 1000)
    F8 = wgemm.F8_DENSE
    MOE_DESC = wgemm.moe_decode_desc()
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": Wm, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": round(value / BASELINE_TOKS, 3),
            "dtype": ("e4m3 activations per (token, 128-column group) x e4m3 weights (dense)" if F8 else
                      "fp16 activations x fp8 weights (dense)") + "; int8 activations per 128-column group x "
                     "4/3-bit weights (decode MoE); fp32 accumulation; LM head fp16 activations x fp8 weights",
            "data": "synthetic (random-init weights N(0,0.02); random cache state for 6k-12k-token contexts)",
            "config": {"model": f"flashnext-shaped {cfg.num_layers}L h{cfg.hidden_size} {cfg.n_experts}/"
                                 f"{cfg.n_experts_orig} experts top-{cfg.top_k} 4/3-bit g128 + FP8 128x128 dense",
                       "global_batch": total_batch, "seq_len": f"{args.ctx_min}-{args.ctx_max} context",
                       "parallelism": (f"dp{world} attention + ep{world} experts ({args.comm} exchange)" if use_ep
                                       else f"dp{world}"),
                       "kv_cache": "fp8 paged, block 64",
                       "l2": "inputs larger than L2 (weights streamed per step >> 126 MB)",
                       "ple": f"layers {list(cfg.ple_layers)}, {cfg.ple_rows // 10**6}M x {cfg.ple_dim} fp8 n-gram table",
                       "mtp": "off (no speculative decoding in this measurement)",
                       "compute": (("dense projections: tcgen05 kind::f8f6f4 (e4m3 x e4m3, per-group scales in "
                                    "the epilogue)" if F8 else "dense projections: fp16 tcgen05 MMA") +
                                   ", fp32 accumulate; decode MoE experts: " + MOE_DESC),
                       "valid": not args.layers},
            "p50_tpot_ms": round(p50, 3),
            "clocks": clk,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": (3 * 4 + 28) * args.batch, "d2h_bytes_per_step": 8 * args.batch},
            "gpu_launches": launches * K,
            "gpu_launches_per_step": launches,
            "weights_gb": {k: round(v / 1e9, 2) for k, v in nbytes.items()},
            "build_s": round(t_w, 1),
        }
        print(json.dumps(out))
        sys.stdout.flush()
    if world > 1:
        llm.graphs.clear()
        del llm
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

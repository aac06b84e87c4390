"""Tensor-parallel decode microbenchmark for the Dots3-shaped model.

Runs one decode step of a D3 slice (the full model's hidden size, head counts, latent ranks and expert shapes;
fewer layers, experts and vocabulary so it builds in seconds) at TP = WORLD_SIZE, with the all-reduces either
fused into the producing kernels over NVLink peer memory (``--comm fused``: wgemm fan-out epilogue + signal +
reduce, csrc/k_tp.cu) or done by NCCL (``--comm nccl``). The step is captured in a CUDA graph; the device time of
K replays is taken with CUDA events and the max over ranks is printed as one JSON line. ``--primitive`` times the
bare ``h += all_reduce(partial)`` for a [T, hidden] fp32 partial instead (10 per captured graph).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29700 \\
        -m arcagi2_flashnext_dots3_b200.launch.tp_bench --comm fused
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from ..config import d3_config
from ..engine.block_manager import BlockAllocator
from ..models.d3 import D3Model, allocate_caches
from ..models.d3_weights import random_dense, to_engine
from ..ops import native
from ..parallel.tp import TPGroup, shard_d3_weights, tp_config


def _time(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / steps], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl", "q8", "q4"])
    ap.add_argument("--layers", type=int, default=3)
    ap.add_argument("--experts", type=int, default=16)
    ap.add_argument("--vocab", type=int, default=32768)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--primitive", action="store_true")
    ap.add_argument("--eager", action="store_true", help="no CUDA graph (for launch lists)")
    args = ap.parse_args()
    for k, v in (("RANK", "0"), ("WORLD_SIZE", "1"), ("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29799")):
        os.environ.setdefault(k, v)   # a plain `python -m` run is a 1-rank group
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    cfg = d3_config(num_layers=args.layers, n_dsa_layers=min(2, args.layers), n_experts=args.experts,
                    n_experts_orig=args.experts, vocab_size=args.vocab)
    tp = TPGroup(rank, world, dev, max_tokens=max(64, args.batch), hidden=cfg.hidden_size, comm=args.comm)
    out = {"bench": "tp_decode" if not args.primitive else "tp_allreduce", "comm": args.comm, "tp": world,
           "model": f"{cfg.name} slice: {args.layers} layers, {args.experts} experts, vocab {args.vocab}"}
    if args.primitive:
        rows = []
        h = torch.zeros(64, cfg.hidden_size, device=dev)
        for T in (1, 8, 32, 64):
            part = torch.randn(T, cfg.hidden_size, device=dev)
            hv = h[:T]
            for _ in range(3):
                tp.allreduce_add(hv, part)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(10):
                    tp.allreduce_add(hv, part)
            ms = _time(g.replay, args.steps, args.warmup) / 10
            del g
            rows.append({"rows": T, "us": round(ms * 1e3, 2)})
        out["sizes"] = rows
    else:
        W = random_dense(cfg, seed=0)
        lc = tp_config(cfg, world)
        B = args.batch
        total = args.ctx + args.warmup + args.steps + 8
        caches = allocate_caches(lc, dev, B, total, block_size=64)
        m = D3Model(lc, to_engine(shard_d3_weights(W, cfg, rank, world), lc, dev), caches, dev, tp=tp)
        del W
        alloc = BlockAllocator(caches.n_blocks, B)
        for s in range(B):
            m.assign_blocks(s, total, alloc)
        m.randomize_caches(torch.Generator(device=dev).manual_seed(1))
        ids = torch.randint(0, cfg.vocab_size, (B,), device=dev, dtype=torch.int32)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        pos = torch.full((B,), args.ctx, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        dist.barrier()   # ranks finish building at different times; the fused all-reduce waits are bounded
        if args.eager:
            ms = _time(lambda: m.pick(m.step(ids, slots, pos, 1)), args.steps, args.warmup)
            native.check_error(dev)
            out.update({"batch": B, "ctx": args.ctx, "ms_per_step": round(ms, 4), "graph": False})
            if rank == 0:
                print(json.dumps(out), flush=True)
            dist.barrier()
            dist.destroy_process_group()
            return
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                m.pick(m.step(ids, slots, pos, 1))
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            lg = m.pick(m.step(ids, slots, pos, 1))
        ms = _time(g.replay, args.steps, args.warmup)
        native.check_error(dev)
        out.update({"batch": B, "ctx": args.ctx, "ms_per_step": round(ms, 4)})
        del g, lg
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

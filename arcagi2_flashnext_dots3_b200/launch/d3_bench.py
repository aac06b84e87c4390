"""Decode throughput of the Dots3-Note-shaped model at its full dimensions (BASELINE config 3 shape).

Random engine weights are generated on the GPU (:func:`..models.d3_weights.random_engine`: block-FP8 dense
weights, 3/2-bit experts). Every session's latent and indexer caches are filled with random rows up to the
context length, as after prefill. Then greedy decode steps run, each one CUDA graph of embed -> 46 layers ->
lm_head -> argmax -> position advance. The metric is generated tokens/s = batch / device time per step (CUDA
events, max over ranks). With torchrun, the ranks run tensor parallel (heads and experts split,
o-projection and MoE all-reduces fused over NVLink, ``--comm nccl`` for the NCCL baseline).

    python -m arcagi2_flashnext_dots3_b200.launch.d3_bench --batch 32 --ctx 32768
    python -m torch.distributed.run --nproc-per-node 4 --master-addr 127.0.0.1 --master-port 29701 \\
        -m arcagi2_flashnext_dots3_b200.launch.d3_bench --batch 32 --ctx 32768
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from ..config import d3_config
from ..engine.block_manager import BlockAllocator
from ..models.d3 import D3Model, allocate_caches
from ..models.d3_weights import random_engine
from ..ops import fn_ops as ops
from ..ops import native


def _max_ms(ms: float, dev) -> float:
    """Device time of this rank -> the maximum over the ranks."""
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=0, help="0: the config's 46")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl", "q8", "q4"])
    ap.add_argument("--eager", action="store_true", help="no CUDA graph (for launch lists)")
    ap.add_argument("--sp", action="store_true",
                    help="sequence parallel: residual rows split over the TP ranks, NCCL reduce-scatter / all-gather")
    ap.add_argument("--turn2", type=int, default=0,
                    help="second turn: every session appends this many new prompt tokens (one prefill step per "
                         "session on the kept cache), then decodes --steps more tokens")
    ap.add_argument("--shard-vocab", action="store_true",
                    help="with TP: each rank holds its slice of the LM head; tokens via the sharded pick")
    args = ap.parse_args()
    for k, v in (("RANK", "0"), ("WORLD_SIZE", "1"), ("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29798")):
        os.environ.setdefault(k, v)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    kw = {"num_layers": args.layers} if args.layers else {}
    cfg = d3_config(**kw)
    t0 = time.time()
    tp = None
    lc = cfg
    if world > 1:
        from ..parallel.tp import TPGroup, tp_config
        lc = tp_config(cfg, world)
        tp = TPGroup(rank, world, dev, max_tokens=max(64, args.batch, args.turn2), hidden=cfg.hidden_size,
                     comm="nccl" if args.sp else args.comm, sequence_parallel=args.sp)
    W = random_engine(cfg, dev, seed=0, tp=(rank, world) if world > 1 else None,
                      shard_vocab=args.shard_vocab and world > 1)
    B = args.batch
    total = args.ctx + args.warmup + args.steps * (2 if args.turn2 else 1) + args.turn2 + 16
    caches = allocate_caches(lc, dev, B, total, block_size=64)
    m = D3Model(lc, W, caches, dev, tp=tp)
    alloc = BlockAllocator(caches.n_blocks, B)
    for s in range(B):
        m.assign_blocks(s, total, alloc)
    m.randomize_caches(torch.Generator(device=dev).manual_seed(1))
    build_s = time.time() - t0
    ids = torch.randint(0, cfg.vocab_size, (B,), device=dev, dtype=torch.int32)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    pos = torch.full((B,), args.ctx, dtype=torch.int32, device=dev)

    def step():
        x = m.step(ids, slots, pos, 1)
        ids.copy_(m.pick(x))
        pos.add_(1)

    torch.cuda.synchronize()
    dist.barrier()   # ranks finish building at different times; the fused all-reduce waits are bounded
    run = step
    g = None
    if not args.eager:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        run = g.replay
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        run()
    b.record()
    torch.cuda.synchronize()
    native.check_error(dev)
    ms = _max_ms(a.elapsed_time(b) / args.steps, dev)
    extra = {}
    if args.turn2:
        # turn 2 of every session: the new user message is prefilled onto the kept cache (one step of turn2 tokens
        # per session, eager), its last row picks the first reply token, then the batch decodes again
        new = torch.randint(0, cfg.vocab_size, (B, args.turn2), device=dev, dtype=torch.int32,
                            generator=torch.Generator(device=dev).manual_seed(2))
        torch.cuda.synchronize()
        dist.barrier()
        a.record()
        for s in range(B):
            x = m.step(new[s], slots[s:s + 1], pos[s:s + 1], args.turn2)
            ids[s:s + 1].copy_(m.pick(x[-1:]))
        b.record()
        pos.add_(args.turn2)
        torch.cuda.synchronize()
        native.check_error(dev)
        pre_ms = _max_ms(a.elapsed_time(b), dev)
        dist.barrier()
        a.record()
        for _ in range(args.steps):
            run()
        b.record()
        torch.cuda.synchronize()
        native.check_error(dev)
        ms2 = _max_ms(a.elapsed_time(b) / args.steps, dev)
        extra = {"turn2_tokens": args.turn2, "turn2_prefill_ms": round(pre_ms, 2),
                 "turn2_prefill_tok_per_s": round(B * args.turn2 / pre_ms * 1e3, 1),
                 "turn2_ctx": args.ctx + args.warmup + args.steps + args.turn2,
                 "turn2_ms_per_step": round(ms2, 3), "turn2_tok_per_s": round(B / ms2 * 1e3, 1)}
    if rank == 0:
        print(json.dumps({"bench": "d3_decode", "model": cfg.name, "layers": cfg.num_layers,
                          "experts": cfg.n_experts, "tp": world,
                          "comm": ("nccl" if args.sp else args.comm) if world > 1 else None,
                          "sp": bool(args.sp and world > 1),
                          "batch": B, "ctx": args.ctx, "ms_per_step": round(ms, 3),
                          "tok_per_s": round(B / ms * 1e3, 1), "graph": g is not None, **extra,
                          "build_s": round(build_s, 1),
                          "mem_GB": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1)}), flush=True)
    # the graph may hold NCCL calls (--comm nccl): every reference to it, the bound replay method included, must
    # be gone before destroy_process_group, or the process waits at exit
    run = None
    del g
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""End-to-end serving benchmark: prefill of long prompts plus generation through the continuous-batching
scheduler, the way a solver drives the engine (prompts of 6k-12k tokens drawn uniformly from a
40-token grid/digit vocabulary subset, greedy, paged KV).

Every request is submitted at t=0; the scheduler admits what fits, interleaves chunked prefill with CUDA-graph
decode, and runs until all requests finish. Reported (device-synchronized wall clock of the whole run, since the run
mixes host scheduling, prefill and decode):
  generated tok/s over the run, prefill tok/s (prompt tokens / time spent in prefill calls), mean time to first
  token, mean time per output token after the first, scheduler counters.

    python -m arcagi2_flashnext_dots3_b200.launch.serve_bench [--seqs 64] [--gen 256] [--ctx-min 6144]
        [--ctx-max 12288] [--layers 0] [--model fn|d3]
"""
from __future__ import annotations

import argparse
import json
import time

import torch


def synthetic_prompts(n: int, lo: int, hi: int, vocab: int, subset: int = 40, seed: int = 0) -> list:
    """n prompts of uniform length in [lo, hi], tokens uniform over a fixed `subset`-token slice of the vocab."""
    g = torch.Generator().manual_seed(seed)
    toks = torch.randperm(vocab, generator=g)[:subset]
    lens = torch.randint(lo, hi + 1, (n,), generator=g).tolist()
    return [toks[torch.randint(0, subset, (L,), generator=g)].tolist() for L in lens]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="fn", choices=["fn", "d3"])
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--ctx-min", type=int, default=6144)
    ap.add_argument("--ctx-max", type=int, default=12288)
    ap.add_argument("--layers", type=int, default=0, help="fewer layers (a smaller model; marked in the output)")
    ap.add_argument("--prefill-budget", type=int, default=8192)
    ap.add_argument("--chunk", type=int, default=4096)
    a = ap.parse_args(argv)
    from ..config import EngineConfig, d3_config, fn_config
    from ..engine.llm import LLM
    from ..engine.scheduler import Scheduler
    from ..ops import native
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    kw = {"num_layers": a.layers} if a.layers else {}
    if a.model == "fn":
        from ..models.fn_weights import random_engine
        cfg = fn_config(**kw)
        W = random_engine(cfg, dev, seed=1)
        model_cls = None
    else:
        from ..models.d3 import D3Model
        from ..models.d3_weights import random_engine
        cfg = d3_config(**kw)
        W = random_engine(cfg, dev, seed=1)
        model_cls = D3Model
    max_len = a.ctx_max + a.gen + 64
    ec = EngineConfig(max_seqs=a.seqs, max_model_len=max_len, block_size=64, kv_dtype="fp8",
                      graph_batch_sizes=tuple(b for b in (1, 2, 4, 8, 16, 32, 64, 128) if b <= a.seqs) or (a.seqs,))
    llm = LLM(cfg, W, dev, ec, model_cls=model_cls)
    prompts = synthetic_prompts(a.seqs, a.ctx_min, a.ctx_max, cfg.vocab_size)
    sch = Scheduler(llm, prefill_budget=a.prefill_budget, chunk=a.chunk)
    # warm-up: capture the decode graphs of every bucket on a short request set (not timed)
    warm = Scheduler(llm, prefill_budget=a.prefill_budget, chunk=a.chunk)
    warm.generate([p[:64] for p in prompts[:min(a.seqs, 4)]], max_new_tokens=4)
    for b in ec.graph_batch_sizes:
        llm._graph_for(b)
    torch.cuda.synchronize()
    t_prefill = 0.0
    orig = sch._prefill

    def timed_prefill():
        nonlocal t_prefill
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        orig()
        torch.cuda.synchronize()
        t_prefill += time.perf_counter() - t0
    sch._prefill = timed_prefill
    t0 = time.perf_counter()
    reqs = [sch.submit(p, a.gen) for p in prompts]
    sch.run(reqs)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    native.check_error(dev)
    gen = sum(len(r.out) for r in reqs)
    ttft = sum(r.t_first - r.t_submit for r in reqs) / len(reqs)
    tpot = sum((r.t_done - r.t_first) / max(1, len(r.out) - 1) for r in reqs) / len(reqs)
    st = vars(sch.stats)
    out = {"metric": "generated tok/s over a run with prefill (scheduler, 1 GPU)", "model": a.model,
           "layers": cfg.num_layers, "full_model": not a.layers, "seqs": a.seqs, "gen_per_seq": a.gen,
           "prompt_tokens": sum(map(len, prompts)), "generated": gen, "run_s": round(t1 - t0, 2),
           "generated_tok_s": round(gen / (t1 - t0), 1),
           "prefill_tok_s": round(st["prefill_tokens"] / max(t_prefill, 1e-9), 1),
           "prefill_s": round(t_prefill, 2), "ttft_s_mean": round(ttft, 2), "tpot_ms_mean": round(tpot * 1e3, 2),
           "scheduler": st}
    print(json.dumps(out), flush=True)
    return out


if __name__ == "__main__":
    main()

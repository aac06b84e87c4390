"""Speculative-decoding benchmark: acceptance and generated tokens/s per drafter at several batch sizes.

    python -m arcagi2_flashnext_dots3_b200.launch.spec_bench [--small] [--batches 1,16,64] [--k 3] [--steps 16]

Random-init weights and random cache state for 6k-12k-token contexts (as in bench.py). With random weights the
MTP head's drafts are uncorrelated with the model, so its acceptance is a floor; prompt lookup (n-gram) accepts
whenever the random model repeats itself. The plain (k = 0) row is the same engine without drafts through the same (graph-captured) verify path.
``oracle@P`` drafts the model's own greedy continuation with each token kept with probability P, which measures
the cost/benefit curve at controlled acceptance. One JSON line per (drafter, batch).
"""
from __future__ import annotations

import argparse
import json
import time

import torch


class ControlledDrafter:
    """Drafts the model's own recorded greedy continuation (``ref[slot]``, from a plain decode of the same
    synthetic context), each draft token kept with probability p and otherwise replaced by a wrong token, so the
    acceptance rate is controlled: the cost/benefit curve of speculative decoding with random weights."""

    def __init__(self, ref: dict, p: float, vocab: int, seed: int = 0):
        self.ref, self.p, self.vocab = ref, p, vocab
        self.g = torch.Generator().manual_seed(seed)

    def propose(self, llm, seqs, k):
        out = []
        for s in seqs:
            n = len(s.out) - 1          # ref[0] follows the context's first pending token, out[0]
            want = (self.ref[s.slot][n:n + k] + [0] * k)[:k]
            keep = torch.rand(k, generator=self.g) < self.p
            out.append([w if kp else (w + 1) % self.vocab for w, kp in zip(want, keep.tolist())])
        return out

    def observe(self, llm, seqs, x, ids, accepted, k):
        pass


def _reference_outputs(cfg, W, dev, ec, lengths, n_new):
    """Greedy continuations of the synthetic contexts by plain graph decoding (same seed as the spec run)."""
    from ..engine.llm import LLM
    llm = LLM(cfg, W, dev, ec)
    seqs = llm.synthesize_context(lengths, n_new + 8)
    while min(len(s.out) for s in seqs) < n_new + 1:
        llm.step()
    ref = {s.slot: list(s.out[1:]) for s in seqs}
    del llm
    torch.cuda.empty_cache()
    return ref


def run(args):
    from ..config import EngineConfig, fn_config, fn_small_config
    from ..engine.llm import LLM
    from ..engine.spec import MTPDrafter, NgramDrafter, SpecDecoder
    from ..models import fn_weights
    from ..models.fn_mtp import MTPHead, random_mtp
    dev = torch.device("cuda")
    cfg = fn_small_config() if args.small else fn_config()
    W = (fn_weights.to_engine(fn_weights.random_dense(cfg, seed=1, symmetric=False), cfg, dev) if args.small
         else fn_weights.random_engine(cfg, dev, seed=1234))
    max_b = max(args.batches)
    steps = args.steps
    max_len = args.ctx_max + (args.k + 1) * (steps + 4) + 64
    ec = EngineConfig(max_seqs=max_b, max_model_len=max_len, block_size=64, graph_batch_sizes=(1,))
    mtp_w = random_mtp(cfg, dev) if "mtp" in args.drafters else None
    for drafter in args.drafters:
        for B in args.batches:
            llm = LLM(cfg, W, dev, ec)
            g = torch.Generator().manual_seed(7)
            lengths = torch.randint(args.ctx_min, args.ctx_max + 1, (B,), generator=g).tolist()
            seqs = llm.synthesize_context(lengths, (args.k + 1) * (steps + 4))
            if drafter == "none":
                sd = SpecDecoder(llm, NgramDrafter(), k=0)
            elif drafter == "ngram":
                sd = SpecDecoder(llm, NgramDrafter(), k=args.k)
            elif drafter.startswith("oracle@"):
                del llm
                torch.cuda.empty_cache()
                ref = _reference_outputs(cfg, W, dev, ec, lengths, (args.k + 1) * (steps + 3))
                llm = LLM(cfg, W, dev, ec)
                seqs = llm.synthesize_context(lengths, (args.k + 1) * (steps + 4))
                sd = SpecDecoder(llm, ControlledDrafter(ref, float(drafter.split("@")[1]), cfg.vocab_size), k=args.k)
            else:
                head = MTPHead(cfg, W, mtp_w, dev, max_b + 1, max_len, block_size=64)
                d = MTPDrafter(head)
                for s in seqs:
                    head.assign_blocks(s.slot, max_len - 8, d.alloc)
                sd = SpecDecoder(llm, d, k=args.k)
            for _ in range(2):  # warm-up
                sd.step()
            torch.cuda.synchronize()
            st0 = dict(sd.stats)
            t0 = time.perf_counter()
            for _ in range(steps):
                sd.step()
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            emitted = sd.stats["emitted"] - st0["emitted"]
            n_seq_steps = B * steps
            print(json.dumps({"drafter": drafter, "batch": B, "k": 0 if drafter == "none" else args.k,
                              "tokens_per_seq_step": round(emitted / n_seq_steps, 3),
                              "tok_s": round(emitted / dt, 1), "ms_per_step": round(1000 * dt / steps, 2),
                              "model": cfg.name, "weights": "random"}), flush=True)
            del llm, sd
            torch.cuda.empty_cache()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--small", action="store_true")
    ap.add_argument("--batches", default="1,16,64")
    ap.add_argument("--drafters", default="none,ngram,mtp",
                    help="none, ngram, mtp and oracle@P (recorded greedy continuation, each token kept with prob P)")
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--ctx-min", type=int, default=6144)
    ap.add_argument("--ctx-max", type=int, default=12288)
    a = ap.parse_args(argv)
    a.batches = [int(x) for x in a.batches.split(",")]
    a.drafters = a.drafters.split(",")
    run(a)


if __name__ == "__main__":
    main()

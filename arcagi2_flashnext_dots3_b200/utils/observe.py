"""Observability: region tracing (CUDA events or wall clock, Chrome-trace export), MoE routing statistics and
a memory census.

Counterparts of the reference's CUDA-event timing around its attention kernels
(dotsnote/engine/arcstats_pkg/arcstats/offload_cuda2.py:143-170), route-statistics ring buffers
(flashnext/kaggle/code_dataset/fnext/moe/fnmoe.py:29-124 `_RouteStats`), its expert placement by routed load
(`FN_EP_PLACE`, fnmoe.py:18-27) and its memory census / phase logging (arcstats/__init__.py:607-977).
"""
from __future__ import annotations

import json
import time
from collections import defaultdict
from contextlib import contextmanager

import torch


class Tracer:
    """``with tracer.region("name"):`` records the region's duration (device time between CUDA events on the
    current stream, or wall time on CPU). Nothing is synchronized until :meth:`summary` / :meth:`chrome`."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self.events = []          # (name, start_event_or_t, end_event_or_t, cuda, wall_start)

    @contextmanager
    def region(self, name: str, device=None):
        if not self.enabled:
            yield
            return
        cuda = torch.cuda.is_available() and (device is None or torch.device(device).type == "cuda")
        w0 = time.perf_counter()
        if cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            yield
            b.record()
            self.events.append((name, a, b, True, w0))
        else:
            yield
            self.events.append((name, w0, time.perf_counter(), False, w0))

    def _durations(self):
        if any(e[3] for e in self.events):
            torch.cuda.synchronize()
        out = []
        for name, a, b, cuda, w0 in self.events:
            ms = a.elapsed_time(b) if cuda else (b - a) * 1000
            out.append((name, w0, ms))
        return out

    def summary(self) -> dict:
        agg = defaultdict(lambda: [0, 0.0])
        for name, _, ms in self._durations():
            agg[name][0] += 1
            agg[name][1] += ms
        return {k: {"count": n, "total_ms": round(t, 4), "avg_ms": round(t / n, 4)} for k, (n, t) in agg.items()}

    def chrome(self, path: str):
        """Chrome trace (chrome://tracing, Perfetto): one complete event per region, start = host time."""
        d = self._durations()
        t0 = min((w for _, w, _ in d), default=0.0)
        ev = [{"name": n, "ph": "X", "ts": (w - t0) * 1e6, "dur": ms * 1000, "pid": 0, "tid": 0} for n, w, ms in d]
        with open(path, "w") as fh:
            json.dump({"traceEvents": ev}, fh)


class RouteStats:
    """Per-layer expert hit counts accumulated on the device (one bincount per MoE call), with a window of recent
    steps for load-aware decisions."""

    def __init__(self, n_layers: int, n_experts: int, device, window: int = 64):
        self.counts = torch.zeros(n_layers, n_experts, dtype=torch.int64, device=device)
        self.window = window
        self.recent = []
        self.steps = 0

    def add(self, layer: int, ids: torch.Tensor):
        self.counts[layer] += torch.bincount(ids.reshape(-1).long(), minlength=self.counts.shape[1])

    def end_step(self):
        self.steps += 1
        self.recent.append(self.counts.clone())
        if len(self.recent) > self.window:
            self.recent.pop(0)

    def load(self) -> torch.Tensor:
        """Counts over the recent window (all steps if no step has ended)."""
        if len(self.recent) >= 2:
            return self.recent[-1] - self.recent[0]
        return self.counts

    def imbalance(self, world: int) -> float:
        """max / mean routed rows per rank under the contiguous expert split."""
        per = self.load().sum(0).view(world, -1).sum(1).double()
        return float(per.max() / per.mean().clamp_min(1))

    def to_json(self) -> dict:
        return {"steps": self.steps, "counts": self.counts.cpu().tolist()}


def place_experts(load: torch.Tensor, world: int) -> list:
    """Expert -> rank assignment balancing total load (greedy longest-processing-time over experts sorted by
    load; every rank gets exactly E / world experts). `load` [E]."""
    E = load.numel()
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    cap = E // world
    order = torch.argsort(load.double(), descending=True).tolist()
    tot = [0.0] * world
    n = [0] * world
    owner = [0] * E
    for e in order:
        r = min((r for r in range(world) if n[r] < cap), key=lambda r: tot[r])
        owner[e] = r
        tot[r] += float(load[e])
        n[r] += 1
    return owner


def memory_census(weights: dict = None, caches=None, device=None) -> dict:
    """Bytes by category: weights (per top-level key), caches (per field), and the allocator's counters."""
    def nbytes(x):
        if isinstance(x, torch.Tensor):
            return x.numel() * x.element_size()
        if hasattr(x, "blob"):
            return x.blob.numel()
        if isinstance(x, dict):
            return sum(nbytes(v) for v in x.values())
        if isinstance(x, (list, tuple)):
            return sum(nbytes(v) for v in x)
        return 0
    out = {}
    if weights is not None:
        out["weights"] = {k: nbytes(v) for k, v in weights.items()}
    if caches is not None:
        out["caches"] = {k: nbytes(v) for k, v in vars(caches).items() if nbytes(v)}
    if torch.cuda.is_available():
        dev = torch.device(device or "cuda")
        s = torch.cuda.memory_stats(dev)
        free, total = torch.cuda.mem_get_info(dev)
        out["allocator"] = {"allocated": s.get("allocated_bytes.all.current", 0),
                            "reserved": s.get("reserved_bytes.all.current", 0),
                            "peak_allocated": s.get("allocated_bytes.all.peak", 0), "free": free, "total": total}
    return out


class TopkOverlap:
    """Top-k agreement between DSA layers (the statistic behind an index-sharing pattern; the reference's
    index_share.py TopkOverlap). For every pair of DSA layers (a, b) and every query row with a sparse selection,
    |topk_a & topk_b| / k is accumulated into bins of the number of visible keys. ``add`` collects one layer's
    selection during a step, ``end_step`` scores the pairs and clears the step; ``table`` / ``save`` report means."""
    BINS = (0, 2048, 4096, 8192, 16384, 32768, 1 << 30)

    def __init__(self):
        self._step = {}
        self.sum = {}
        self.cnt = {}

    def add(self, layer: int, sel: torch.Tensor, positions: torch.Tensor, n_tok: int):
        pos = positions.long().repeat_interleave(n_tok) + torch.arange(n_tok, device=positions.device).repeat(
            positions.shape[0])
        self._step[layer] = (sel.detach().clone(), pos + 1)

    def end_step(self):
        layers = sorted(self._step)
        nb = len(self.BINS) - 1
        for i, a in enumerate(layers):
            sa, vis = self._step[a]
            T, k = sa.shape
            ok = sa[:, 0] >= 0
            if not bool(ok.any()):
                continue
            L = int(vis.max())
            mark = torch.zeros(T, L + 1, dtype=torch.bool, device=sa.device)
            mark.scatter_(1, sa.long().clamp(0, L), True)
            bins = torch.bucketize(vis, torch.tensor(self.BINS[1:-1], device=vis.device), right=True)
            for b in layers[i + 1:]:
                sb = self._step[b][0]
                hit = (mark.gather(1, sb.long().clamp(0, L)) & (sb >= 0)).sum(1).float() / k
                valid = ok & (sb[:, 0] >= 0)
                s = torch.zeros(nb, device=sa.device).index_add_(0, bins[valid], hit[valid])
                n = torch.zeros(nb, device=sa.device).index_add_(0, bins[valid], torch.ones_like(hit[valid]))
                key = (a, b)
                self.sum[key] = self.sum.get(key, 0) + s.cpu()
                self.cnt[key] = self.cnt.get(key, 0) + n.cpu()
        self._step = {}

    def table(self) -> dict:
        """{(layer_a, layer_b): [mean overlap per context bin, nan where empty]}."""
        return {k: (self.sum[k] / self.cnt[k]).tolist() for k in self.sum}

    def save(self, path: str):
        import numpy as np
        keys = sorted(self.sum)
        np.savez(path, pairs=np.array(keys, dtype=np.int64), bins=np.array(self.BINS, dtype=np.int64),
                 sum=np.stack([self.sum[k].numpy() for k in keys]) if keys else np.zeros((0, 6)),
                 cnt=np.stack([self.cnt[k].numpy() for k in keys]) if keys else np.zeros((0, 6)))


# ------------------------------------------------------------------------------------------ runtime flags
RUNTIME_FLAGS = {
    "FW_MOE_GEMV": ("1", "decode MoE on the int8 grouped GEMV (0: tcgen05 grouped GEMM)"),
    "FW_MOE_GEMV_PAIRS": ("4", "largest mean (token, expert) pairs per expert served by the GEMV"),
    "FW_EP_GEMV_PAIRS": ("8", "same crossover under expert parallelism"),
    "FW_SIDE_STREAM": ("1", "shared expert on a side stream concurrent with the routed experts"),
    "FW_DENSE_PLAN": ("", "'old': dense GEMMs without the token-tile/split-K launch plan"),
    "FW_MLA_CUDA_CORE": ("0", "D3 latent attention on the CUDA-core kernel instead of tcgen05"),
    "FW_MLA_SPLITS": ("0", "fixed key-split count of the latent attention (0: automatic)"),
    "FW_DSA_CUDA_CORE": ("0", "DSA indexer scores on the CUDA-core kernel instead of tcgen05"),
    "FW_D3_ABSORB": ("bmm", "D3 per-head absorption: batched GEMM or 'grouped' tcgen05"),
    "FW_WAIT_TIMEOUT_MS": ("", "bound of every in-kernel wait before it reports an error"),
    "FW_STEPLOG": ("", "path of the binary per-step engine log"),
}


def flag_report(env=None) -> list:
    """Every runtime switch with its effective value, whether it differs from the default, and what it does; the
    engine logs this at start-up so a run records which optional paths were active."""
    import os
    env = os.environ if env is None else env
    out = []
    for name, (default, what) in RUNTIME_FLAGS.items():
        val = env.get(name, default)
        out.append({"flag": name, "value": val, "changed": name in env and env[name] != default, "what": what})
    return out


def reclaim(llm=None, keep_graphs: bool = True) -> dict:
    """Give memory back: drop dense-copy caches of weight sets (test/oracle views), optionally the captured decode
    graphs (their private pools), then release the caching allocator's free blocks. Returns bytes freed per kind
    (the reference's mem_reclaim.py frees vLLM's unused workspaces the same way after start-up)."""
    import gc
    import torch
    freed = {"dense_caches": 0, "graphs": 0, "allocator": 0}
    if llm is not None:
        def walk(x):
            if hasattr(x, "_dense_cache") and x._dense_cache:
                freed["dense_caches"] += sum(t.numel() * t.element_size() for t in x._dense_cache.values())
                x._dense_cache = None
            elif isinstance(x, dict):
                for v in x.values():
                    walk(v)
            elif isinstance(x, (list, tuple)):
                for v in x:
                    walk(v)
        walk(llm.model.W)
        if not keep_graphs and getattr(llm, "graphs", None):
            freed["graphs"] = len(llm.graphs)
            llm.graphs.clear()
    gc.collect()
    if torch.cuda.is_available():
        before = torch.cuda.memory_reserved()
        torch.cuda.empty_cache()
        freed["allocator"] = before - torch.cuda.memory_reserved()
    return freed

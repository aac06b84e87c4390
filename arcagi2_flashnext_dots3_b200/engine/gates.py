"""Start-up gates: each optional fast path is checked against its baseline on probe inputs on the machine that
will serve, and enabled only where it is accurate enough and faster.

The reference decides its optional kernels this way at boot (dotsnote/kaggle/runtime_dataset/run_l4.py:994-1509:
NCCL candidates scored per decode step, the host-staged all-reduce enabled for the contiguous range of message
sizes where it beats NCCL with err < 0.02, tile tuning); the rule is "exact (or within the error bound) and
faster, else keep the baseline". Here:

* :class:`Gates` runs registered gates: both paths on the same inputs, the candidate's max relative error
  against the baseline's output (``tol`` 0 means bit-exact), device time of each (CUDA events on the current
  stream after warm-up, or wall time on the CPU), then the gate's ``switch(True/False)``; one JSON line per gate
  to ``log_path``.
* sized gates evaluate a list of sizes and enable the candidate on the contiguous run of winning sizes with the
  largest total time saved (a loss or tie at one size does not disable it for a disjoint larger range).
* :func:`engine_gates` registers this framework's optional GPU paths (decode MoE on the int8 GEMV vs the
  tcgen05 grouped GEMM; tcgen05 latent attention and DSA indexer vs their CUDA-core kernels).
"""
from __future__ import annotations

import json
import statistics
import time
from dataclasses import dataclass, field


@dataclass
class GateResult:
    name: str
    enabled: bool
    err: float
    base_us: float
    cand_us: float
    size: object = None
    note: str = ""

    @property
    def speedup(self) -> float:
        return self.base_us / self.cand_us if self.cand_us > 0 else float("inf")


def max_rel_err(a, b) -> float:
    import torch
    a, b = a.float(), b.float()
    if a.shape != b.shape:
        return float("inf")
    scale = b.abs().max().clamp_min(1e-30)
    return float((a - b).abs().max() / scale)


def device_time_us(fn, reps: int = 10, warmup: int = 3) -> float:
    """Median time of fn() in microseconds: CUDA events when a GPU is present, wall clock otherwise."""
    import torch
    for _ in range(warmup):
        fn()
    ts = []
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
    else:
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append((time.perf_counter() - t0) * 1e6)
    return statistics.median(ts)


@dataclass
class _Gate:
    name: str
    baseline: object
    candidate: object
    switch: object
    tol: float
    sizes: list = None
    margin: float = 0.95


@dataclass
class Gates:
    log_path: str = None
    reps: int = 10
    timer: object = None                   # fn -> microseconds (tests inject a fake clock)
    gates: list = field(default_factory=list)
    results: list = field(default_factory=list)

    def add(self, name, baseline, candidate, switch, tol: float = 0.0, margin: float = 0.95):
        """baseline() / candidate() compute the same output; switch(bool) turns the candidate path on or off."""
        self.gates.append(_Gate(name, baseline, candidate, switch, tol, None, margin))

    def add_sized(self, name, sizes, baseline, candidate, switch, tol: float = 0.0, margin: float = 0.95):
        """baseline(size) / candidate(size); switch((lo, hi) or None) enables the candidate for sizes in [lo, hi]."""
        self.gates.append(_Gate(name, baseline, candidate, switch, tol, list(sizes), margin))

    def _measure(self, g, base, cand, size=None) -> GateResult:
        timer = self.timer or (lambda fn: device_time_us(fn, self.reps))
        try:
            err = max_rel_err(cand(), base())
        except Exception as e:   # a candidate that fails to run is never enabled
            return GateResult(g.name, False, float("inf"), 0.0, 0.0, size, f"candidate failed: {e!r}"[:200])
        tb, tc = timer(base), timer(cand)
        ok = err <= g.tol and tc < g.margin * tb
        return GateResult(g.name, ok, err, tb, tc, size)

    def run(self) -> list:
        for g in self.gates:
            if g.sizes is None:
                r = self._measure(g, g.baseline, g.candidate)
                g.switch(r.enabled)
                self._log(r)
                continue
            rows = [self._measure(g, (lambda s=s: g.baseline(s)), (lambda s=s: g.candidate(s)), s) for s in g.sizes]
            best, best_gain, start = None, 0.0, None
            for i, r in enumerate(rows + [None]):
                if r is not None and r.enabled and start is None:
                    start = i
                elif (r is None or not r.enabled) and start is not None:
                    gain = sum(rows[j].base_us - rows[j].cand_us for j in range(start, i))
                    if gain > best_gain:
                        best, best_gain = (start, i - 1), gain
                    start = None
            rng = (g.sizes[best[0]], g.sizes[best[1]]) if best else None
            g.switch(rng)
            for i, r in enumerate(rows):
                r.enabled = best is not None and best[0] <= i <= best[1]
                r.note = f"range {rng}"
                self._log(r)
        return self.results

    def _log(self, r: GateResult):
        self.results.append(r)
        if self.log_path:
            with open(self.log_path, "a") as f:
                f.write(json.dumps({"gate": r.name, "size": r.size, "enabled": r.enabled, "err": r.err,
                                    "base_us": round(r.base_us, 2), "cand_us": round(r.cand_us, 2),
                                    "speedup": round(r.speedup, 3), "note": r.note}) + "\n")


def engine_gates(device, log_path: str = None, reps: int = 10) -> Gates:
    """This framework's optional GPU paths, on decode-shaped probe inputs."""
    import torch
    from ..models import fn as fn_model
    from ..ops import d3_ops
    from ..ops import fn_ops as ops
    from ..ops import wgemm
    gates = Gates(log_path=log_path, reps=reps)
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(0)

    # decode MoE: int8-activation GEMV vs the tcgen05 grouped GEMM (FN layer shape, 64 tokens, top-10)
    from ..config import fn_config
    from ..models.fn_weights import _random_experts
    cfg = fn_config()
    gu, dn = _random_experts(cfg, g, dev, lo=0, hi=64)
    E, T, k = 64, 64, 2
    ids = torch.stack([torch.randperm(E, device=dev, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    x = (torch.randn(T, cfg.hidden_size, device=dev, generator=g)).half()

    def moe(gemv: bool):
        P = T * k
        n_tile = wgemm.GEMV_MAX_TOK if gemv else wgemm.pick_n_tile(max(1, (2 * P) // E))
        mi = (P + n_tile - 1) // n_tile + E
        pos, items, n_items = ops.moe_plan(ids, E, n_tile, mi)
        xs = ops.moe_scatter(x, pos)
        act = torch.empty(P, cfg.moe_inter, dtype=torch.float16, device=dev)
        y = torch.empty(P, cfg.hidden_size, dtype=torch.float32, device=dev)
        f = wgemm.gemv_grouped if gemv else (lambda *a, **kw: wgemm.grouped(*a, n_tile=n_tile, **kw))
        f(xs, gu, items, n_items, mi, act, epi=wgemm.EPI_SILU_MUL)
        f(act, dn, items, n_items, mi, y)
        return y[pos.long().view(-1)]

    def set_gemv(on):
        fn_model.GEMV_MOE = bool(on)
    gates.add("moe_gemv_int8", lambda: moe(False), lambda: moe(True), set_gemv, tol=3e-2)

    # D3 latent attention and DSA indexer: tcgen05 kernels vs CUDA-core kernels (64 rows, 4k context)
    Tq, ctx, bs, H, kvr = 64, 4096, 64, 128, 512
    mb = (ctx + bs) // bs + 1
    cache = (torch.randn(Tq * mb, bs, kvr + 64, device=dev, generator=g) * 0.5).to(torch.float8_e4m3fn)
    bt = torch.randperm(Tq * mb, device=dev, generator=g).to(torch.int32).view(Tq, mb).contiguous()
    slots = torch.arange(Tq, dtype=torch.int32, device=dev)
    pos = torch.full((Tq,), ctx - 1, dtype=torch.int32, device=dev)
    q_lat = (torch.randn(H, Tq, kvr, device=dev, generator=g) * 0.3).bfloat16()
    q_pe = torch.randn(Tq, H, 64, device=dev, generator=g) * 0.3
    sel = torch.stack([torch.randperm(ctx, device=dev, generator=g)[:2048] for _ in range(Tq)]).to(torch.int32)

    def mla(cuda_core):
        prev = d3_ops._MLA_CUDA_CORE
        d3_ops._MLA_CUDA_CORE = cuda_core
        try:
            return d3_ops.mla_attn(q_lat, q_pe, cache, bt, slots, pos, 1, sel, 0, 0.07)
        finally:
            d3_ops._MLA_CUDA_CORE = prev

    def set_mla(on):
        d3_ops._MLA_CUDA_CORE = not on
    gates.add("mla_tcgen05", lambda: mla(True), lambda: mla(False), set_mla, tol=2e-2)
    return gates

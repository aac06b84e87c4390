"""Training-run monitor over the trainers' ``log.jsonl`` files (one JSON object per optimizer step; the
reference's trainers write the same kind of per-step JSON log and its READMEs track runs from it,
flashnext/training/rl/train_rl.py:197-210).

:func:`summarize` reads a log and reports per-key rolling means, the last value and anomalies: non-finite values,
gradient-norm spikes (more than ``spike`` times the median of the previous ``window`` steps) and a rising loss
trend (the mean of the last window above the first window by more than ``rise``). ``follow`` tails a live log.

    python -m arcagi2_flashnext_dots3_b200.training.monitor OUT/log.jsonl [--follow]
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
import time


def read_log(path) -> list:
    rows = []
    for line in open(path):
        line = line.strip()
        if line:
            try:
                rows.append(json.loads(line))
            except ValueError:      # a line being written
                break
    return rows


def summarize(rows: list, window: int = 20, spike: float = 5.0, rise: float = 0.25, loss_key: str = None) -> dict:
    keys = sorted({k for r in rows for k, v in r.items() if isinstance(v, (int, float)) and not isinstance(v, bool)})
    out = {"steps": len(rows), "last": rows[-1] if rows else {}, "mean_last_window": {}, "anomalies": []}
    for k in keys:
        vals = [r[k] for r in rows if isinstance(r.get(k), (int, float)) and math.isfinite(r[k])]
        if vals:
            out["mean_last_window"][k] = statistics.fmean(vals[-window:])
        for i, r in enumerate(rows):
            v = r.get(k)
            if isinstance(v, float) and not math.isfinite(v):
                out["anomalies"].append({"step": r.get("step", i), "key": k, "kind": "non-finite"})
    for i, r in enumerate(rows):
        g = r.get("grad_norm")
        prev = [x.get("grad_norm") for x in rows[max(0, i - window):i] if isinstance(x.get("grad_norm"), (int, float))]
        if isinstance(g, (int, float)) and len(prev) >= 3 and g > spike * statistics.median(prev):
            out["anomalies"].append({"step": r.get("step", i), "key": "grad_norm", "kind": "spike", "value": g})
    lk = loss_key or next((k for k in ("loss", "kl", "loss_lp") if k in keys), None)
    if lk and len(rows) >= 2 * window:
        fin = lambda rs: [r[lk] for r in rs if isinstance(r.get(lk), (int, float)) and math.isfinite(r[lk])]
        first = statistics.fmean(fin(rows[:window]) or [0.0])
        last = statistics.fmean(fin(rows[-window:]) or [0.0])
        rising = (last - first) > rise * abs(first) if lk != "loss_lp" else (first - last) > rise * abs(first)
        if rising:
            out["anomalies"].append({"key": lk, "kind": "trend", "first": first, "last": last})
    return out


def follow(path, every: float = 10.0, **kw):
    seen = 0
    while True:
        rows = read_log(path)
        if len(rows) > seen:
            seen = len(rows)
            s = summarize(rows, **kw)
            print(json.dumps({"steps": s["steps"], "mean": s["mean_last_window"], "anomalies": s["anomalies"][-3:]}),
                  flush=True)
        time.sleep(every)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("log")
    ap.add_argument("--follow", action="store_true")
    ap.add_argument("--window", type=int, default=20)
    a = ap.parse_args(argv)
    if a.follow:
        follow(a.log, window=a.window)
    s = summarize(read_log(a.log), window=a.window)
    print(json.dumps(s, indent=1, default=str))
    return s


if __name__ == "__main__":
    main()

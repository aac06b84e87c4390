"""Paired comparison of two builds over the same tasks (the reference's eval/paired_diff.py, both trees).

Per task, each build's expected score under a budget comes from :func:`.scoring.expected_scores`; the per-task
differences are resampled with replacement (bootstrap) for a confidence interval of the mean difference. Pairing by
task removes the task-difficulty variance that dominates an unpaired comparison.

    python -m arcagi2_flashnext_dots3_b200.evaluation.paired --build DIR [DIR ...] --ref DIR [DIR ...]
"""
from __future__ import annotations

import argparse
import random

from .scoring import Pool, expected_scores


def paired_bootstrap(a: dict, b: dict, n_boot: int = 2000, seed: int = 7, level: float = 0.95):
    """Mean of a[t] - b[t] over the common tasks (in points of 100) and its bootstrap interval (lo, hi)."""
    tasks = sorted(set(a) & set(b))
    if not tasks:
        raise ValueError("no common tasks")
    d = [a[t] - b[t] for t in tasks]
    rng = random.Random(seed)
    n = len(d)
    means = sorted(100.0 * sum(rng.choice(d) for _ in range(n)) / n for _ in range(n_boot))
    lo = means[int((1 - level) / 2 * n_boot)]
    hi = means[min(n_boot - 1, int((1 + level) / 2 * n_boot))]
    return 100.0 * sum(d) / n, lo, hi


def compare(build: Pool, ref: Pool, budgets, draws: int = 100, exclude=()):
    tasks = sorted((set(build.tasks) & set(ref.tasks)) - set(exclude))
    rows = []
    for B in budgets:
        sb, tb = expected_scores(build, tasks, B, draws)
        sr, tr = expected_scores(ref, tasks, B, draws)
        diff, lo, hi = paired_bootstrap(sb, sr)
        rows.append({"budget": B, "build": 100 * sum(sb.values()) / len(tasks),
                     "ref": 100 * sum(sr.values()) / len(tasks), "diff": diff, "lo": lo, "hi": hi,
                     "tok_build": tb, "tok_ref": tr, "tasks": len(tasks)})
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--build", nargs="+", required=True)
    ap.add_argument("--ref", nargs="+", required=True)
    ap.add_argument("--budgets", default="50000,80000,118000,140000")
    ap.add_argument("--draws", type=int, default=100)
    ap.add_argument("--exclude", default="")
    a = ap.parse_args(argv)
    rows = compare(Pool(a.build), Pool(a.ref), [float(x) for x in a.budgets.split(",")], a.draws,
                   [x for x in a.exclude.split(",") if x])
    for r in rows:
        print(f"B {r['budget'] / 1000:5.0f}k  build {r['build']:5.1f}  ref {r['ref']:5.1f}  diff {r['diff']:+5.1f} "
              f"[{r['lo']:+5.1f},{r['hi']:+5.1f}]  tok/in {r['tok_build'] / 1000:.0f}k/{r['tok_ref'] / 1000:.0f}k")
    return rows


if __name__ == "__main__":
    main()

"""Scoring of ARC answers and a budget-limited replay of recorded solver samples.

The reference scores its builds by replaying recorded samples under token budgets (flashnext/training/eval/
policy_sim.py, score.py; dotsnote/training/eval/score_hold.py, direct_score.py): what would a solver that may
spend B tokens per test input have submitted, given the samples a build produced? Here a *pool* holds, per task,
the solver sample records (the records :mod:`..agent.vote` ranks, plus ``used`` tokens and per-test ground truth
flags), :func:`simulate` draws each task's samples in a random order until the task's budget is spent, votes with
the solver's own ranking rule and scores pass@2 per test input.

Record format (one JSON object per line of ``samples.jsonl``)::

    {"task": id, "n_test": n, "used": tokens, "progs": [{"verified", "tests", "n_ok", "n_train", "k"}],
     "answer": [grid per test]}

plus a ``truth.json`` of {task: [expected grid per test]} next to it.
"""
from __future__ import annotations

import json
import random
from collections import defaultdict
from pathlib import Path

from ..agent.vote import key, rank


def grid_equal(a, b) -> bool:
    return a is not None and b is not None and key(a) == key(b)


def score_attempts(attempts: list, truth: list) -> float:
    """Fraction of a task's test inputs whose expected grid is among that input's attempts (pass@len(attempts))."""
    if not truth:
        return 0.0
    hit = sum(any(grid_equal(a, t) for a in atts) for atts, t in zip(attempts, truth))
    return hit / len(truth)


def score_submission(sub: dict, truth: dict) -> dict:
    """{task: score} for a submission {task: [{"attempt_1", "attempt_2"} per test]}; missing tasks score 0."""
    out = {}
    for t, exp in truth.items():
        rows = sub.get(t, [])
        atts = [[r.get("attempt_1"), r.get("attempt_2")] for r in rows]
        atts += [[None, None]] * (len(exp) - len(atts))
        out[t] = score_attempts(atts, exp)
    return out


class Pool:
    """Recorded samples of one build, grouped by task."""

    def __init__(self, dirs):
        self.samples = defaultdict(list)
        self.n_test = {}
        self.truth = {}
        for d in ([dirs] if isinstance(dirs, (str, Path)) else dirs):
            d = Path(d)
            for line in open(d / "samples.jsonl"):
                if not line.strip():
                    continue
                r = json.loads(line)
                if r.get("status") == "error":
                    continue
                self.samples[r["task"]].append(r)
                self.n_test[r["task"]] = r["n_test"]
            tp = d / "truth.json"
            if tp.exists():
                self.truth.update(json.load(open(tp)))
        self.tasks = sorted(self.n_test)

    @classmethod
    def from_records(cls, records: list, truth: dict):
        p = cls.__new__(cls)
        p.samples, p.n_test, p.truth = defaultdict(list), {}, dict(truth)
        for r in records:
            p.samples[r["task"]].append(r)
            p.n_test[r["task"]] = r["n_test"]
        p.tasks = sorted(p.n_test)
        return p


def simulate(pool: Pool, tasks: list, budget_per_input: float, rng: random.Random):
    """One replay: per task, samples in a random order are admitted while the task's budget (budget_per_input x
    its test inputs) still covers their token cost; the admitted samples are voted and scored. Returns
    ({task: score}, tokens spent per test input)."""
    scores, spent, n_inputs = {}, 0.0, 0
    for t in tasks:
        n = pool.n_test[t]
        n_inputs += n
        cap = budget_per_input * n
        order = rng.sample(pool.samples[t], len(pool.samples[t]))
        used, admitted = 0.0, []
        for r in order:
            if used + r.get("used", 0) > cap:
                break
            used += r.get("used", 0)
            admitted.append(r)
        spent += used
        ranked = rank(admitted, n) if admitted else [{"attempts": []} for _ in range(n)]
        scores[t] = score_attempts([x["attempts"][:2] for x in ranked], pool.truth.get(t, []))
    return scores, spent / max(1, n_inputs)


def expected_scores(pool: Pool, tasks: list, budget_per_input: float, draws: int = 100, seed: int = 1234):
    """Mean per-task score over `draws` replays (and the mean tokens per input)."""
    rng = random.Random(seed)
    acc = {t: 0.0 for t in tasks}
    tok = 0.0
    for _ in range(draws):
        s, spent = simulate(pool, tasks, budget_per_input, rng)
        tok += spent
        for t in tasks:
            acc[t] += s[t]
    return {t: v / draws for t, v in acc.items()}, tok / draws

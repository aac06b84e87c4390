"""Answer voting across a task's samples: two attempts per test input.

The ranking rule is the reference's (flashnext/kaggle/code_dataset/repl_vote.py:22-50); this module states it
as a ballot per test input:

* each sample casts at most three kinds of evidence for a test input: the output of its last program that
  passed every train pair (**verified**, one vote), its final answer when it has no verified program
  (**answer**, weight 1), and the output of its best partially passing program (**partial**, weight 0.5 times
  that program's train pass rate; best = most train pairs passed, then the latest);
* grids with verified votes rank first, by vote count; every other grid ranks after them by its summed
  answer/partial weight, and evidence of those kinds for a grid that has verified votes is ignored;
* ties go to the grid whose evidence of its ranking kind came from the earliest sample.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field


def key(g) -> str:
    """Canonical text of a grid, used to compare answers."""
    return json.dumps(g, separators=(",", ":"))


@dataclass
class Evidence:
    """What one sample says about one test input."""
    verified: list = None      # grid from a program that passed all train pairs
    answer: list = None        # final answer (only when nothing is verified)
    partial: tuple = None      # (grid, weight) from the best partially passing program


def _best_partial(progs: list):
    """The unverified program with the most passed train pairs (later attempts win ties), if it passed any."""
    best = None
    for p in progs:
        if p.get("verified") or not p.get("tests"):
            continue
        score = (p["n_ok"], p.get("k", 0))
        if best is None or score >= (best["n_ok"], best.get("k", 0)):
            best = p
    return best if best is not None and best["n_ok"] > 0 else None


def sample_evidence(rec: dict, n_test: int) -> list:
    """One :class:`Evidence` per test input from a sample record
    ``{"progs": [{"verified", "tests", "n_ok", "n_train", "k"}], "answer": [grid per test]}``."""
    progs = rec.get("progs") or []
    verified = next((p["tests"] for p in reversed(progs) if p.get("verified")), None)
    part = _best_partial(progs)
    answers = rec.get("answer") or []
    out = []
    for k in range(n_test):
        ev = Evidence()
        if verified is not None:
            ev.verified = verified[k] if k < len(verified) else None
        elif k < len(answers):
            ev.answer = answers[k]
        if part is not None and k < len(part["tests"]) and part["tests"][k] is not None:
            ev.partial = (part["tests"][k], 0.5 * part["n_ok"] / max(1, part["n_train"]))
        out.append(ev)
    return out


@dataclass
class _Entry:
    grid: list
    votes: int = 0
    weight: float = 0.0
    first_vote: int = None     # earliest sample with a verified vote
    first_weight: int = None   # earliest sample with answer/partial evidence


@dataclass
class Ballot:
    """Tally of the evidence for one test input."""
    entries: dict = field(default_factory=dict)

    def _entry(self, grid) -> _Entry:
        return self.entries.setdefault(key(grid), _Entry(grid))

    def add(self, sample: int, ev: Evidence):
        if ev.verified is not None:
            e = self._entry(ev.verified)
            e.votes += 1
            e.first_vote = sample if e.first_vote is None else e.first_vote
        for grid, w in ((ev.answer, 1.0), ev.partial or (None, 0.0)):
            if grid is not None:
                e = self._entry(grid)
                e.weight += w
                e.first_weight = sample if e.first_weight is None else e.first_weight

    def standings(self) -> list:
        """Entries best first: verified grids by votes, then the rest by weight; earliest evidence breaks ties."""
        def order(e: _Entry):
            if e.votes:
                return (0, -e.votes, e.first_vote)
            return (1, -e.weight, e.first_weight)
        return sorted(self.entries.values(), key=order)


def rank(recs: list, n_test: int) -> list:
    """Per test input: the two best grids over all sample records, with their verified vote counts, their tier
    ("ver" or "fb") and the total number of verified votes cast."""
    ballots = [Ballot() for _ in range(n_test)]
    for i, rec in enumerate(recs):
        for k, ev in enumerate(sample_evidence(rec, n_test)):
            ballots[k].add(i, ev)
    res = []
    for b in ballots:
        top = b.standings()[:2]
        res.append({"attempts": [e.grid for e in top],
                    "votes": [e.votes for e in top],
                    "from": ["ver" if e.votes else "fb" for e in top],
                    "n_verified": sum(e.votes for e in b.entries.values())})
    return res

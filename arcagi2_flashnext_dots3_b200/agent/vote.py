"""Candidate voting across a task's samples: two attempts per test input.

Ranking rule (the reference's repl_vote.py:22-50): outputs of programs that pass every train pair ("verified")
are ranked by vote count, earliest sample first on ties; below them come unverified answers (weight 1) and the
test outputs of the best partially-correct program (weight 0.5 x its train pass rate), never re-counting a grid
that already has verified votes.
"""
from __future__ import annotations

import json


def key(g) -> str:
    return json.dumps(g, separators=(",", ":"))


def sample_candidates(rec: dict, n_test: int) -> list:
    """rec: {"progs": [{"verified", "tests", "n_ok", "n_train", "k"}], "answer": [grid per test]}"""
    progs = rec.get("progs") or []
    ver = [p for p in progs if p.get("verified")]
    v = ver[-1]["tests"] if ver else None
    part = None
    nv = [p for p in progs if not p.get("verified") and p.get("tests")]
    if nv:
        best = max(nv, key=lambda p: (p["n_ok"], p.get("k", 0)))
        if best["n_ok"] > 0:
            part = (best["tests"], best["n_ok"] / max(1, best["n_train"]))
    ans = rec.get("answer") or []
    out = []
    for k in range(n_test):
        out.append({"verified": v[k] if v and k < len(v) else None,
                    "answer": ans[k] if not v and k < len(ans) else None,
                    "partial": (part[0][k], part[1]) if part and k < len(part[0]) and part[0][k] is not None else None})
    return out


def rank(recs: list, n_test: int) -> list:
    res = []
    cands = [sample_candidates(r, n_test) for r in recs]
    for k in range(n_test):
        vv, first, grids, fb = {}, {}, {}, {}
        for i, c in enumerate(cands):
            g = c[k]["verified"]
            if g is not None:
                kk = key(g)
                vv[kk] = vv.get(kk, 0) + 1
                first.setdefault(kk, i)
                grids[kk] = g
        for i, c in enumerate(cands):
            for src in ("answer", "partial"):
                x = c[k][src]
                if x is None:
                    continue
                g, w = (x, 1.0) if src == "answer" else (x[0], 0.5 * x[1])
                kk = key(g)
                if kk in vv:
                    continue
                fb[kk] = fb.get(kk, 0.0) + w
                first.setdefault(kk, i)
                grids[kk] = g
        order = sorted(vv, key=lambda q: (-vv[q], first[q])) + sorted(fb, key=lambda q: (-fb[q], first[q]))
        res.append({"attempts": [grids[q] for q in order[:2]],
                    "votes": [vv.get(q, 0) for q in order[:2]],
                    "from": ["ver" if q in vv else "fb" for q in order[:2]],
                    "n_verified": sum(vv.values())})
    return res

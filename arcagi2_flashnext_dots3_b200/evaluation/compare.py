"""Leaf-by-leaf comparison of two checkpoint trees or two build directories (the reference's
flashnext/training/eval/cmp_builds.py): how many tensors differ, by how much, and where.

    python -m arcagi2_flashnext_dots3_b200.evaluation.compare BUILD_A BUILD_B
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch


def leaves(x, path=""):
    """(path, leaf) pairs of a nested dict/list/tuple tree in traversal order."""
    if isinstance(x, dict):
        for k, v in x.items():
            yield from leaves(v, f"{path}.{k}" if path else str(k))
    elif isinstance(x, (list, tuple)):
        for i, v in enumerate(x):
            yield from leaves(v, f"{path}[{i}]")
    else:
        yield path, x


def compare_trees(a, b) -> dict:
    """{"leaves", "differ", "missing", "max_abs": {path: max |a - b|} (tensors of equal shape), "changed": [paths]}."""
    lb = dict(leaves(b))
    out = {"leaves": 0, "differ": 0, "missing": 0, "max_abs": {}, "changed": []}
    for p, x in leaves(a):
        out["leaves"] += 1
        if p not in lb:
            out["missing"] += 1
            continue
        y = lb[p]
        if torch.is_tensor(x) and torch.is_tensor(y):
            same = x.dtype == y.dtype and x.shape == y.shape and torch.equal(x, y)
            if not same and x.shape == y.shape:
                out["max_abs"][p] = float((x.float() - y.float()).abs().max()) if x.numel() else 0.0
        else:
            same = x == y
        if not same:
            out["differ"] += 1
            out["changed"].append(p)
    return out


def compare_builds(dir_a, dir_b) -> dict:
    """{file name: compare_trees(...)} over the .pt files present in both build directories."""
    res = {}
    for f in sorted(Path(dir_a).glob("*.pt")):
        g = Path(dir_b) / f.name
        if g.exists():
            res[f.name] = compare_trees(torch.load(f, map_location="cpu", weights_only=False),
                                        torch.load(g, map_location="cpu", weights_only=False))
    return res


def main(argv=None):
    a, b = (argv or sys.argv[1:])[:2]
    for name, r in compare_builds(a, b).items():
        worst = max(r["max_abs"].values()) if r["max_abs"] else 0.0
        print(f"{name}: {r['differ']}/{r['leaves']} leaves differ, {r['missing']} missing, max |diff| {worst:.3g}")


if __name__ == "__main__":
    main()

"""Grid helper library for model-written ARC programs (imported as ``ak`` inside the sandbox), plus the
train-pair invariants the solver uses to flag suspicious test outputs.

Capabilities follow the reference's helper module (flashnext/kaggle/code_dataset/arckit.py: grid basics :7-66,
geometry and painting :66-160, regions/objects :157-430, diffs :440-570, size rules :576-625, colour maps :645,
invariants and flags :655-708, transform checking :722-800, gravity :840); the implementation here is
independent. Grids are numpy int arrays; every function accepts lists too.
"""
from __future__ import annotations

from collections import Counter, deque

import numpy as np


# ----------------------------------------------------------------------------------------------- basics
def grid(x) -> np.ndarray:
    g = np.asarray(x, dtype=np.int64)
    if g.ndim != 2:
        raise ValueError(f"expected a 2-D grid, got shape {g.shape}")
    return g


def counts(g) -> dict:
    return dict(Counter(grid(g).ravel().tolist()))


def palette(g) -> list:
    return sorted(counts(g))


def bg(g) -> int:
    """Most common colour (ties: the smaller colour), the usual background."""
    c = counts(g)
    return min(c, key=lambda k: (-c[k], k))


def show(g) -> str:
    return "\n".join("".join(str(int(v)) for v in row) for row in grid(g))


D8 = {"id": lambda g: g, "rot90": lambda g: np.rot90(g, 1), "rot180": lambda g: np.rot90(g, 2),
      "rot270": lambda g: np.rot90(g, 3), "fliplr": np.fliplr, "flipud": np.flipud, "transpose": lambda g: g.T,
      "antitranspose": lambda g: np.rot90(g, 2).T}


def d8(g, name=None):
    """All 8 dihedral images {name: grid} or the named one."""
    g = grid(g)
    return D8[name](g).copy() if name else {k: f(g).copy() for k, f in D8.items()}


def bbox(mask):
    m = np.asarray(mask, dtype=bool)
    if not m.any():
        return None
    r = np.where(m.any(1))[0]
    c = np.where(m.any(0))[0]
    return int(r[0]), int(c[0]), int(r[-1]) + 1, int(c[-1]) + 1


def crop(g, box):
    r0, c0, r1, c1 = box
    return grid(g)[r0:r1, c0:c1].copy()


def trim(g, bgc=None):
    g = grid(g)
    b = bbox(g != (bg(g) if bgc is None else bgc))
    return g.copy() if b is None else crop(g, b)


def scale(g, ky, kx=None):
    return np.kron(grid(g), np.ones((ky, kx or ky), dtype=np.int64))


def downscale(g, ky, kx=None):
    """Block-mode downscale (each ky x kx block -> its most common colour)."""
    g = grid(g)
    kx = kx or ky
    H, W = g.shape[0] // ky, g.shape[1] // kx
    out = np.zeros((H, W), dtype=np.int64)
    for r in range(H):
        for c in range(W):
            out[r, c] = bg(g[r * ky:(r + 1) * ky, c * kx:(c + 1) * kx])
    return out


def tile(g, ny, nx=None):
    return np.tile(grid(g), (ny, nx or ny))


def find_sub(big, small, wildcard=None, limit=100) -> list:
    """Top-left positions where `small` occurs in `big` (cells equal to `wildcard` in small match anything)."""
    B, S = grid(big), grid(small)
    out = []
    for r in range(B.shape[0] - S.shape[0] + 1):
        for c in range(B.shape[1] - S.shape[1] + 1):
            win = B[r:r + S.shape[0], c:c + S.shape[1]]
            ok = (win == S) if wildcard is None else ((win == S) | (S == wildcard))
            if ok.all():
                out.append((r, c))
                if len(out) >= limit:
                    return out
    return out


def paste(dst, src, r, c, skip=None):
    d, s = grid(dst).copy(), grid(src)
    for i in range(s.shape[0]):
        for j in range(s.shape[1]):
            if 0 <= r + i < d.shape[0] and 0 <= c + j < d.shape[1] and (skip is None or s[i, j] != skip):
                d[r + i, c + j] = s[i, j]
    return d


def line(g, r0, c0, r1, c1, colour):
    """Straight (horizontal, vertical or 45-degree) segment, endpoints included."""
    g = grid(g).copy()
    n = max(abs(r1 - r0), abs(c1 - c0))
    dr, dc = np.sign(r1 - r0), np.sign(c1 - c0)
    for t in range(n + 1):
        g[r0 + t * dr, c0 + t * dc] = colour
    return g


def _nbrs(diag):
    return [(-1, 0), (1, 0), (0, -1), (0, 1)] + ([(-1, -1), (-1, 1), (1, -1), (1, 1)] if diag else [])


def _region(g, r, c, diag=False):
    g = grid(g)
    col = g[r, c]
    seen = {(r, c)}
    q = deque([(r, c)])
    while q:
        y, x = q.popleft()
        for dy, dx in _nbrs(diag):
            ny, nx = y + dy, x + dx
            if 0 <= ny < g.shape[0] and 0 <= nx < g.shape[1] and (ny, nx) not in seen and g[ny, nx] == col:
                seen.add((ny, nx))
                q.append((ny, nx))
    return seen


def flood(g, r, c, colour, diag=False):
    g2 = grid(g).copy()
    for y, x in _region(g2, r, c, diag):
        g2[y, x] = colour
    return g2


def enclosed(g, bgc=None, diag=False):
    """Mask of background cells not connected to the border."""
    g = grid(g)
    b = bg(g) if bgc is None else bgc
    H, W = g.shape
    outside = np.zeros_like(g, dtype=bool)
    for r in range(H):
        for c in range(W):
            if (r in (0, H - 1) or c in (0, W - 1)) and g[r, c] == b and not outside[r, c]:
                for y, x in _region(g, r, c, diag):
                    outside[y, x] = True
    return (g == b) & ~outside


def gravity(g, direction="down", bgc=None):
    """Cells fall towards `direction` column- or row-wise (each cell independently)."""
    g = grid(g)
    b = bg(g) if bgc is None else bgc
    rot = {"down": 0, "right": 1, "up": 2, "left": 3}[direction]
    h = np.rot90(g, rot).copy()
    for c in range(h.shape[1]):
        col = [v for v in h[:, c] if v != b]
        h[:, c] = [b] * (h.shape[0] - len(col)) + col
    return np.rot90(h, -rot).copy()


# ---------------------------------------------------------------------------------------------- objects
class Obj:
    def __init__(self, cells, colours, box, grid_):
        self.cells = cells
        self.colours = colours
        self.box = box
        self.size = len(cells)
        r0, c0, r1, c1 = box
        self.patch = np.full((r1 - r0, c1 - c0), -1, dtype=np.int64)
        for y, x in cells:
            self.patch[y - r0, x - c0] = grid_[y, x]

    @property
    def colour(self):
        return max(self.colours, key=self.colours.get)

    @property
    def shape(self):
        return self.patch >= 0

    def __repr__(self):
        return f"Obj(size={self.size}, box={self.box}, colours={self.colours})"


def objects(g, bgc=None, diag=False, multicolour=False, min_size=1) -> list:
    """Connected components of non-background cells (single colour unless multicolour)."""
    g = grid(g)
    b = bg(g) if bgc is None else bgc
    seen = np.zeros_like(g, dtype=bool)
    out = []
    for r in range(g.shape[0]):
        for c in range(g.shape[1]):
            if seen[r, c] or g[r, c] == b:
                continue
            cells, q = [], deque([(r, c)])
            seen[r, c] = True
            while q:
                y, x = q.popleft()
                cells.append((y, x))
                for dy, dx in _nbrs(diag):
                    ny, nx = y + dy, x + dx
                    if 0 <= ny < g.shape[0] and 0 <= nx < g.shape[1] and not seen[ny, nx] and g[ny, nx] != b and \
                            (multicolour or g[ny, nx] == g[r, c]):
                        seen[ny, nx] = True
                        q.append((ny, nx))
            if len(cells) >= min_size:
                ys, xs = zip(*cells)
                out.append(Obj(cells, dict(Counter(int(g[y, x]) for y, x in cells)),
                               (min(ys), min(xs), max(ys) + 1, max(xs) + 1), g))
    return out


# --------------------------------------------------------------------------------------------- structure
def symmetries(g) -> list:
    g = grid(g)
    out = []
    for name in ("fliplr", "flipud", "rot180"):
        if np.array_equal(D8[name](g), g):
            out.append(name)
    if g.shape[0] == g.shape[1]:
        for name in ("transpose", "rot90"):
            if np.array_equal(D8[name](g), g):
                out.append(name)
    return out


def period(g):
    """Smallest (row period, column period) with which the grid repeats exactly."""
    g = grid(g)

    def p(axis):
        n = g.shape[axis]
        for k in range(1, n + 1):
            a = g if axis == 0 else g.T
            if all(np.array_equal(a[i], a[i % k]) for i in range(n)):
                return k
        return n
    return p(0), p(1)


def diff(a, b) -> dict:
    a, b = grid(a), grid(b)
    if a.shape != b.shape:
        return {"shape": (a.shape, b.shape)}
    m = a != b
    return {"n": int(m.sum()), "cells": [(int(r), int(c), int(a[r, c]), int(b[r, c])) for r, c in zip(*np.where(m))][:8]}


def color_map(train):
    m = {}
    for i, o in _pairs(train):
        if i.shape != o.shape:
            return None
        for x, y in zip(i.ravel().tolist(), o.ravel().tolist()):
            if m.setdefault(x, y) != y:
                return None
    return m


def _pairs(train):
    return [(grid(p["input"]), grid(p["output"])) for p in train]


def size_rule(train):
    """A rule predicting the output shape from the input shape, or None."""
    P = _pairs(train)
    rules = [("same", lambda s: s), ("transpose", lambda s: (s[1], s[0]))]
    o0 = P[0][1].shape
    if all(o.shape == o0 for _, o in P):
        rules.append(("constant", lambda s, o0=o0: o0))
    i0 = P[0][0].shape
    if i0[0] and i0[1] and o0[0] % i0[0] == 0 and o0[1] % i0[1] == 0:
        ky, kx = o0[0] // i0[0], o0[1] // i0[1]
        rules.append((f"scale {ky}x{kx}", lambda s, ky=ky, kx=kx: (s[0] * ky, s[1] * kx)))
    for name, f in rules:
        if all(f(i.shape) == o.shape for i, o in P):
            return name, f
    return None


# -------------------------------------------------------------------------------------------- invariants
def _inv_defs(train):
    P = _pairs(train)
    out_cols = set().union(*(set(palette(o)) for _, o in P))
    added = set().union(*(set(palette(o)) - set(palette(i)) for i, o in P))
    defs = [
        ("output shape == input shape", lambda i, o: i.shape == o.shape),
        ("output colours subset of input colours", lambda i, o: set(palette(o)) <= set(palette(i))),
        ("output colours subset of input colours + colours added in training outputs",
         lambda i, o: set(palette(o)) <= set(palette(i)) | added),
        ("output colours subset of training-output colours + input colours",
         lambda i, o: set(palette(o)) <= out_cols | set(palette(i))),
        ("output differs from input", lambda i, o: i.shape != o.shape or not np.array_equal(i, o)),
        ("output has >= 2 colours", lambda i, o: len(palette(o)) >= 2),
        ("non-background input cells kept",
         lambda i, o: i.shape == o.shape and np.array_equal(o[i != bg(i)], i[i != bg(i)])),
        ("only background cells change", lambda i, o: i.shape == o.shape and bool(np.all((i == o) | (i == bg(i))))),
        ("same number of colours", lambda i, o: len(palette(o)) == len(palette(i))),
        ("output smaller than input", lambda i, o: o.size < i.size),
        ("output larger than input", lambda i, o: o.size > i.size),
        ("output is a sub-grid of the input",
         lambda i, o: o.shape[0] <= i.shape[0] and o.shape[1] <= i.shape[1] and bool(find_sub(i, o, limit=1))),
    ]
    sr = size_rule(train)
    if sr:
        defs.append((f"output shape follows rule: {sr[0]}", lambda i, o, f=sr[1]: f(i.shape) == o.shape))
    return defs


SIZE_INV = ("output shape", "output smaller", "output larger", "output is a sub-grid")


def invariants(train, names_only=True):
    out = []
    for name, f in _inv_defs(train):
        try:
            if all(bool(f(i, o)) for i, o in _pairs(train)):
                out.append((name, f))
        except Exception:
            continue
    return [n for n, _ in out] if names_only else out


def violations(train, test_inputs, test_outputs) -> list:
    inv = invariants(train, names_only=False)
    res = []
    for ti, to in zip(test_inputs, test_outputs):
        if to is None:
            res.append(["no output"])
            continue
        i, o = grid(ti), grid(to)
        bad = []
        for n, f in inv:
            try:
                if not f(i, o):
                    bad.append(n)
            except Exception:
                bad.append(n)
        res.append(bad)
    return res


def flag(train, test_inputs, test_outputs) -> list:
    """Train invariants (other than size ones) that a candidate's test outputs break."""
    bad = set()
    for v in violations(train, test_inputs, test_outputs):
        bad.update(x for x in v if not x.startswith(SIZE_INV))
    return sorted(bad)


def check(transform, train, verbose=False) -> dict:
    """Run transform on every train input: {"ok": all equal, "pairs": [{"ok", "diff"}]}."""
    pairs = []
    for i, o in _pairs(train):
        try:
            got = grid(transform(i.copy()))
            ok = got.shape == o.shape and bool(np.array_equal(got, o))
            pairs.append({"ok": ok, "diff": None if ok else diff(o, got)})
        except Exception as e:
            pairs.append({"ok": False, "error": repr(e)[:200]})
    res = {"ok": all(p["ok"] for p in pairs), "pairs": pairs}
    if verbose:
        print(res)
    return res


def describe(train) -> str:
    """Short text summary of a task's train pairs (shapes, palettes, invariants)."""
    lines = []
    for k, (i, o) in enumerate(_pairs(train)):
        lines.append(f"pair {k}: {i.shape} -> {o.shape}, colours {palette(i)} -> {palette(o)}, "
                     f"objects {len(objects(i))} -> {len(objects(o))}")
    lines.append("invariants: " + "; ".join(invariants(train)))
    return "\n".join(lines)

"""Grid helper library for model-written ARC programs (pre-loaded as ``ak`` inside the sandbox), plus the
train-pair invariants and transform checks the solver feeds back to the model.

The public surface is the reference's helper module (flashnext/kaggle/code_dataset/arckit.py:4 ``__all__``):
programs written against it run here unchanged, so every name, signature, return type, box convention
(``(r0, c0, r1, c1)`` inclusive), ordering rule and report text follows that module. The code is this
framework's own. Grids are numpy int64 arrays; every function also accepts nested lists and returns new arrays.
"""
from __future__ import annotations

import inspect
import time
from collections import Counter, deque

import numpy as np

__all__ = ["grid", "show", "bg", "task_bg", "palette", "counts", "d8", "D8", "crop", "trim", "bbox", "scale",
           "downscale", "tile", "find_sub", "paste", "line", "ray", "move", "flood", "enclosed", "split_grid",
           "period", "repair_period", "symmetries", "complete_symmetry", "objects", "Obj", "diff", "obj_diff",
           "size_rule", "color_map", "invariants", "violations", "flag", "check", "equivariance", "gravity",
           "describe", "help"]

# dihedral group names, identity first
D8 = ("id", "rot90", "rot180", "rot270", "flipud", "fliplr", "transpose", "antitranspose")
_D8_OPS = {
    "id": lambda a: a,
    "rot90": lambda a: np.rot90(a, 3),          # clockwise quarter turn
    "rot180": lambda a: a[::-1, ::-1],
    "rot270": lambda a: np.rot90(a, 1),         # counter-clockwise quarter turn
    "flipud": lambda a: a[::-1, :],
    "fliplr": lambda a: a[:, ::-1],
    "transpose": lambda a: a.T,
    "antitranspose": lambda a: a[::-1, ::-1].T,
}
_NEIGHBOURS4 = ((-1, 0), (1, 0), (0, -1), (0, 1))
_NEIGHBOURS8 = _NEIGHBOURS4 + ((-1, -1), (-1, 1), (1, -1), (1, 1))


# ----------------------------------------------------------------------------------------------- basics
def grid(x) -> np.ndarray:
    """A new 2-D int64 array from a grid given as nested lists or an array."""
    g = np.array(x, dtype=np.int64)
    if g.ndim != 2:
        raise ValueError(f"expected a 2-D grid, got shape {g.shape}")
    return g


def show(g, name=None, coords=False) -> str:
    """Text rendering, one digit per cell ('?' outside 0..9); coords=True adds column and row indices."""
    g = grid(g)
    body = ["".join(str(int(v)) if 0 <= v <= 9 else "?" for v in row) for row in g]
    if coords:
        header = "   " + "".join(str(j % 10) for j in range(g.shape[1]))
        body = [header] + [f"{i:2d} {row}" for i, row in enumerate(body)]
    title = f"{name} ({g.shape[0]}x{g.shape[1]}):\n" if name else ""
    return title + "\n".join(body)


def counts(g) -> dict:
    """{colour: cells}, most frequent colour first (ties: smaller colour first)."""
    vals, ns = np.unique(grid(g), return_counts=True)
    pairs = sorted(zip(vals.tolist(), ns.tolist()), key=lambda p: (-p[1], p[0]))
    return dict(pairs)


def palette(g) -> list:
    return np.unique(grid(g)).tolist()


def _dominant(tally: dict) -> int:
    """Most frequent colour of a tally; among tied colours 0 wins, else the smallest."""
    top = max(tally.values())
    tied = sorted(c for c, n in tally.items() if n == top)
    return 0 if 0 in tied else tied[0]


def bg(g) -> int:
    """Background colour of a grid: its most frequent colour (ties: 0 if tied, else the smallest)."""
    return _dominant(counts(g))


def task_bg(train) -> int:
    """Background colour over all grids of a task's train pairs (same tie rule as :func:`bg`)."""
    tally = Counter()
    for pair in train:
        for side in ("input", "output"):
            if side in pair:
                tally.update(counts(pair[side]))
    return _dominant(tally)


def d8(g, name=None):
    """The named dihedral image of g, or all eight as {name: grid} in :data:`D8` order."""
    g = grid(g)
    if name is not None:
        return np.ascontiguousarray(_D8_OPS[name](g)).copy()
    return {k: np.ascontiguousarray(_D8_OPS[k](g)).copy() for k in D8}


def bbox(mask):
    """Inclusive bounding box (r0, c0, r1, c1) of the true cells of a mask, or None when it has none."""
    m = np.asarray(mask).astype(bool)
    rows = np.flatnonzero(m.any(axis=1))
    if rows.size == 0:
        return None
    cols = np.flatnonzero(m.any(axis=0))
    return int(rows[0]), int(cols[0]), int(rows[-1]), int(cols[-1])


def crop(g, box):
    """Sub-grid inside an inclusive box."""
    r0, c0, r1, c1 = box
    return grid(g)[r0:r1 + 1, c0:c1 + 1].copy()


def trim(g, bgc=None):
    """Crop to the bounding box of the cells that differ from the background (a copy if there are none)."""
    g = grid(g)
    box = bbox(g != (bg(g) if bgc is None else bgc))
    return g.copy() if box is None else crop(g, box)


def scale(g, ky, kx=None):
    """Every cell becomes a ky x kx block."""
    kx = ky if kx is None else kx
    return grid(g).repeat(ky, axis=0).repeat(kx, axis=1)


def downscale(g, ky, kx=None, how="mode"):
    """Every ky x kx block becomes one cell: its most frequent colour (ties: the colour met first in raster
    order). how='any': a block with any non-background cell ignores the background."""
    g = grid(g)
    kx = ky if kx is None else kx
    H, W = g.shape
    if H % ky or W % kx:
        raise ValueError(f"grid {H}x{W} is not divisible into {ky}x{kx} blocks")
    b = bg(g)
    blocks = g.reshape(H // ky, ky, W // kx, kx).transpose(0, 2, 1, 3).reshape(H // ky, W // kx, ky * kx)
    out = np.empty((H // ky, W // kx), dtype=np.int64)
    for i in range(out.shape[0]):
        for j in range(out.shape[1]):
            cells = blocks[i, j].tolist()
            if how == "any" and any(v != b for v in cells):
                cells = [v for v in cells if v != b]
            tally = Counter(cells)
            top = max(tally.values())
            out[i, j] = next(v for v in cells if tally[v] == top)
    return out


def tile(g, ny, nx=None):
    return np.tile(grid(g), (ny, ny if nx is None else nx))


def find_sub(big, small, wildcard=None, limit=100) -> list:
    """Top-left (r, c) of every occurrence of `small` in `big`, raster order, at most `limit`; cells of `small`
    equal to `wildcard` match anything."""
    B, S = grid(big), grid(small)
    h, w = S.shape
    if h > B.shape[0] or w > B.shape[1]:
        return []
    windows = np.lib.stride_tricks.sliding_window_view(B, (h, w))
    match = windows == S
    if wildcard is not None:
        match |= (S == wildcard)
    hit_r, hit_c = np.nonzero(match.all(axis=(2, 3)))
    return [(int(r), int(c)) for r, c in list(zip(hit_r, hit_c))[:limit]]


def paste(dst, src, r, c, skip=None):
    """Copy of `dst` with `src` written at top-left (r, c), clipped to dst; cells of src equal to `skip` are left
    out."""
    D, S = grid(dst), grid(src)
    top, left = max(r, 0), max(c, 0)
    bottom, right = min(r + S.shape[0], D.shape[0]), min(c + S.shape[1], D.shape[1])
    if top >= bottom or left >= right:
        return D
    part = S[top - r:bottom - r, left - c:right - c]
    view = D[top:bottom, left:right]
    if skip is None:
        view[...] = part
    else:
        keep = part != skip
        view[keep] = part[keep]
    return D


def _step(a, b) -> int:
    return (b > a) - (b < a)


def line(g, r0, c0, r1, c1, colour):
    """Copy with a horizontal, vertical or 45-degree segment drawn, both ends included (cells outside the grid
    are skipped); other directions raise ValueError."""
    g = grid(g)
    dy, dx = r1 - r0, c1 - c0
    n = max(abs(dy), abs(dx))
    if n and dy and dx and abs(dy) != abs(dx):
        raise ValueError("line: only horizontal, vertical or 45-degree segments")
    sr, sc = _step(r0, r1), _step(c0, c1)
    H, W = g.shape
    for k in range(n + 1):
        y, x = r0 + k * sr, c0 + k * sc
        if 0 <= y < H and 0 <= x < W:
            g[y, x] = colour
    return g


def ray(g, r, c, dr, dc, colour, stop=None, overwrite=True):
    """Copy with a ray painted from the cell after (r, c) in direction (dr, dc) to the border. It ends before
    the first cell whose colour is in `stop` (a colour or a collection of colours); with overwrite=False only
    background cells along the way are painted."""
    g = grid(g)
    b = bg(g)
    if stop is None:
        stops = set()
    elif isinstance(stop, (int, np.integer)):
        stops = {int(stop)}
    else:
        stops = set(stop)
    H, W = g.shape
    y, x = r + dr, c + dc
    while 0 <= y < H and 0 <= x < W and g[y, x] not in stops:
        if overwrite or g[y, x] == b:
            g[y, x] = colour
        y, x = y + dr, x + dc
    return g


def move(g, obj, dr, dc, bgc=None):
    """Copy with an object (from :func:`objects`) shifted by (dr, dc): its old cells take the background
    (the object's, or `bgc`), then its cells are drawn at the new place, clipped to the grid."""
    g = grid(g)
    fill = obj.bg if bgc is None else bgc
    for y, x in obj.cells:
        g[y, x] = fill
    H, W = g.shape
    for y, x in obj.cells:
        ny, nx = y + dr, x + dc
        if 0 <= ny < H and 0 <= nx < W:
            g[ny, nx] = obj.sub[y - obj.r0, x - obj.c0]
    return g


def _bfs(start: list, passable, H: int, W: int, diag: bool) -> np.ndarray:
    """Mask of the cells reachable from `start` through cells where passable(y, x) holds."""
    seen = np.zeros((H, W), dtype=bool)
    queue = deque()
    for y, x in start:
        if not seen[y, x]:
            seen[y, x] = True
            queue.append((y, x))
    steps = _NEIGHBOURS8 if diag else _NEIGHBOURS4
    while queue:
        y, x = queue.popleft()
        for dy, dx in steps:
            ny, nx = y + dy, x + dx
            if 0 <= ny < H and 0 <= nx < W and not seen[ny, nx] and passable(ny, nx):
                seen[ny, nx] = True
                queue.append((ny, nx))
    return seen


def _region(g, r, c, diag=False) -> np.ndarray:
    """Mask of the same-colour region containing (r, c)."""
    g = grid(g)
    colour = g[r, c]
    return _bfs([(r, c)], lambda y, x: g[y, x] == colour, g.shape[0], g.shape[1], diag)


def flood(g, r, c, colour, diag=False):
    """Copy with the same-colour region containing (r, c) painted."""
    g = grid(g)
    g[_region(g, r, c, diag)] = colour
    return g


def enclosed(g, bgc=None, diag=False):
    """Mask of background cells that cannot reach the border through background cells (holes)."""
    g = grid(g)
    b = bg(g) if bgc is None else bgc
    H, W = g.shape
    free = g == b
    edge = [(y, x) for y in range(H) for x in (0, W - 1)] + [(y, x) for x in range(W) for y in (0, H - 1)]
    outside = _bfs([p for p in edge if free[p]], lambda y, x: free[y, x], H, W, diag)
    return free & ~outside


# --------------------------------------------------------------------------------------------- structure
def _runs_between(lines: list, n: int) -> list:
    """Inclusive (start, end) index ranges of [0, n) left between separator lines."""
    cut = sorted(set(lines))
    out, start = [], 0
    for s in cut + [n]:
        if s > start:
            out.append((start, s - 1))
        start = s + 1
    return out


def split_grid(g):
    """Split along full rows and columns of one non-background colour (the colour that yields the most
    cells). Returns {'rows', 'cols', 'colour', 'boxes' (inclusive, one list per band of rows), 'cells' (the
    sub-grids)} or None when no colour makes at least two cells."""
    g = grid(g)
    H, W = g.shape
    b = bg(g)
    best = None
    for colour in palette(g):
        if colour == b:
            continue
        full = g == colour
        rows = np.flatnonzero(full.all(axis=1)).tolist()
        cols = np.flatnonzero(full.all(axis=0)).tolist()
        if not (rows or cols) or len(rows) == H or len(cols) == W:
            continue
        rb, cb = _runs_between(rows, H), _runs_between(cols, W)
        n_cells = len(rb) * len(cb)
        if n_cells >= 2 and (best is None or n_cells > best[0]):
            best = (n_cells, rows, cols, colour, rb, cb)
    if best is None:
        return None
    _, rows, cols, colour, rb, cb = best
    boxes = [[(r0, c0, r1, c1) for (c0, c1) in cb] for (r0, r1) in rb]
    return {"rows": rows, "cols": cols, "colour": colour, "boxes": boxes,
            "cells": [[crop(g, box) for box in band] for band in boxes]}


def _classes_agree(g, care, pr: int, pc: int) -> bool:
    """Do all cared cells with the same (row mod pr, col mod pc) share one colour?"""
    H, W = g.shape
    cls = (np.arange(H)[:, None] % pr) * pc + (np.arange(W)[None, :] % pc)
    seen = {}
    for k, v in zip(cls[care].tolist(), g[care].tolist()):
        if seen.setdefault(k, v) != v:
            return False
    return True


def period(g, ignore=None):
    """Smallest tile (pr, pc) that the grid repeats, cells equal to `ignore` matching anything. Candidate row
    periods are those up to H/2 under which every row class agrees column by column (likewise for columns), plus
    H (W); pairs are tried by area, then row period, and the first that holds jointly wins; (H, W) otherwise."""
    g = grid(g)
    H, W = g.shape
    care = np.ones(g.shape, dtype=bool) if ignore is None else g != ignore

    def axis_ok(a, m, p):
        for off in range(p):
            sl, ms = a[off::p], m[off::p]
            for j in range(a.shape[1]):
                v = sl[:, j][ms[:, j]]
                if v.size and (v != v[0]).any():
                    return False
        return True

    prs = [p for p in range(1, H // 2 + 1) if axis_ok(g, care, p)] + [H]
    pcs = [p for p in range(1, W // 2 + 1) if axis_ok(g.T, care.T, p)] + [W]
    for pr, pc in sorted(((a, b) for a in prs for b in pcs), key=lambda t: (t[0] * t[1], t[0])):
        if (pr, pc) == (H, W) or _classes_agree(g, care, pr, pc):
            return pr, pc
    return H, W


def repair_period(g, ignore):
    """Fill the cells equal to `ignore` from the grid's period (:func:`period` with that ignore colour). None if
    the grid has no period smaller than itself or a class has no known cell."""
    g = grid(g)
    pr, pc = period(g, ignore)
    if (pr, pc) == g.shape:
        return None
    H, W = g.shape
    known = {}
    for y in range(H):
        for x in range(W):
            if g[y, x] != ignore:
                known.setdefault((y % pr, x % pc), g[y, x])
    out = g.copy()
    for y, x in zip(*np.nonzero(g == ignore)):
        v = known.get((y % pr, x % pc))
        if v is None:
            return None
        out[y, x] = v
    return out


def symmetries(g, ignore=None) -> list:
    """Names of the non-identity dihedral maps that leave g unchanged (with `ignore`, compared only where
    neither the grid nor its image has that colour)."""
    g = grid(g)
    out = []
    for name, img in d8(g).items():
        if name == "id" or img.shape != g.shape:
            continue
        if ignore is None:
            same = np.array_equal(img, g)
        else:
            both = (g != ignore) & (img != ignore)
            same = np.array_equal(img[both], g[both])
        if same:
            out.append(name)
    return out


def complete_symmetry(g, ignore, syms=None):
    """Fill the cells equal to `ignore` from their images under the grid's symmetries (three passes over
    `syms`, default :func:`symmetries` with that ignore colour). None if no symmetry or cells stay unknown."""
    g = grid(g)
    syms = symmetries(g, ignore) if syms is None else syms
    if not syms:
        return None
    out = g.copy()
    for _ in range(3):
        for name in syms:
            img = d8(out, name)
            fill = (out == ignore) & (img != ignore)
            out[fill] = img[fill]
    return None if (out == ignore).any() else out


# ---------------------------------------------------------------------------------------------- objects
class Obj:
    """A connected component. Fields: colour (most frequent), colours, size, r0 c0 r1 c1 (inclusive box), h w,
    cells (sorted (r, c)), mask [h, w], sub [h, w] (the object on its background), bg, shape_key, holes (enclosed
    background regions), border (touches the grid edge), rect (fills its box), idx (rank in :func:`objects`);
    properties box, slice, center, sym (symmetries of the mask)."""
    __slots__ = ("colour", "colours", "size", "r0", "c0", "r1", "c1", "h", "w", "cells", "mask", "sub", "bg",
                 "shape_key", "holes", "border", "rect", "_sym", "idx")

    @property
    def box(self):
        return self.r0, self.c0, self.r1, self.c1

    @property
    def slice(self):
        return np.s_[self.r0:self.r1 + 1, self.c0:self.c1 + 1]

    @property
    def center(self):
        return (self.r0 + self.r1) / 2, (self.c0 + self.c1) / 2

    @property
    def sym(self):
        if self._sym is None:
            self._sym = symmetries(self.mask.astype(np.int64))
        return self._sym

    def __repr__(self):
        extra = " rect" if self.rect else ""
        extra += f" holes={self.holes}" if self.holes else ""
        extra += " border" if self.border else ""
        multi = f" colours={self.colours}" if len(self.colours) > 1 else ""
        return (f"Obj(colour={self.colour}{multi} size={self.size} box=({self.r0},{self.c0},{self.r1},{self.c1}) "
                f"{self.h}x{self.w}{extra})")


def _holes(mask: np.ndarray) -> int:
    """Number of 4-connected regions of non-object cells that do not reach beyond the object's box."""
    if mask.all():
        return 0
    free = np.pad(~mask, 1, constant_values=True)
    H, W = free.shape
    label = np.zeros(free.shape, dtype=bool)
    regions = 0
    for y, x in zip(*np.nonzero(free)):
        if label[y, x]:
            continue
        label |= _bfs([(y, x)], lambda a, b: free[a, b], H, W, False)
        regions += 1
    return regions - 1          # the padded ring is one region that is outside


def _make_obj(g, cells: list, b: int) -> Obj:
    H, W = g.shape
    o = Obj()
    ys = [y for y, _ in cells]
    xs = [x for _, x in cells]
    o.r0, o.r1, o.c0, o.c1 = min(ys), max(ys), min(xs), max(xs)
    o.h, o.w = o.r1 - o.r0 + 1, o.c1 - o.c0 + 1
    o.cells = sorted(cells)
    o.size = len(cells)
    o.bg = b
    o.mask = np.zeros((o.h, o.w), dtype=bool)
    o.mask[np.array(ys) - o.r0, np.array(xs) - o.c0] = True
    o.sub = np.full((o.h, o.w), b, dtype=np.int64)
    o.sub[o.mask] = g[o.r0:o.r1 + 1, o.c0:o.c1 + 1][o.mask]
    vals = o.sub[o.mask].tolist()
    tally = Counter(vals)
    top = max(tally.values())
    o.colour = next(v for v in vals if tally[v] == top)
    o.colours = sorted(tally)
    o.shape_key = (o.h, o.w, o.mask.tobytes())
    o.rect = bool(o.mask.all())
    o.border = o.r0 == 0 or o.c0 == 0 or o.r1 == H - 1 or o.c1 == W - 1
    o.holes = _holes(o.mask)
    o._sym = None
    o.idx = -1
    return o


def objects(g, bgc=None, diag=False, multicolour=False, min_size=1) -> list:
    """Connected components of non-background cells (one colour each unless multicolour), largest first, then
    by top row and left column; each gets its rank as ``idx``."""
    g = grid(g)
    b = bg(g) if bgc is None else bgc
    H, W = g.shape
    taken = g == b
    found = []
    for y, x in zip(*np.nonzero(~taken)):
        if taken[y, x]:
            continue
        colour = g[y, x]
        same = (lambda a, c: g[a, c] != b) if multicolour else (lambda a, c: g[a, c] == colour)
        comp = _bfs([(y, x)], lambda a, c: not taken[a, c] and same(a, c), H, W, diag)
        taken |= comp
        found.append(_make_obj(g, [(int(a), int(c)) for a, c in zip(*np.nonzero(comp))], b))
    found = [o for o in found if o.size >= min_size]
    found.sort(key=lambda o: (-o.size, o.r0, o.c0))
    for k, o in enumerate(found):
        o.idx = k
    return found


# ------------------------------------------------------------------------------------------------- diffs
class Diff(dict):
    """dict of a grid comparison whose str() is its one-line text."""

    def __str__(self):
        return self["text"]

    __repr__ = __str__


def _shape_relation(A, B):
    """A sentence naming how B's content derives from A's when the shapes differ, or None."""
    ha, wa = A.shape
    hb, wb = B.shape
    images = d8(A)
    for name, img in images.items():
        if img.shape == B.shape and np.array_equal(img, B):
            return f"output = input {name}"
    if hb % ha == 0 and wb % wa == 0:
        fy, fx = hb // ha, wb // wa
        if np.array_equal(scale(A, fy, fx), B):
            return f"output = input scaled x{fy}x{fx}"
        if np.array_equal(tile(A, fy, fx), B):
            return f"output = input tiled {fy}x{fx}"
        layout = [[next((n for n, img in images.items()
                         if img.shape == (ha, wa) and np.array_equal(img, B[i * ha:(i + 1) * ha, j * wa:(j + 1) * wa])),
                        None) for j in range(fx)] for i in range(fy)]
        if all(n is not None for row in layout for n in row):
            return f"output = {fy}x{fx} blocks of the input under {layout}"
    if ha % hb == 0 and wa % wb == 0 and np.array_equal(scale(B, ha // hb, wa // wb), A):
        return f"output = input downscaled /{ha // hb}x{wa // wb}"
    if hb <= ha and wb <= wa:
        at = find_sub(A, B, limit=4)
        if at:
            return f"output = crop of input at {at[:3]}"
        for name, img in d8(B).items():
            if img.shape[0] <= ha and img.shape[1] <= wa and find_sub(A, img, limit=1):
                return f"output = {name} of a crop of the input"
    return None


def diff(a, b, max_list=6):
    """Compare two grids. Same shape: changed-cell count, (from, to) transition counts, inclusive box and mask of
    the changes; different shapes: the shape change, a derivation of b from a when one is found, and colours
    gained or lost. str() of the result is its summary line."""
    A, B = grid(a), grid(b)
    d = Diff(same_shape=A.shape == B.shape, shape_a=A.shape, shape_b=B.shape)
    if A.shape != B.shape:
        parts = [f"shape {A.shape[0]}x{A.shape[1]} -> {B.shape[0]}x{B.shape[1]}"]
        rel = _shape_relation(A, B)
        if rel:
            parts.append(rel)
        pa, pb = set(palette(A)), set(palette(B))
        if pb - pa:
            parts.append(f"new colours {sorted(pb - pa)}")
        if pa - pb:
            parts.append(f"dropped colours {sorted(pa - pb)}")
        d.update(n_changed=None, transitions={}, box=None, text="; ".join(parts))
        return d
    changed = A != B
    n = int(changed.sum())
    trans = Counter(zip(A[changed].tolist(), B[changed].tolist())).most_common()
    d.update(n_changed=n, transitions=dict(trans), box=bbox(changed), mask=changed)
    if n == 0:
        d["text"] = "identical"
        return d
    shown = ", ".join(f"{x}->{y}:{k}" for (x, y), k in trans[:max_list])
    rest = f" (+{len(trans) - max_list} more)" if len(trans) > max_list else ""
    d["text"] = f"same shape; {n}/{A.size} cells change in box {d['box']}; {shown}{rest}"
    return d


_EVENT_KINDS = ("same", "moved", "recoloured", "reshaped", "deleted", "created")


def obj_diff(a, b, bgc=None, diag=False, multicolour=False) -> list:
    """Match the objects of a to those of b and list the events: ('same', x, y), ('moved', x, y, (dr, dc)),
    ('recoloured', x, y, (old, new)), ('reshaped', x, y), ('deleted', x), ('created', y). Matching runs in
    passes: identical content (nearest first), then the same mask at the same place (a recolouring), then
    overlapping boxes (nearest first); what is left was deleted or created."""
    A, B = grid(a), grid(b)
    b0 = bg(A) if bgc is None else bgc
    xs, ys = objects(A, b0, diag, multicolour), objects(B, b0, diag, multicolour)
    free_x = {x.idx for x in xs}
    free_y = {y.idx for y in ys}
    events = []

    def near(x, y):
        return abs(x.r0 - y.r0) + abs(x.c0 - y.c0)

    def match_pass(keyf, kind):
        pool = {}
        for y in ys:
            if y.idx in free_y:
                pool.setdefault(keyf(y), []).append(y)
        for x in xs:
            if x.idx not in free_x:
                continue
            options = [y for y in pool.get(keyf(x), ()) if y.idx in free_y]
            if not options:
                continue
            y = min(options, key=lambda y: near(x, y))
            free_x.discard(x.idx)
            free_y.discard(y.idx)
            if kind == "recoloured":
                events.append(("recoloured", x, y, (x.colour, y.colour)))
            elif (x.r0, x.c0) == (y.r0, y.c0):
                events.append(("same", x, y))
            else:
                events.append(("moved", x, y, (y.r0 - x.r0, y.c0 - x.c0)))

    match_pass(lambda o: (o.shape_key, o.sub.tobytes()), "exact")
    match_pass(lambda o: (o.shape_key, o.r0, o.c0), "recoloured")
    left_x = [x for x in xs if x.idx in free_x]
    left_y = [y for y in ys if y.idx in free_y]
    if len(left_x) * len(left_y) <= 40000:
        for x in left_x:
            overl = [y for y in left_y if y.idx in free_y and not (x.r1 < y.r0 or y.r1 < x.r0 or x.c1 < y.c0 or
                                                                    y.c1 < x.c0)]
            if overl:
                y = min(overl, key=lambda y: near(x, y))
                free_x.discard(x.idx)
                free_y.discard(y.idx)
                events.append(("reshaped", x, y))
    events += [("deleted", x) for x in xs if x.idx in free_x]
    events += [("created", y) for y in ys if y.idx in free_y]
    return events


def obj_diff_text(a, b, **kw) -> str:
    """Event counts of :func:`obj_diff` and up to 12 event lines."""
    ev = obj_diff(a, b, **kw)
    n = Counter(e[0] for e in ev)
    out = [", ".join(f"{k} {n[k]}" for k in _EVENT_KINDS if n[k])]
    for e in ev:
        kind = e[0]
        if kind == "moved":
            out.append(f"moved {e[1]!r} by {e[3]}")
        elif kind == "recoloured":
            out.append(f"recoloured {e[1]!r} -> {e[3][1]}")
        elif kind == "reshaped":
            out.append(f"reshaped {e[1]!r} -> {e[2]!r}")
        elif kind in ("deleted", "created"):
            out.append(f"{kind} {e[1]!r}")
    return "\n".join(out[:13])


# -------------------------------------------------------------------------------------------- size rules
def _pairs(train):
    return [(grid(p["input"]), grid(p["output"])) for p in train]


class SizeRule:
    """A rule giving the output shape from the input grid: ``kind`` names it, ``predict(g)`` -> (h, w) or None."""

    def __init__(self, kind, fn):
        self.kind, self.fn = kind, fn

    def predict(self, g):
        try:
            return self.fn(grid(g))
        except Exception:
            return None

    def __repr__(self):
        return f"SizeRule({self.kind})"


def _cell_shape(g):
    s = split_grid(g)
    if s is None:
        return None
    shapes = {c.shape for band in s["cells"] for c in band}
    return shapes.pop() if len(shapes) == 1 else None


def _object_shape(g, diag, mc, which):
    objs = objects(g, diag=diag, multicolour=mc)
    if not objs:
        return None
    if which == "largest":
        if len(objs) > 1 and objs[1].size == objs[0].size:
            return None          # no unique largest object
        return objs[0].h, objs[0].w
    return objs[-1].h, objs[-1].w


def _size_candidates(P):
    i0, o0 = P[0]
    (hi, wi), (ho, wo) = i0.shape, o0.shape
    out = [("same as input", lambda g: g.shape), ("transposed input", lambda g: g.shape[::-1])]
    shapes = {o.shape for _, o in P}
    if len(shapes) == 1:
        s = next(iter(shapes))
        out.append((f"constant {s[0]}x{s[1]}", lambda g, s=s: s))
    if ho % hi == 0 and wo % wi == 0:
        fy, fx = ho // hi, wo // wi
        out.append((f"input x{fy} rows, x{fx} cols", lambda g, a=fy, b=fx: (g.shape[0] * a, g.shape[1] * b)))
    if hi % ho == 0 and wi % wo == 0:
        fy, fx = hi // ho, wi // wo
        out.append((f"input /{fy} rows, /{fx} cols", lambda g, a=fy, b=fx: (g.shape[0] // a, g.shape[1] // b)))
    out.append(("input size squared (h*h x w*w)", lambda g: (g.shape[0] ** 2, g.shape[1] ** 2)))
    out.append(("one cell of the separator split", _cell_shape))
    out.append(("box of non-background cells", lambda g: trim(g).shape))
    for diag in (False, True):
        for mc in (False, True):
            tag = ("8" if diag else "4") + ("-multicolour" if mc else "")
            for which in ("largest", "smallest"):
                out.append((f"{which} object box ({tag})", lambda g, d=diag, m=mc, w=which: _object_shape(g, d, m, w)))
    out.append(("n_colours x n_colours", lambda g: (len(palette(g)) - 1,) * 2))
    dy, dx = ho - hi, wo - wi
    out.append((f"input {dy:+d} rows, {dx:+d} cols", lambda g, a=dy, b=dx: (g.shape[0] + a, g.shape[1] + b)))
    return out


def size_rule(train, all_rules=False):
    """The first candidate rule (in a fixed order, simplest first) that predicts every train output's shape, or
    all fitting rules with all_rules=True."""
    P = _pairs(train)
    fits = []
    for kind, fn in _size_candidates(P):
        try:
            if all(tuple(fn(i)) == o.shape for i, o in P):
                fits.append(SizeRule(kind, lambda g, f=fn: tuple(int(v) for v in f(g))))
        except Exception:
            continue
    if all_rules:
        return fits
    return fits[0] if fits else None


def color_map(train):
    """{input colour: output colour} when every train pair is a cell-wise recolouring by one map, else None."""
    m = {}
    for i, o in _pairs(train):
        if i.shape != o.shape:
            return None
        for x, y in zip(i.ravel().tolist(), o.ravel().tolist()):
            if m.setdefault(x, y) != y:
                return None
    return m


# -------------------------------------------------------------------------------------------- invariants
def _inv_defs(train):
    """(name, predicate(input, output)) pairs of candidate train-pair invariants."""
    P = _pairs(train)
    out_colours = set().union(*(set(palette(o)) for _, o in P))
    added = [set(palette(o)) - set(palette(i)) for i, o in P]
    always_added = set.intersection(*added) if added else set()
    ever_added = set().union(*added)
    in_every_output = set.intersection(*(set(palette(o)) for _, o in P))

    def kept_fg(i, o):
        b = bg(i)
        return i.shape == o.shape and np.array_equal(o[i != b], i[i != b])

    def counts_grow(i, o):
        b, ci, co = bg(i), counts(i), counts(o)
        return i.shape == o.shape and all(co.get(c, 0) >= n for c, n in ci.items() if c != b)

    def counts_shrink(i, o):
        b, ci, co = bg(i), counts(i), counts(o)
        return i.shape == o.shape and all(n <= ci.get(c, 0) for c, n in co.items() if c != b)

    defs = [
        ("output shape == input shape", lambda i, o: i.shape == o.shape),
        ("output colours subset of input colours", lambda i, o: set(palette(o)) <= set(palette(i))),
        ("output colours subset of input colours + colours added in training outputs",
         lambda i, o: set(palette(o)) <= set(palette(i)) | ever_added),
        ("output colours subset of training-output colours + input colours",
         lambda i, o: set(palette(o)) <= out_colours | set(palette(i))),
        ("output background == input background", lambda i, o: bg(o) == bg(i)),
        ("output differs from input", lambda i, o: i.shape != o.shape or not np.array_equal(i, o)),
        ("output has >= 2 colours", lambda i, o: len(palette(o)) >= 2),
        ("non-background input cells kept", kept_fg),
        ("only background cells change",
         lambda i, o: i.shape == o.shape and bool(np.all((i == o) | (i == bg(i))))),
        ("background input cells kept", lambda i, o: i.shape == o.shape and bool(np.all(o[i == bg(i)] == bg(i)))),
        ("output is a sub-grid of the input",
         lambda i, o: o.shape[0] <= i.shape[0] and o.shape[1] <= i.shape[1] and bool(find_sub(i, o, limit=1))),
        ("output colours in every training output",
         lambda i, o: set(palette(o)) <= in_every_output | set(palette(i))),
        ("colour counts never decrease", counts_grow),
        ("colour counts never increase", counts_shrink),
        ("same number of colours", lambda i, o: len(palette(o)) == len(palette(i))),
        ("same object count (4-conn)", lambda i, o: len(objects(i)) == len(objects(o, bgc=bg(i)))),
        ("output smaller than input", lambda i, o: o.size < i.size),
        ("output larger than input", lambda i, o: o.size > i.size),
    ]
    if always_added:
        defs.append((f"output contains colour(s) {sorted(always_added)}",
                     lambda i, o, need=frozenset(always_added): need <= set(palette(o))))
    for s in ("fliplr", "flipud", "transpose", "rot180", "rot90"):
        defs.append((f"output symmetric ({s})", lambda i, o, s=s: s in symmetries(o)))
    rules = size_rule(train, all_rules=True)
    if rules:
        defs.append((f"output shape follows rule: {rules[0].kind}",
                     lambda i, o, rs=tuple(rules): any(r.predict(i) == o.shape for r in rs)))
    return defs


# invariants reliable enough to warn about (name prefixes)
SAFE = ("output colours subset of training-output colours + input colours",
        "output colours subset of input colours + colours added in training outputs", "output differs from input",
        "output has >= 2 colours", "output colours in every training output", "output shape follows rule",
        "output colours subset of input colours", "output shape == input shape", "same number of colours",
        "colour counts never decrease", "colour counts never increase", "non-background input cells kept",
        "only background cells change", "output smaller than input", "output larger than input",
        "output is a sub-grid of the input")
# invariants about the output's size (test inputs may legitimately break them)
SIZE_INV = ("output shape follows rule", "output smaller than input", "output larger than input",
            "output shape == input shape", "output is a sub-grid of the input")


def invariants(train, names_only=True):
    """The candidate invariants that hold on every train pair (names, or (name, predicate) pairs)."""
    P = _pairs(train)
    held = []
    for name, f in _inv_defs(train):
        try:
            if all(bool(f(i, o)) for i, o in P):
                held.append((name, f))
        except Exception:
            continue
    return [n for n, _ in held] if names_only else held


def violations(train, test_inputs, test_outputs, safe_only=True) -> list:
    """Per test: the train invariants its output breaks (['no output'] when it has none)."""
    held = invariants(train, names_only=False)
    if safe_only:
        held = [(n, f) for n, f in held if n.startswith(SAFE)]
    res = []
    for ti, to in zip(test_inputs, test_outputs):
        if to is None:
            res.append(["no output"])
            continue
        i, o = grid(ti), grid(to)
        broken = []
        for n, f in held:
            try:
                ok = f(i, o)
            except Exception:
                ok = False
            if not ok:
                broken.append(n)
        res.append(broken)
    return res


def flag(train, test_inputs, test_outputs) -> list:
    """Sorted names of the non-size invariants broken by any test output."""
    bad = set()
    for v in violations(train, test_inputs, test_outputs):
        bad.update(n for n in v if not n.startswith(SIZE_INV))
    return sorted(bad)


# ------------------------------------------------------------------------------------- transform checks
def _params(f):
    try:
        return inspect.signature(f).parameters
    except (TypeError, ValueError):
        return {}


def _call(f, g, **kw):
    """Run a transform on a grid given as nested lists (falling back to an array) and return its output grid."""
    try:
        out = f(grid(g).tolist(), **kw)
    except Exception:
        out = f(grid(g), **kw)
    return grid(out)


def _masked(exp, got, max_cells=400) -> str:
    """The produced grid with correct cells shown as '.', for grids of at most max_cells cells."""
    if exp.size > max_cells:
        return ""
    return "\n".join("".join("." if e == x else str(int(x)) for e, x in zip(er, gr)) for er, gr in zip(exp, got))


def _pair_report(transform, i, o, kw, show_diff):
    r = {"ok": False}
    try:
        got = _call(transform, i, **kw)
        r["out"] = got
        if got.shape != o.shape:
            r["why"] = f"shape {got.shape[0]}x{got.shape[1]}, expected {o.shape[0]}x{o.shape[1]}"
        elif np.array_equal(got, o):
            r["ok"] = True
        else:
            wrong = got != o
            top = Counter(zip(o[wrong].tolist(), got[wrong].tolist())).most_common(4)
            r["why"] = (f"{int(wrong.sum())}/{o.size} cells wrong in box {bbox(wrong)}; expected->got "
                        + ", ".join(f"{a}->{b}:{n}" for (a, b), n in top))
            if show_diff:
                r["masked"] = _masked(o, got)
    except Exception as e:
        r["why"] = f"raised {type(e).__name__}: {str(e)[:150]}"
    return r


def _test_notes(t, g, out, P, rules, broken, eq):
    """Warnings for one test output: strong (non-size invariants broken), soft (size checks), notes."""
    strong = [v for v in broken if v != "no output" and not v.startswith(SIZE_INV)]
    soft = [v for v in broken if v.startswith(SIZE_INV)]
    notes = []
    if out is not None:
        pred = [r.predict(g) for r in rules]
        if pred and out.shape not in pred and None not in pred:
            soft = [v for v in soft if not v.startswith("output shape follows")]
            soft.insert(0, f"shape {out.shape[0]}x{out.shape[1]} but the training size rule '{rules[0].kind}' "
                           f"predicts {pred[0][0]}x{pred[0][1]}")
        distinct_outputs = len({o.tobytes() for _, o in P}) == len(P)
        if distinct_outputs and any(np.array_equal(out, o) for _, o in P):
            soft.append("output equals a training output")
        if eq and eq[t]:
            notes.append("transform is equivariant under " + ", ".join(eq[t])
                         + " on every training pair but not on this test input")
    return strong, soft, notes


def check(transform, train, test_inputs=None, verbose=True, show_diff=True, equiv=True) -> dict:
    """Run `transform` on every train input and report. A transform with a ``train`` parameter receives the
    train pairs, and is also run leave-one-out (each pair predicted from the others). With test inputs, their
    outputs are checked against the train invariants, the size rule and (when every pair passes) the
    transform's own equivariances. Returns {'pairs', 'tests', 'loo', 'text', 'ok'}; verbose prints the text."""
    P = _pairs(train)
    takes_train = "train" in _params(transform)
    kw = {"train": train} if takes_train else {}
    rep = {"pairs": [], "tests": [], "loo": None}
    lines = []
    for k, (i, o) in enumerate(P):
        r = _pair_report(transform, i, o, kw, show_diff)
        rep["pairs"].append(r)
        lines.append(f"pair {k}: " + ("ok" if r["ok"] else r["why"]))
        if r.get("masked") and sum(not x["ok"] for x in rep["pairs"]) <= 2:
            lines.append(r["masked"])
    n_ok = sum(r["ok"] for r in rep["pairs"])
    lines.insert(0, f"check: {n_ok}/{len(P)} training pairs correct")
    if takes_train and len(P) > 1:
        loo = []
        for k, (i, o) in enumerate(P):
            others = [p for j, p in enumerate(train) if j != k]
            try:
                loo.append(bool(np.array_equal(_call(transform, i, train=others), o)))
            except Exception:
                loo.append(False)
        rep["loo"] = loo
        lines.append(f"leave-one-out: {sum(loo)}/{len(loo)} pairs reproduced from the other pairs "
                     + str(["ok" if x else "FAIL" for x in loo]))
    if test_inputs:
        outs = []
        for t, g in enumerate(test_inputs):
            try:
                outs.append(_call(transform, g, **kw))
            except Exception as e:
                outs.append(None)
                lines.append(f"test {t}: raised {type(e).__name__}: {str(e)[:150]}")
        rules = size_rule(train, all_rules=True)
        broken = violations(train, test_inputs, outs)
        eq = equivariance(transform, train, test_inputs, outs) if equiv and n_ok == len(P) else None
        for t, (g, out) in enumerate(zip(test_inputs, outs)):
            strong, soft, notes = _test_notes(t, g, out, P, rules, broken[t], eq)
            rep["tests"].append({"out": out, "warnings": strong, "soft": soft, "notes": notes})
            if out is None:
                continue
            txt = f"test {t}: output {out.shape[0]}x{out.shape[1]}"
            if strong:
                txt += "; WARNING (every training pair satisfies this, the test output does not): " + "; ".join(strong)
            if soft:
                txt += "; size check (test inputs may legitimately differ): " + "; ".join(soft)
            if notes:
                txt += "; note (weak signal): " + "; ".join(notes)
            if not (strong or soft or notes):
                txt += "; no warnings"
            lines.append(txt)
    rep["text"] = "\n".join(lines)
    rep["ok"] = n_ok == len(P)
    if verbose:
        print(rep["text"])
    return rep


# colour permutations of 1..9 (0 fixed) used as equivariance probes
_COLOUR_PERMS = ((1, 2, 3, 4, 5, 6, 7, 8, 9), (2, 3, 4, 5, 6, 7, 8, 9, 1), (5, 6, 7, 8, 9, 1, 2, 3, 4),
                 (9, 8, 7, 6, 5, 4, 3, 2, 1))


def _colour_perm(k):
    table = np.arange(10)
    table[1:] = _COLOUR_PERMS[k]
    return lambda g: table[grid(g)]


def equivariance(transform, train, test_inputs, test_outputs=None, budget_s=2.0) -> list:
    """Per test input: the maps (non-identity dihedral maps, then three colour permutations) under which the
    transform commutes on every train pair but not on that test input, a hint that the test output is off.
    Stops trying maps after budget_s seconds."""
    t0 = time.time()
    P = _pairs(train)
    kw = {"train": train} if "train" in _params(transform) else {}
    maps = [(k, lambda g, k=k: d8(g, k)) for k in D8[1:]] + [(f"colour perm {k}", _colour_perm(k)) for k in (1, 2, 3)]
    if test_outputs is None:
        test_outputs = []
        for g in test_inputs:
            try:
                test_outputs.append(_call(transform, g, **kw))
            except Exception:
                test_outputs.append(None)
    res = [[] for _ in test_inputs]
    for name, m in maps:
        if time.time() - t0 > budget_s:
            break
        try:
            if not all(np.array_equal(_call(transform, m(i), **kw), m(o)) for i, o in P):
                continue
        except Exception:
            continue
        for t, (g, out) in enumerate(zip(test_inputs, test_outputs)):
            if out is None:
                continue
            try:
                holds = np.array_equal(_call(transform, m(g), **kw), m(out))
            except Exception:
                holds = False
            if not holds:
                res[t].append(name)
    return res


# ---------------------------------------------------------------------------------------------- physics
_TURNS = {"down": 0, "left": 1, "up": 2, "right": 3}


def gravity(g, direction="down", rigid=False, bgc=None, diag=False):
    """Let cells fall towards `direction`. Default: every column settles independently (cells keep their
    order); rigid=True: whole objects fall, lowest first, until blocked by the edge or another cell."""
    g = grid(g)
    b = bg(g) if bgc is None else bgc
    k = _TURNS[direction]
    r = np.rot90(g, k).copy()          # the fall direction is now "down"
    H, W = r.shape
    if not rigid:
        out = np.full_like(r, b)
        for j in range(W):
            col = r[:, j][r[:, j] != b]
            if col.size:
                out[H - col.size:, j] = col
        return np.rot90(out, -k).copy()
    for o in sorted(objects(r, b, diag=diag), key=lambda o: -o.r1):
        cells = list(o.cells)
        vals = [r[y, x] for y, x in cells]
        own = set(cells)
        drop = 0
        while all(y + drop + 1 < H and ((y + drop + 1, x) in own or r[y + drop + 1, x] == b) for y, x in cells):
            drop += 1
        if drop:
            for y, x in cells:
                r[y, x] = b
            for (y, x), v in zip(cells, vals):
                r[y + drop, x] = v
    return np.rot90(r, -k).copy()


# ---------------------------------------------------------------------------------------------- summary
def _pair_line(k, i, o, b):
    d = diff(i, o)
    text = f"pair {k}: {i.shape[0]}x{i.shape[1]} -> {o.shape[0]}x{o.shape[1]}; {d['text']}"
    objs = objects(i, b)
    text += f"; input objects {len(objs)}"
    if d["same_shape"] and d["n_changed"]:
        n = Counter(e[0] for e in obj_diff(i, o, b))
        text += " (" + ", ".join(f"{x} {n[x]}" for x in _EVENT_KINDS if n[x]) + ")"
    s = split_grid(i)
    if s:
        text += f"; separators colour {s['colour']} -> {len(s['boxes'])}x{len(s['boxes'][0])} cells"
    p = period(i)
    if p != i.shape:
        text += f"; input period {p}"
    sy = symmetries(o)
    if sy:
        text += f"; output symmetric {sy}"
    return text, objs


def describe(train, test_inputs=(), max_obj=4, budget=1800) -> str:
    """A text overview of a task for the model: background, size rule, colour map, one line per train pair
    (diff, objects, separators, period, symmetry), the objects of the first input, the invariants that hold on
    every pair and a line per test input; cut to `budget` characters."""
    P = _pairs(train)
    sr = size_rule(train)
    cm = color_map(train)
    b = task_bg(train)
    head = f"{len(P)} train pairs; task background {b}; output size rule: {sr.kind if sr else 'none found'}"
    if cm and any(k != v for k, v in cm.items()):
        head += f"; consistent cell colour map {cm}"
    out = [head]
    for k, (i, o) in enumerate(P):
        text, objs = _pair_line(k, i, o, b)
        out.append(text)
        if k == 0 and objs:
            shown = "; ".join(repr(x)[4:-1] for x in objs[:max_obj])
            more = f"; +{len(objs) - max_obj} more" if len(objs) > max_obj else ""
            out.append("  objects of pair 0 input: " + shown + more)
    inv = [n for n in invariants(train) if not n.startswith("output shape follows")]
    if "output colours subset of input colours" in inv:   # the weaker colour statements add nothing then
        inv = [n for n in inv if not n.startswith(("output colours subset of input colours +",
                                                   "output colours subset of training-output"))]
    if inv:
        out.append("holds on all pairs: " + "; ".join(inv[:10]))
    seen_colours = set().union(*(set(palette(i)) for i, _ in P))
    for t, g in enumerate(test_inputs):
        g = grid(g)
        extra = []
        unseen = set(palette(g)) - seen_colours
        if unseen:
            extra.append(f"unseen colours {sorted(unseen)}")
        if sr is not None:
            extra.append(f"predicted output size {sr.predict(g)}")
        line_ = f"test {t}: {g.shape[0]}x{g.shape[1]}, {len(objects(g, b))} objects"
        out.append(line_ + (f"; {'; '.join(extra)}" if extra else ""))
    txt = "\n".join(out)
    if len(txt) > budget:
        txt = txt[:budget - 20].rsplit("\n", 1)[0] + "\n[... truncated]"
    return txt


HELP = """\
`ak` (arckit) is already imported; it needs only numpy (no scipy: label with ak.objects, fill holes with
ak.enclosed). Pass grids as lists or arrays; every function returns a new numpy int array (use .tolist()).
Coordinates are (row, col); boxes are (r0, c0, r1, c1) with both ends included.
 ak.describe(train, test_inputs) -> str     overview: size rule, per-pair diffs, objects, invariants
 ak.check(transform, train, test_inputs)    per-pair results and warnings about the test outputs; a
     transform(grid, train=None) signature also gets a leave-one-out run
 ak.objects(g, bgc=None, diag=False, multicolour=False) -> [Obj], largest first; an Obj has colour colours
     size box r0 c0 r1 c1 h w cells mask sub shape_key holes border rect sym center slice
 ak.diff(a, b)                              changed cells, (from, to) counts, box, or how the shape changed
 ak.obj_diff(a, b) -> [(kind, obj_a, obj_b, ...)], kind in same moved recoloured reshaped deleted created
 ak.bg(g) ak.task_bg(train) ak.palette(g) ak.counts(g) ak.bbox(mask) ak.crop(g, box) ak.trim(g)
 ak.d8(g) -> {name: grid} for id rot90 rot180 rot270 flipud fliplr transpose antitranspose; ak.d8(g, name)
 ak.scale(g, k) ak.downscale(g, k) ak.tile(g, ny, nx) ak.paste(dst, src, r, c, skip=None)
 ak.find_sub(big, small, wildcard=None) -> [(r, c)]   ak.flood(g, r, c, colour)   ak.enclosed(g) -> mask
 ak.line(g, r0, c0, r1, c1, colour)   ak.ray(g, r, c, dr, dc, colour, stop=None)   ak.move(g, obj, dr, dc)
 ak.gravity(g, 'down'|'up'|'left'|'right', rigid=False)   rigid=True moves whole objects until blocked
 ak.show(g, coords=True) -> str with row and column indices
 ak.split_grid(g) -> {rows cols colour boxes cells} for full separator lines, or None
 ak.period(g, ignore=None) -> (pr, pc)   ak.repair_period(g, ignore)   ak.symmetries(g, ignore=None)
 ak.complete_symmetry(g, ignore)   ak.size_rule(train).predict(g)   ak.color_map(train)   ak.invariants(train)"""


def help():
    print(HELP)

"""Pre-flight checks before serving a build (the reference runs fn_preflight.py before its Kaggle launcher:
flashnext/kaggle/code_dataset/fn_preflight.py; delta manifests, router/expert agreement, keep layout).

Checks, each recorded as (name, ok, detail):

* every delta directory matches its ``manifest.json`` (sizes and md5);
* for the first and the last expert layer: the low-bit layer loads with the delta scales applied
  (``deltas.build`` semantics), its router has one row per kept expert, every expert's bit width is 2, 3 or 4;
* ``keep.json`` (the last delta's, else the base's) has one entry per layer and the same count in every layer;
* runtime: the native extension loads; on a GPU, compute capability 10.x (sm_100a kernels) and the free device
  memory against the build's weight bytes.

    python -m arcagi2_flashnext_dots3_b200.launch.preflight BUILD [DELTA ...] [--no-gpu]
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import torch


def check_build(base, deltas=()) -> list:
    from ..formats import deltas as D
    from ..formats import lowbit_file
    out = []
    for d in deltas:
        try:
            D.verify_manifest(d)
            out.append(("manifest " + os.path.basename(str(d)), True, "md5 ok"))
        except Exception as e:
            out.append(("manifest " + os.path.basename(str(d)), False, str(e)))
    layers = lowbit_file.list_layers(base)
    if not layers:
        out.append(("layers", False, f"no lowbit-LNN.pt in {base}"))
        return out
    for l in sorted({layers[0], layers[-1]}):
        try:
            lay = lowbit_file.load_layer(base, l, mmap=True)
            n = len(lay.experts)
            for d in deltas:                       # later deltas override earlier ones
                sp = Path(d) / f"scales-L{l:02d}.pt"
                if sp.exists():
                    sc = torch.load(sp, map_location="cpu", weights_only=False)
                    if set(sc) - set(lay.experts):
                        raise ValueError(f"delta {d} has experts not in the layer")
                rp = Path(d) / f"router-L{l:02d}.pt"
                if rp.exists():
                    r = torch.load(rp, map_location="cpu", weights_only=False)
                    w = r["weight"] if isinstance(r, dict) else r
                    if w.shape[0] != n:
                        raise ValueError(f"router rows {w.shape[0]} != experts {n}")
            if lay.router.shape[0] != n:
                raise ValueError(f"router rows {lay.router.shape[0]} != experts {n}")
            bad = [b.bits for b in lay.blobs if b.bits not in (2, 3, 4)]
            if bad:
                raise ValueError(f"unsupported bit widths {sorted(set(bad))}")
            out.append((f"layer {l}", True, f"{n} experts"))
        except Exception as e:
            out.append((f"layer {l}", False, str(e)))
    keep = next((Path(d) / "keep.json" for d in reversed(list(deltas)) if (Path(d) / "keep.json").exists()),
                Path(base) / "keep.json")
    if keep.exists():
        k = json.load(open(keep))
        rows = k.get("keep", k) if isinstance(k, dict) else k
        sizes = {len(v) for v in (rows.values() if isinstance(rows, dict) else rows)}
        ok = len(rows) == len(layers) and len(sizes) == 1
        out.append(("keep.json", ok, f"{len(rows)} layers, K={sorted(sizes)} from {keep.parent.name}"))
    return out


def check_runtime(weight_bytes: int = 0, gpu: bool = True) -> list:
    out = []
    try:
        from ..ops import native
        native.C()
        out.append(("extension", True, "_C loaded"))
    except Exception as e:
        out.append(("extension", False, repr(e)[:200]))
    if gpu:
        if not torch.cuda.is_available():
            out.append(("gpu", False, "no CUDA device"))
            return out
        cc = torch.cuda.get_device_capability()
        out.append(("gpu arch", cc[0] == 10, f"sm_{cc[0]}{cc[1]} {torch.cuda.get_device_name()}"))
        free, total = torch.cuda.mem_get_info()
        out.append(("gpu memory", free > weight_bytes, f"{free / 2**30:.1f} GiB free of {total / 2**30:.1f}, "
                                                       f"weights {weight_bytes / 2**30:.1f} GiB"))
    return out


def build_bytes(base) -> int:
    return sum(p.stat().st_size for p in Path(base).glob("*.pt"))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("build")
    ap.add_argument("deltas", nargs="*")
    ap.add_argument("--no-gpu", action="store_true")
    a = ap.parse_args(argv)
    res = check_build(a.build, a.deltas) + check_runtime(build_bytes(a.build), gpu=not a.no_gpu)
    for name, ok, detail in res:
        print(f"{'ok ' if ok else 'FAIL'} {name}: {detail}")
    if not all(ok for _, ok, _ in res):
        raise SystemExit("PREFLIGHT FAILED")
    print(f"PREFLIGHT OK: {len(a.deltas)} delta(s)")
    return res


if __name__ == "__main__":
    main()

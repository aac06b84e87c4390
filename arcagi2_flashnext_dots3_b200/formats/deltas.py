"""Repair-training deltas over a base low-bit build (L0).

Two delta formats exist, both kept file-compatible with the reference:

* **FN delta directory** (flashnext/kaggle/code_dataset/delta_build.py:12-79): ``scales-LNN.pt`` =
  ``{expert_id: {"gu_s", "d_s"}}`` (fp16 scales), ``router-LNN.pt``, ``keep.json``, optional extra files and a
  ``manifest.json`` of ``{name: {"bytes", "md5"}}``. :func:`make` extracts a delta from a derived build,
  :func:`build` rebuilds a full build from base + deltas (manifest-verified), :func:`verify_build` compares two
  builds (byte-identical, or identical content digests).
* **D3 ulp overlay** (dotsnote/engine/arcstats_pkg/arcstats/delta_overlay.py:1-20): one safetensors file with, per
  layer, ``lowbit.LNN.experts`` (int64 ids), ``lowbit.LNN.gu_s`` / ``.d_s`` (int8 or int16 differences of the fp16
  scale bit patterns, in ulp steps), ``lowbit.LNN.base_ck`` (checksum of the base scale bits; a different base is
  refused) and ``dense.<name>`` replacement tensors.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
from dataclasses import dataclass, field
from pathlib import Path

import torch


# ----------------------------------------------------------------------------------------------- FN deltas
def md5(path) -> str:
    h = hashlib.md5()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(64 << 20), b""):
            h.update(blk)
    return h.hexdigest()


def write_manifest(delta_dir):
    """manifest.json with size and md5 of every file in the delta directory."""
    delta_dir = Path(delta_dir)
    man = {}
    for n in sorted(os.listdir(delta_dir)):
        p = delta_dir / n
        if n == "manifest.json" or not p.is_file():
            continue
        man[n] = {"bytes": p.stat().st_size, "md5": md5(p)}
    with open(delta_dir / "manifest.json", "w") as f:
        json.dump(man, f, indent=1, sort_keys=True)
    return man


def verify_manifest(delta_dir):
    mp = Path(delta_dir) / "manifest.json"
    if not mp.exists():
        return True
    for n, v in json.load(open(mp)).items():
        if n.startswith("_") or not isinstance(v, dict):
            continue
        p = Path(delta_dir) / n
        if not p.exists() or p.stat().st_size != v["bytes"] or md5(p) != v["md5"]:
            raise ValueError(f"{p}: does not match manifest.json")
    return True


def _layers(d):
    return sorted(int(m.group(1)) for n in os.listdir(d) if (m := re.match(r"^lowbit-L(\d+)\.pt$", n)))


def make(base_dir, derived_dir, out_dir):
    """Extract the scale/router delta of a derived build into out_dir (plus a manifest)."""
    os.makedirs(out_dir, exist_ok=True)
    for l in _layers(derived_dir):
        d = torch.load(f"{derived_dir}/lowbit-L{l:02d}.pt", map_location="cpu", weights_only=False)
        sc = {e: {"gu_s": d[e]["gu_s"].clone(), "d_s": d[e]["d_s"].clone()} for e in d["experts"]}
        torch.save(sc, f"{out_dir}/scales-L{l:02d}.pt")
        shutil.copy2(f"{derived_dir}/router-L{l:02d}.pt", f"{out_dir}/router-L{l:02d}.pt")
    if os.path.exists(f"{derived_dir}/keep.json"):
        shutil.copy2(f"{derived_dir}/keep.json", f"{out_dir}/keep.json")
    write_manifest(out_dir)


def build(base_dir, deltas, out_dir):
    """Rebuild a full build from base + a list of deltas (later deltas win)."""
    if not deltas:
        raise ValueError("need at least one delta dir")
    os.makedirs(out_dir, exist_ok=True)
    for d in deltas:
        verify_manifest(d)
    for l in _layers(base_dir):
        b = torch.load(f"{base_dir}/lowbit-L{l:02d}.pt", map_location="cpu", weights_only=False)
        router = f"{base_dir}/router-L{l:02d}.pt"
        for d in deltas:
            sp = f"{d}/scales-L{l:02d}.pt"
            if os.path.exists(sp):
                sc = torch.load(sp, map_location="cpu", weights_only=False)
                if list(sc) != list(b["experts"]):
                    raise ValueError(f"L{l}: expert ids differ between base and delta {d}")
                for e, v in sc.items():
                    b[e]["gu_s"], b[e]["d_s"] = v["gu_s"], v["d_s"]
            if os.path.exists(f"{d}/router-L{l:02d}.pt"):
                router = f"{d}/router-L{l:02d}.pt"
        torch.save(b, f"{out_dir}/lowbit-L{l:02d}.pt")
        shutil.copy2(router, f"{out_dir}/router-L{l:02d}.pt")
    keep = next((f"{d}/keep.json" for d in reversed(deltas) if os.path.exists(f"{d}/keep.json")),
                f"{base_dir}/keep.json")
    if os.path.exists(keep):
        shutil.copy2(keep, f"{out_dir}/keep.json")
    skip = re.compile(r"^(scales|router|lowbit)-L\d+\.pt$|^(keep\.json|manifest\.json|LICENSE)$")
    for d in deltas:
        for n in sorted(os.listdir(d)):
            if not skip.match(n) and os.path.isfile(f"{d}/{n}"):
                shutil.copy2(f"{d}/{n}", f"{out_dir}/{n}")


def content_digest(obj) -> str:
    """SHA-256 of a loaded checkpoint tree's content, independent of how the pickle was written: containers
    contribute their type, length and (for dicts, in insertion order) their keys; tensors their dtype, shape and
    raw bytes; other leaves their repr. Two trees with equal digests hold the same keys and bit-identical
    tensors."""
    h = hashlib.sha256()
    stack = [obj]
    while stack:
        x = stack.pop()
        if torch.is_tensor(x):
            t = x.detach().cpu().contiguous()
            h.update(f"T{t.dtype}{tuple(t.shape)}".encode())
            h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
        elif isinstance(x, dict):
            h.update(f"D{len(x)}".encode())
            for k in x:
                h.update(("K" + repr(k)).encode())
            stack.extend(reversed(list(x.values())))
        elif isinstance(x, (list, tuple)):
            h.update(f"{type(x).__name__[0]}{len(x)}".encode())
            stack.extend(reversed(list(x)))
        else:
            h.update(("V" + repr(x)).encode())
    return h.hexdigest()


@dataclass
class BuildDiff:
    """Result of :func:`verify_build`: files byte-identical, files whose loaded contents are identical though
    their bytes differ (a re-pickled but equal tensor tree), and files that differ or are missing."""
    identical: list = field(default_factory=list)
    same_content: list = field(default_factory=list)
    differ: list = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.differ


def _build_files(d) -> list:
    layers = _layers(d)
    names = [f"{kind}-L{l:02d}.pt" for kind in ("lowbit", "router") for l in layers]
    return names + (["keep.json"] if os.path.exists(f"{d}/keep.json") else [])


def verify_build(rebuilt_dir, derived_dir) -> BuildDiff:
    """Check that a build rebuilt from base + deltas reproduces the derived build it was extracted from (the
    reference's delta_build.py `check` step): every low-bit layer, router and keep file of the derived build must
    be byte-identical in the rebuilt one, or, for .pt files, identical in content (:func:`content_digest`)."""
    res = BuildDiff()
    for name in _build_files(derived_dir):
        a, b = Path(rebuilt_dir) / name, Path(derived_dir) / name
        if not a.exists():
            res.differ.append(name)
        elif a.stat().st_size == b.stat().st_size and md5(a) == md5(b):
            res.identical.append(name)
        elif name.endswith(".pt") and content_digest(torch.load(a, map_location="cpu", weights_only=False)) == \
                content_digest(torch.load(b, map_location="cpu", weights_only=False)):
            res.same_content.append(name)
        else:
            res.differ.append(name)
    return res


# ------------------------------------------------------------------------------------------ D3 ulp overlay
def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16).to(torch.int32)


def checksum(t: torch.Tensor) -> int:
    """Position-weighted sum of fp16 bit patterns; identifies the base scales an overlay was made against."""
    b = _bits(t).to(torch.int64)
    w = torch.arange(t.numel(), dtype=torch.int64).view(t.shape) % 9973 + 1
    return int((b * w).sum())


def make_ulp_overlay(base_layers: dict, new_layers: dict, dense: dict | None = None) -> dict:
    """Tensors of an ulp overlay. ``*_layers`` map layer index -> lowbit dict ({"experts", id: {...}})."""
    out = {}
    for l, base in base_layers.items():
        new = new_layers[l]
        ids = list(base["experts"])
        if list(new["experts"]) != ids:
            raise ValueError(f"layer {l}: expert order differs")
        k = f"lowbit.L{l:02d}."
        out[k + "experts"] = torch.tensor(ids, dtype=torch.int64)
        cks = []
        for nm in ("gu_s", "d_s"):
            b0 = torch.stack([base[e][nm] for e in ids])
            b1 = torch.stack([new[e][nm] for e in ids])
            diff = _bits(b1) - _bits(b0)
            dt = torch.int8 if int(diff.abs().max()) < 128 else torch.int16
            out[k + nm] = diff.to(dt)
            cks.append(checksum(b0))
        out[k + "base_ck"] = torch.tensor(cks, dtype=torch.int64)
    for n, t in (dense or {}).items():
        out["dense." + n] = t.contiguous()
    return out


def apply_ulp_overlay(overlay: dict, layer_idx: int, d: dict) -> bool:
    """Patch a loaded lowbit dict's scales in place; False if the overlay has no entry for this layer."""
    k = f"lowbit.L{layer_idx:02d}."
    if k + "experts" not in overlay:
        return False
    ids = overlay[k + "experts"].tolist()
    if ids != list(d["experts"]):
        raise ValueError(f"ulp overlay: expert order mismatch in layer {layer_idx}")
    gu0 = torch.stack([d[e]["gu_s"] for e in ids])
    dn0 = torch.stack([d[e]["d_s"] for e in ids])
    if [checksum(gu0), checksum(dn0)] != overlay[k + "base_ck"].tolist():
        raise ValueError(f"ulp overlay: base checkpoint mismatch in layer {layer_idx}")
    for nm, base in (("gu_s", gu0), ("d_s", dn0)):
        new = (_bits(base) + overlay[k + nm].to(torch.int32)).to(torch.int16).view(torch.float16)
        for i, e in enumerate(ids):
            d[e][nm] = new[i].clone()
    return True


def dense_replacements(overlay: dict) -> dict:
    return {n[len("dense."):]: t for n, t in overlay.items() if n.startswith("dense.")}


def save_overlay(path, tensors: dict):
    from safetensors.torch import save_file
    save_file(tensors, str(path))


def load_overlay(path) -> dict:
    from safetensors.torch import load_file
    return load_file(str(path))

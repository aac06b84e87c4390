"""Checkpoint files of a low-bit build (L0): ``lowbit-LNN.pt``, ``router-LNN.pt``, ``keep.json``.

File contents follow the reference so existing builds load unchanged:

* ``lowbit-LNN.pt`` = ``{"experts": [kept original ids ascending], id: {"bits", "gu", "gu_s", "gu_z", "d", "d_s",
  "d_z"}}`` where ``gu``/``d`` are planar plane dicts (``p4`` or ``p2``[+``p1``]), ``gu`` rows are [gate I; up I]
  and w = fp16 s * (q - z) (flashnext/training/prune_gptq/mkreadme.py:13; dotsnote/training/README.md:218-224).
* ``router-LNN.pt`` = ``{"weight": bf16 [K_kept, H] router rows in kept order, "keep": ids}``.
* ``keep.json`` = ``{"keep": [[bool]*E_orig for each layer], ...}`` (one row per layer incl. the MTP layer).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path

import torch

from .planar import G, dequant, pack_planar, quantize_rtn


@dataclass
class ExpertBlob:
    """One expert's packed gate_up and down projections."""
    bits: int
    gu: dict
    gu_s: torch.Tensor
    gu_z: torch.Tensor
    d: dict
    d_s: torch.Tensor
    d_z: torch.Tensor

    def to_dict(self) -> dict:
        return {"bits": self.bits, "gu": self.gu, "gu_s": self.gu_s, "gu_z": self.gu_z,
                "d": self.d, "d_s": self.d_s, "d_z": self.d_z}

    @staticmethod
    def from_dict(d: dict) -> "ExpertBlob":
        return ExpertBlob(int(d["bits"]), d["gu"], d["gu_s"], d["gu_z"], d["d"], d["d_s"], d["d_z"])

    def dense(self, dtype=torch.float32):
        """(W_gu [2I, H], W_d [H, I]) dequantized."""
        return (dequant(self.gu, self.bits, self.gu_s, self.gu_z, dtype),
                dequant(self.d, self.bits, self.d_s, self.d_z, dtype))


@dataclass
class LowbitLayer:
    """All kept experts of one MoE layer plus its router rows (kept order)."""
    experts: list
    blobs: list
    router: torch.Tensor  # [E_kept, H]
    keep: list = field(default_factory=list)

    @property
    def n_experts(self):
        return len(self.experts)


def quantize_expert(w_gu: torch.Tensor, w_d: torch.Tensor, bits: int, symmetric=False, clip_search=0) -> ExpertBlob:
    """RTN-quantize one expert's dense weights into an :class:`ExpertBlob`."""
    q, s, z = quantize_rtn(w_gu, bits, symmetric, clip_search)
    qd, sd, zd = quantize_rtn(w_d, bits, symmetric, clip_search)
    return ExpertBlob(bits, pack_planar(q, bits), s, z, pack_planar(qd, bits), sd, zd)


def random_layer(n_experts: int, hidden: int, inter: int, bits, gen: torch.Generator, std=0.02,
                 symmetric=False, n_orig=None, device="cpu") -> LowbitLayer:
    """Random-init low-bit layer: dense N(0, std) weights quantized per expert (bits may be an int or a list)."""
    if isinstance(bits, int):
        bits = [bits] * n_experts
    blobs = []
    for e in range(n_experts):
        wgu = torch.randn(2 * inter, hidden, generator=gen) * std
        wd = torch.randn(hidden, inter, generator=gen) * std
        blobs.append(quantize_expert(wgu, wd, bits[e], symmetric))
    router = (torch.randn(n_experts, hidden, generator=gen) * std).to(torch.bfloat16)
    n_orig = n_orig or n_experts
    experts = sorted(torch.randperm(n_orig, generator=gen)[:n_experts].tolist()) if n_orig > n_experts \
        else list(range(n_experts))
    keep = [False] * n_orig
    for e in experts:
        keep[e] = True
    return LowbitLayer(experts, blobs, router, keep)


def save_layer(build_dir, layer_idx: int, layer: LowbitLayer):
    build_dir = Path(build_dir)
    build_dir.mkdir(parents=True, exist_ok=True)
    d = {"experts": list(layer.experts)}
    for e, b in zip(layer.experts, layer.blobs):
        d[e] = b.to_dict()
    torch.save(d, build_dir / f"lowbit-L{layer_idx:02d}.pt")
    torch.save({"weight": layer.router.to(torch.bfloat16), "keep": list(layer.experts)},
               build_dir / f"router-L{layer_idx:02d}.pt")


def load_layer(build_dir, layer_idx: int, mmap: bool = False) -> LowbitLayer:
    build_dir = Path(build_dir)
    kw = {"map_location": "cpu", "weights_only": False}
    if mmap:
        kw["mmap"] = True
    d = torch.load(build_dir / f"lowbit-L{layer_idx:02d}.pt", **kw)
    r = torch.load(build_dir / f"router-L{layer_idx:02d}.pt", **kw)
    experts = list(d["experts"])
    blobs = [ExpertBlob.from_dict(d[e]) for e in experts]
    router = r["weight"]
    if router.shape[0] != len(experts):
        raise ValueError(f"router-L{layer_idx:02d}: {router.shape[0]} rows for {len(experts)} kept experts")
    return LowbitLayer(experts, blobs, router, list(r.get("keep", experts)))


def save_keep(build_dir, keep_rows, src: str = "", weighted: bool = True, tiers: str = ""):
    """keep.json: one boolean row per layer (kept experts)."""
    Path(build_dir).mkdir(parents=True, exist_ok=True)
    with open(Path(build_dir) / "keep.json", "w") as f:
        json.dump({"keep": [[bool(x) for x in row] for row in keep_rows], "src": src, "weighted": weighted,
                   "tiers": tiers}, f)


def load_keep(build_dir):
    with open(Path(build_dir) / "keep.json") as f:
        return json.load(f)


def layer_bytes(layer: LowbitLayer) -> int:
    """Streamed bytes of a layer's experts (planes + scales + zeros)."""
    n = 0
    for b in layer.blobs:
        for p in (b.gu, b.d):
            n += sum(t.numel() * t.element_size() for t in p.values())
        n += sum(t.numel() * t.element_size() for t in (b.gu_s, b.gu_z, b.d_s, b.d_z))
    return n


def list_layers(build_dir):
    out = []
    for n in sorted(os.listdir(build_dir)):
        if n.startswith("lowbit-L") and n.endswith(".pt"):
            out.append(int(n[len("lowbit-L"):-3]))
    return out


__all__ = ["G", "ExpertBlob", "LowbitLayer", "quantize_expert", "random_layer", "save_layer", "load_layer",
           "save_keep", "load_keep", "layer_bytes", "list_layers"]

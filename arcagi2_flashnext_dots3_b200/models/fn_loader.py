"""Build directories of the FN-shaped model: low-bit experts per layer plus the dense (non-expert) weights.

Layout (the reference's build layout, flashnext/kaggle/README.md:28-30, with the FP8 base checkpoint's dense
tensors collected into one file): ``lowbit-LNN.pt`` and ``router-LNN.pt`` per MoE layer (:mod:`..formats.lowbit_file`),
``keep.json``, and ``dense.pt`` = {"config": FNConfig fields, "W": the dense weight dict of
:func:`.fn_weights.random_dense` without the expert entries}.
"""
from __future__ import annotations

import dataclasses
from pathlib import Path

import torch

from ..config import FNConfig
from ..formats import lowbit_file

_EXPERT_KEYS = ("lowbit", "experts_dense", "gate")


def save_build(W: dict, cfg, build_dir) -> Path:
    d = Path(build_dir)
    d.mkdir(parents=True, exist_ok=True)
    dense = {k: v for k, v in W.items() if k != "layers"}
    dense["layers"] = []
    for l, L in enumerate(W["layers"]):
        L2 = {k: v for k, v in L.items() if k != "moe"}
        L2["moe"] = {k: v for k, v in L["moe"].items() if k not in _EXPERT_KEYS}
        dense["layers"].append(L2)
        lowbit_file.save_layer(d, l, L["moe"]["lowbit"])
    torch.save({"config": dataclasses.asdict(cfg), "W": dense}, d / "dense.pt")
    lowbit_file.save_keep(d, [[True] * L["moe"]["lowbit"].n_experts for L in W["layers"]], src="save_build")
    return d


def expert_layers(build_dir, layers: int | None = None) -> list:
    n = len(lowbit_file.list_layers(build_dir))
    return [lowbit_file.load_layer(build_dir, l) for l in range(n if layers is None else min(n, layers))]


def load_dense_build(build_dir, layers: int | None = None):
    """(cfg, W) with W in the layout of :func:`.fn_weights.random_dense` (experts as LowbitLayer objects)."""
    d = torch.load(Path(build_dir) / "dense.pt", map_location="cpu", weights_only=False)
    fields = {f.name for f in dataclasses.fields(FNConfig)}
    cfgd = {k: (tuple(v) if isinstance(v, list) else v) for k, v in d["config"].items() if k in fields}
    if layers:
        cfgd["num_layers"] = layers
    cfg = FNConfig(**cfgd)
    W = d["W"]
    W["layers"] = W["layers"][: cfg.num_layers]
    for l, lay in enumerate(expert_layers(build_dir, cfg.num_layers)):
        m = W["layers"][l]["moe"]
        m["lowbit"] = lay
        m["gate"] = lay.router.float()
    return cfg, W

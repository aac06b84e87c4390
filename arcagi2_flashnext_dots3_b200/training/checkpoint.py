"""Training checkpoints and delta export.

* :func:`save` / :func:`load`: trainable parameters (`trained.pt`, rank 0), each rank's optimizer shard
  (`opt-rank{r}.pt`) and the step/RNG state, written to a temporary name and renamed so an interrupted save
  never leaves a truncated file (the reference resumes from `trained.pt`, flashnext/training/rl/train_rl.py:53).
* :func:`export_delta`: the FN delta directory (`scales-LNN.pt` {expert id: {"gu_s", "d_s"}} fp16,
  `router-LNN.pt` {"weight", "keep"}, `keep.json`, `manifest.json`), the format the reference's export and
  `delta_build.py` produce (flashnext/training/student/export_build.py; flashnext/kaggle/code_dataset/
  delta_build.py:12-79), so :func:`..formats.deltas.build` rebuilds a servable build from base + delta.
"""
from __future__ import annotations

import json
import os
import random
from pathlib import Path

import numpy as np
import torch

from ..formats import deltas


def _atomic_save(obj, path: Path):
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def save(out_dir, step: int, model, opt, rank: int = 0, extra: dict | None = None):
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    if rank == 0:
        sd = {k: v.detach().cpu().clone() for k, v in model.state_dict().items()}
        _atomic_save({"step": step, "params": sd, "extra": extra or {}}, out / "trained.pt")
    _atomic_save({"step": step, "opt": opt.state_dict() if opt is not None else None,
                  "rng": {"torch": torch.get_rng_state(), "numpy": np.random.get_state(),
                          "python": random.getstate(),
                          "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None}},
                 out / f"opt-rank{rank}.pt")


def load(out_dir, model, opt=None, rank: int = 0) -> int:
    """Restore parameters (and this rank's optimizer shard if present). Returns the saved step."""
    out = Path(out_dir)
    t = torch.load(out / "trained.pt", map_location="cpu", weights_only=False)
    with torch.no_grad():
        for k, v in model.state_dict().items():
            v.copy_(t["params"][k].to(v.device))
    o = out / f"opt-rank{rank}.pt"
    if opt is not None and o.exists():
        s = torch.load(o, map_location="cpu", weights_only=False)
        if s["step"] != t["step"]:
            raise ValueError(f"{o} is from step {s['step']}, trained.pt from step {t['step']}")
        opt.load_state_dict(s["opt"])
        torch.set_rng_state(s["rng"]["torch"])
        np.random.set_state(s["rng"]["numpy"])
        random.setstate(s["rng"]["python"])
        if s["rng"]["cuda"] is not None and torch.cuda.is_available():
            torch.cuda.set_rng_state_all(s["rng"]["cuda"])
    return int(t["step"])


def export_delta(model, layers, out_dir, keep_json: str | None = None):
    """Write the FN delta of a trained student. `layers` = the LowbitLayer list the student was built from
    (expert ids in kept order)."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    for l, (lay, sc) in enumerate(zip(layers, model.export_scales())):
        d = {e: {"gu_s": sc["gu_s"][i].clone(), "d_s": sc["d_s"][i].clone()} for i, e in enumerate(lay.experts)}
        torch.save(d, out / f"scales-L{l:02d}.pt")
        torch.save({"weight": sc["router"].to(torch.bfloat16), "keep": list(lay.experts)}, out / f"router-L{l:02d}.pt")
    if keep_json and os.path.exists(keep_json):
        (out / "keep.json").write_text(Path(keep_json).read_text())
    deltas.write_manifest(out)
    return out

"""Routing capture: teacher-forced replay of token sequences through the serving engine, recording per MoE layer
the router's inputs and logits (calibration rows for GPTQ Hessians and REAP saliency) and per-expert routing
statistics (top-k counts and summed gate weights, the keep-coverage denominator).

The reference installs a capture hook in its vLLM MoE block and replays recorded solver traces through a server
(flashnext/training/plugin/fnplug.py:135-160 `_cap_flush`/`_install_capture`, prune_gptq/replay.py). Here the
hook is :attr:`models.fn.FNModel.capture`, and :func:`replay` drives the engine's own chunked prefill; the files
it writes are what :mod:`.compress` consumes:

* ``<dir>/L{layer:02d}_{chunk:04d}.pt``: {"x": [rows, H] fp16, "logits": [rows, E] fp32}, rows sampled with stride
  ``every`` (all rows with every=1), flushed whenever a layer buffers ``flush_rows`` rows;
* ``<dir>/stats.pt``: {"layers", "counts": {l: [E] int64}, "wsum": {l: [E] fp64}, "tokens": {l: int}}.
"""
from __future__ import annotations

import os
from pathlib import Path

import torch


class RoutingCapture:
    def __init__(self, out_dir, top_k: int, every: int = 1, flush_rows: int = 65536, keep_rows: bool = True):
        self.dir = Path(out_dir)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.top_k, self.every, self.flush_rows, self.keep_rows = top_k, max(1, every), flush_rows, keep_rows
        self.buf, self.nbuf, self.chunk = {}, {}, {}
        self.counts, self.wsum, self.tokens = {}, {}, {}
        self._seen = {}

    def record(self, layer: int, x: torch.Tensor, logits: torch.Tensor):
        """One MoE call: x [T, H] router inputs, logits [T, E] (softmax routing, as the FN router)."""
        E = logits.shape[1]
        pr = torch.softmax(logits.float(), -1)
        w, ids = pr.topk(self.top_k, -1)
        w = w / w.sum(-1, keepdim=True)
        if layer not in self.counts:
            self.counts[layer] = torch.zeros(E, dtype=torch.int64)
            self.wsum[layer] = torch.zeros(E, dtype=torch.float64)
            self.tokens[layer] = 0
        self.counts[layer] += torch.bincount(ids.reshape(-1), minlength=E).cpu()
        self.wsum[layer] += torch.zeros(E, dtype=torch.float64, device=w.device).index_add_(
            0, ids.reshape(-1), w.reshape(-1).double()).cpu()
        self.tokens[layer] += x.shape[0]
        if not self.keep_rows:
            return
        start = (-self._seen.get(layer, 0)) % self.every
        self._seen[layer] = self._seen.get(layer, 0) + x.shape[0]
        rows = torch.arange(start, x.shape[0], self.every, device=x.device)
        if rows.numel():
            self.buf.setdefault(layer, []).append((x[rows].half().cpu(), logits[rows].float().cpu()))
            self.nbuf[layer] = self.nbuf.get(layer, 0) + rows.numel()
            if self.nbuf[layer] >= self.flush_rows:
                self._flush(layer)

    def _flush(self, layer: int):
        parts = self.buf.pop(layer, [])
        if not parts:
            return
        k = self.chunk.get(layer, 0)
        self.chunk[layer] = k + 1
        torch.save({"x": torch.cat([a for a, _ in parts]), "logits": torch.cat([b for _, b in parts])},
                   self.dir / f"L{layer:02d}_{k:04d}.pt")
        self.nbuf[layer] = 0

    def close(self):
        for layer in list(self.buf):
            self._flush(layer)
        L = sorted(self.counts)
        torch.save({"layers": L, "counts": {l: self.counts[l] for l in L}, "wsum": {l: self.wsum[l] for l in L},
                    "tokens": {l: self.tokens[l] for l in L}}, self.dir / "stats.pt")


def load_layer(out_dir, layer: int):
    """(x [rows, H] fp16, logits [rows, E] fp32) of one layer, all chunks concatenated."""
    files = sorted(Path(out_dir).glob(f"L{layer:02d}_*.pt"))
    if not files:
        return None, None
    parts = [torch.load(f, map_location="cpu") for f in files]
    return torch.cat([p["x"] for p in parts]), torch.cat([p["logits"] for p in parts])


def load_stats(out_dir) -> dict:
    return torch.load(Path(out_dir) / "stats.pt", map_location="cpu")


def replay(llm, sequences, capture: RoutingCapture, chunk: int = 2048):
    """Teacher-forced prefill of each token sequence through the engine's model with the capture hook installed
    (eager chunks: graph replays cannot run host code). The sequences' caches are released afterwards."""
    model = llm.model
    prev, model.capture = model.capture, capture
    try:
        for ids in sequences:
            slot = llm.free_slots.pop()
            try:
                model.reset_slot(slot)
                model.assign_blocks(slot, len(ids), llm.alloc)
                t = torch.tensor(ids, dtype=torch.int32)
                for p0 in range(0, len(ids), chunk):
                    n = min(chunk, len(ids) - p0)
                    model.step(t[p0:p0 + n].to(llm.device), torch.tensor([slot], dtype=torch.int32, device=llm.device),
                               torch.tensor([p0], dtype=torch.int32, device=llm.device), n)
            finally:
                llm.alloc.release(slot)
                model.reset_slot(slot)
                llm.free_slots.append(slot)
    finally:
        model.capture = prev
    capture.close()

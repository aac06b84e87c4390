"""Sampling parameters and the sampler (csrc/k_sample.cu on GPU, the same algorithm and hash on CPU).

Rules: temperature <= 0 is greedy; without top-k / top-p the draw is Gumbel-max over the full vocabulary; with
either, the top min(k, 1024) logits are sorted, softmaxed at the temperature, cut to the smallest prefix whose
mass reaches top_p, and sampled by one inverse-CDF draw. Randomness is a pure function of (seed, step, index), so
a sequence's samples do not depend on batch composition and replays reproduce them.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import native

CAND = 1024
_C1, _C2, _C3 = np.uint64(0x9E3779B97F4A7C15), np.uint64(0xD1B54A32D192ED03), np.uint64(0x8CB92BA72F3D8DD7)


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int = 0
    max_tokens: int = 64
    stop_token_ids: list = field(default_factory=list)
    logprobs: bool = False

    @staticmethod
    def from_request(b: dict, default_temperature: float = 1.0) -> "SamplingParams":
        return SamplingParams(temperature=float(b.get("temperature", default_temperature)),
                              top_p=float(b.get("top_p", 1.0)), top_k=int(b.get("top_k") or 0),
                              seed=int(b["seed"]) if b.get("seed") is not None else int(np.random.randint(1 << 62)),
                              max_tokens=int(b.get("max_tokens", 16)),
                              stop_token_ids=list(b.get("stop_token_ids") or []),
                              logprobs=b.get("logprobs") is not None)


def _mix64(z):
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, step: int, idx) -> np.ndarray:
    """The kernel's uniforms in (0, 1) as float32."""
    i = np.asarray(idx, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed % (1 << 64)) * _C1 + np.uint64(step % (1 << 64)) * _C2 + i * _C3 + np.uint64(1)
    h = _mix64(z)
    return (((h >> np.uint64(41)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 8388608.0))


def _i64(c) -> int:
    """uint64 constant as the int64 with the same bits (torch integer arithmetic wraps modulo 2^64)."""
    c = int(c)
    return c - (1 << 64) if c >= (1 << 63) else c


_M = [_i64(0xBF58476D1CE4E5B9), _i64(0x94D049BB133111EB)]


def _shr(z: torch.Tensor, n: int) -> torch.Tensor:
    """Logical right shift of int64 bit patterns."""
    return (z >> n) & ((1 << (64 - n)) - 1)


def uniform_torch(seed: int, step: int, idx: torch.Tensor) -> torch.Tensor:
    """:func:`uniform` on a torch int64 index tensor (any device), bit-identical: the same counter hash in
    wrapping int64 arithmetic."""
    with np.errstate(over="ignore"):
        base = _i64(np.uint64(seed % (1 << 64)) * _C1 + np.uint64(step % (1 << 64)) * _C2 + np.uint64(1))
    z = idx.long() * _i64(_C3) + base
    z = (z ^ _shr(z, 30)) * _M[0]
    z = (z ^ _shr(z, 27)) * _M[1]
    z = z ^ _shr(z, 31)
    return (_shr(z, 41).float() + 0.5) * (1.0 / 8388608.0)


def _sample_row(x: torch.Tensor, T: float, k: int, p: float, seed: int, step: int) -> int:
    V = x.shape[0]
    if T <= 0:
        return int(torch.argmax(x))
    xf = x.float().numpy()
    if k <= 0 and p >= 1.0:
        u = uniform(seed, step, np.arange(V))
        g = xf * np.float32(1.0 / T) - np.log(-np.log(u))
        return int(np.argmax(g))
    K = min(k if k > 0 else CAND, CAND, V)
    order = torch.sort(x.float(), descending=True, stable=True).indices[:K].numpy()
    v = xf[order]
    cum = np.cumsum(np.exp((v - v[0]) / np.float32(T)).astype(np.float32), dtype=np.float32)
    cut = K - 1
    if p < 1.0:
        cut = int(np.argmax(cum >= np.float32(p) * cum[-1]))
    u = uniform(seed, step, [V])[0] * cum[cut]
    pick = int(np.argmax(cum[: cut + 1] > u)) if (cum[: cut + 1] > u).any() else cut
    return int(order[pick])


def sample(logits: torch.Tensor, temp, top_k, top_p, seed, step, want_lp: bool = True):
    """logits [B, V] fp32; per-row parameter tensors [>= B] (temp f32, top_k i32, top_p f32, seed/step i64).
    Returns (ids int32 [B], logprob of each chosen token under log_softmax(logits) [B] or None)."""
    B = logits.shape[0]
    if logits.is_cuda:
        ids = torch.empty(B, dtype=torch.int32, device=logits.device)
        lp = torch.empty(B, dtype=torch.float32, device=logits.device) if want_lp else None
        native.C().sample_rows(logits, temp, top_k, top_p, seed, step, ids, lp)
        return ids, lp
    ids = torch.tensor([_sample_row(logits[b], float(temp[b]), int(top_k[b]), float(top_p[b]), int(seed[b]),
                                    int(step[b])) for b in range(B)], dtype=torch.int32)
    lp = None
    if want_lp:
        lp = torch.log_softmax(logits.float(), -1).gather(1, ids.long()[:, None])[:, 0]
    return ids, lp


def params_tensors(sps: list, steps: list, device):
    """Parameter vectors for a batch of SamplingParams (host tensors; pinned when the device is a GPU)."""
    pin = torch.device(device).type == "cuda"
    t = torch.tensor([s.temperature for s in sps], dtype=torch.float32)
    k = torch.tensor([s.top_k for s in sps], dtype=torch.int32)
    p = torch.tensor([s.top_p for s in sps], dtype=torch.float32)
    sd = torch.tensor([s.seed for s in sps], dtype=torch.int64)
    st = torch.tensor(steps, dtype=torch.int64)
    out = [t, k, p, sd, st]
    return [x.pin_memory() for x in out] if pin else out

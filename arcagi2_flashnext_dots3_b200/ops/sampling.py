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


# ------------------------------------------------------------------------------------ speculative verify
ACCEPT_INDEX = -1     # RNG index of the acceptance draw (vocabulary indices are >= 0)


def _row_candidates(lg: torch.Tensor, drafts: torch.Tensor, T: float, seed: int, step: int, v0: int = 0):
    """Per verify position j of one sequence (lg [k1, Vl] logits of a vocabulary slice starting at global index
    v0, drafts [k]): (max, sum of exp(l/T - max), logit of draft j or -inf, best Gumbel-max value, its global
    index); position j's candidate excludes draft j, the last position excludes nothing. Greedy (T <= 0) uses
    the raw logits with no noise and no probabilities."""
    k1, Vl = lg.shape
    k = k1 - 1
    idx = torch.arange(v0, v0 + Vl, device=lg.device)
    x = lg.float()
    out = torch.empty(k1, 5, dtype=torch.float64, device=lg.device)
    for j in range(k1):
        d = int(drafts[j]) if j < k else -1
        local_d = d - v0
        own = 0 <= local_d < Vl
        if T > 0:
            z = x[j] / T
            m = z.max()
            out[j, 0] = m
            out[j, 1] = torch.exp(z - m).sum()
            out[j, 2] = z[local_d] if own else float("-inf")
            key = z - torch.log(-torch.log(uniform_torch(seed, step + j, idx)))
        else:
            out[j, 0], out[j, 1] = 0.0, 1.0
            out[j, 2] = x[j, local_d] if own else float("-inf")
            key = x[j].clone()
        if own:
            key[local_d] = float("-inf")
        best = int(key.argmax())
        out[j, 3] = key[best]
        out[j, 4] = v0 + best
    return out


def _decide(cands: torch.Tensor, drafts, T: float, seed: int, step: int, k: int):
    """cands [shards, k1, 5] (shards in vocabulary order) -> (accepted drafts, next token)."""
    m, s, ld = cands[..., 0], cands[..., 1], cands[..., 2]
    for j in range(k):
        if T > 0:
            gm = m.max(0).values[j]
            logz = gm + torch.log((s[:, j] * torch.exp(m[:, j] - gm)).sum())
            p_d = float(torch.exp(ld.max(0).values[j] - logz))
            u = float(uniform_torch(seed, step + j, torch.tensor([ACCEPT_INDEX]))[0])
            ok = u < p_d
        else:   # greedy: the draft must be the argmax (lowest index on ties)
            best_other = cands[:, j, 3].max()
            dl = float(ld[:, j].max())
            ok = dl > best_other or (dl == best_other and int(drafts[j]) < _first_index(cands[:, j]))
        if not ok:
            return j, _first_index(cands[:, j])
    return k, _first_index(cands[:, k])


def _first_index(c: torch.Tensor) -> int:
    """Global index of the largest candidate value over shards, lowest index among equal values."""
    vals, ids = c[:, 3], c[:, 4]
    top = vals.max()
    return int(ids[vals == top].min())


def speculative_accept(logits: torch.Tensor, drafts: torch.Tensor, temps, seeds, steps):
    """Speculative verification of point-mass drafts, per sequence b: logits [B, k + 1, V], drafts [B, k],
    temps / seeds / steps per sequence (step = index of the first token this verify emits). Draft j is accepted
    with probability p_j(d_j) (p_j = softmax(logits[b, j] / T)), drawn from the counter RNG at (seed, step + j,
    index -1); at the first rejection the token comes from p_j with d_j removed (renormalized), by Gumbel-max
    with the noise at (seed, step + j, token index); with every draft accepted a bonus token comes from p_k. The
    emitted tokens are distributed as sampling from the model. Greedy rows (T <= 0): accept while the draft is
    the argmax; the next token is the argmax. Returns (accepted [B] int, next [B] int) as lists."""
    B, k1, V = logits.shape
    acc, nxt = [], []
    for b in range(B):
        T, sd, st = float(temps[b]), int(seeds[b]), int(steps[b])
        c = _row_candidates(logits[b], drafts[b], T, sd, st)
        a, t = _decide(c[None], drafts[b], T, sd, st, k1 - 1)
        acc.append(a)
        nxt.append(t)
    return acc, nxt

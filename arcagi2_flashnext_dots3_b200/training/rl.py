"""Policy-gradient repair training (REINFORCE leave-one-out, optional PPO clipping).

The objective is the reference's (flashnext/training/rl/train_rl.py:17 `seq_pg`, :63-72 defaults; rewards and
advantages from rl/prep_rl.py): for each rollout sequence, advantage A = r - mean(r of the other samples of the
same task), clipped to [-clip, clip]; loss = -sum_seq A * sum_{generated t} log pi(y_t) / (n * tok_norm) with n
the samples of one optimizer step over all replicas and tok_norm = 16384. With ``ppo_clip > 0`` the per-token
term becomes min(r A, clip(r, 1-eps, 1+eps) A), r = exp(lp - lp_old). Learning-rate schedule: linear warm-up,
then cosine to zero.
"""
from __future__ import annotations

import math

import numpy as np
import torch
from torch.utils.checkpoint import checkpoint


def loo_advantages(rewards, clip: float | None = 2.0) -> np.ndarray:
    """rewards [n_tasks, n_samples] -> leave-one-out advantages (same shape)."""
    r = np.asarray(rewards, dtype=np.float64)
    n = r.shape[1]
    if n < 2:
        raise ValueError("leave-one-out needs at least 2 samples per task")
    a = r - (r.sum(1, keepdims=True) - r) / (n - 1)
    return np.clip(a, -clip, clip) if clip is not None else a


def lp_chunk(h, lm_head, y):
    ls = torch.log_softmax((h @ lm_head.float().t()).float(), -1)
    lp = ls.gather(1, y[:, None].long())[:, 0]
    ent = -(ls.exp() * ls).sum(1)
    return lp, ent.detach()


def seq_pg(model, ids, pos, A: float, chunk: int = 1024, grad: bool = True, old=None, eps: float = 0.2):
    """Policy-gradient objective of one sequence. ids [L] token ids, pos [n] positions of generated tokens
    (scored from the hidden state at pos - 1). Returns (objective tensor, stats dict)."""
    dev = model.device
    ids = torch.as_tensor(ids, dtype=torch.long, device=dev)
    pos_t = torch.as_tensor(pos, dtype=torch.long, device=dev)
    h = model.hidden(ids, ckpt=grad)
    y = ids[pos_t]
    old_t = torch.as_tensor(old, dtype=torch.float32, device=dev) if old is not None else None
    tot = h.new_zeros(())
    slp, sent, nclip = 0.0, 0.0, 0
    lps = []
    for a in range(0, len(pos_t), chunk):
        b = min(len(pos_t), a + chunk)
        args = (h[pos_t[a:b] - 1], model.lm_head, y[a:b])
        lp, ent = checkpoint(lp_chunk, *args, use_reentrant=False) if grad else lp_chunk(*args)
        lps.append(lp.detach())
        if old_t is None:
            tot = tot + A * lp.sum()
        else:
            r = torch.exp(lp - old_t[a:b])
            tot = tot + torch.minimum(r * A, torch.clamp(r, 1 - eps, 1 + eps) * A).sum()
            nclip += int(((r < 1 - eps) | (r > 1 + eps)).sum())
        slp += float(lp.detach().sum())
        sent += float(ent.sum())
    return tot, {"lp": slp, "ent": sent, "n": len(pos_t), "clipped": nclip, "A": A,
                 "token_lp": torch.cat(lps) if lps else torch.zeros(0)}


def lr_factor(step: int, total: int, warmup: int) -> float:
    if step < warmup:
        return (step + 1) / max(1, warmup)
    if total <= warmup:
        return 1.0
    p = (step - warmup) / max(1, total - warmup)
    return 0.5 * (1 + math.cos(math.pi * min(1.0, p)))

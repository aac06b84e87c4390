"""Policy-gradient repair training: REINFORCE with leave-one-out baselines, optional PPO ratio clipping.

Objective (the recipe of flashnext/training/rl/train_rl.py:17-43 and :63-72; rewards and advantages from
rl/prep_rl.py): every rollout of a task gets the advantage A = r - mean(rewards of the task's other rollouts),
clipped to [-clip, clip]. A sequence contributes A * sum over its generated tokens of log pi(token); the trainer
divides the summed contributions by (rollouts per optimizer step * tok_norm) and descends on the negative. With
a PPO epsilon the per-token term is min(rho A, clip(rho, 1 - eps, 1 + eps) A), rho = pi / pi_old. The learning
rate warms up linearly, then follows a cosine to zero.

Implementation: token log-probabilities come from :class:`VocabLogProb`, an autograd function over row chunks
that keeps only the hidden rows and recomputes the [rows, vocab] projection during backward (the gradient of
log_softmax at the target is onehot - softmax), so no vocabulary-sized activation outlives its chunk. The
surrogate is then one vectorized expression over all of the sequence's tokens.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


def loo_advantages(rewards, clip: float | None = 2.0) -> np.ndarray:
    """rewards [n_tasks, n_samples] -> leave-one-out advantages (same shape)."""
    r = np.asarray(rewards, dtype=np.float64)
    n = r.shape[1]
    if n < 2:
        raise ValueError("leave-one-out needs at least 2 samples per task")
    others_mean = (r.sum(axis=1, keepdims=True) - r) / (n - 1)
    adv = r - others_mean
    return adv if clip is None else np.clip(adv, -clip, clip)


class VocabLogProb(torch.autograd.Function):
    """log softmax(h W^T)[target] per row, computed ``rows`` rows at a time.

    Forward keeps h, W and the per-row log-normalizers; backward recomputes each chunk's logits once and forms
    d logits = g (onehot(target) - softmax) in place, then d h = d logits W and, when W is trainable,
    d W += d logits^T h. Peak extra memory is one [rows, vocab] fp32 block."""

    @staticmethod
    def forward(ctx, h, W, target, rows: int):
        Wf = W.float()
        lse = torch.empty(h.shape[0], dtype=torch.float32, device=h.device)
        picked = torch.empty_like(lse)
        for s in range(0, h.shape[0], rows):
            z = h[s:s + rows].float() @ Wf.t()
            lse[s:s + rows] = torch.logsumexp(z, dim=-1)
            picked[s:s + rows] = z.gather(1, target[s:s + rows, None])[:, 0]
        ctx.save_for_backward(h, W, target, lse)
        ctx.rows = rows
        return picked - lse

    @staticmethod
    def backward(ctx, g):
        h, W, target, lse = ctx.saved_tensors
        Wf = W.float()
        dh = torch.empty_like(h) if ctx.needs_input_grad[0] else None
        dW = torch.zeros_like(Wf) if ctx.needs_input_grad[1] else None
        for s in range(0, h.shape[0], ctx.rows):
            hs = h[s:s + ctx.rows].float()
            d = hs @ Wf.t()
            d.sub_(lse[s:s + ctx.rows, None]).exp_().neg_()                # -softmax
            d.scatter_add_(1, target[s:s + ctx.rows, None], torch.ones_like(d[:, :1]))
            d.mul_(g[s:s + ctx.rows, None].float())
            if dh is not None:
                dh[s:s + ctx.rows] = (d @ Wf).to(dh.dtype)
            if dW is not None:
                dW.addmm_(d.t(), hs)
        return dh, (dW.to(W.dtype) if dW is not None else None), None, None


@torch.no_grad()
def token_entropy(h: torch.Tensor, W: torch.Tensor, rows: int = 1024) -> torch.Tensor:
    """Entropy of the next-token distribution per row of h (no gradient)."""
    out = torch.empty(h.shape[0], dtype=torch.float32, device=h.device)
    Wf = W.float()
    for s in range(0, h.shape[0], rows):
        lp = torch.log_softmax(h[s:s + rows].float() @ Wf.t(), dim=-1)
        out[s:s + rows] = -(lp.exp() * lp).sum(-1)
    return out


@dataclass
class PGStats:
    lp: float          # summed log-probability of the scored tokens
    ent: float         # summed entropy at the scored positions
    n: int             # scored tokens
    clipped: int       # tokens whose PPO ratio left [1 - eps, 1 + eps]
    A: float
    token_lp: torch.Tensor

    def __getitem__(self, k):   # dict-style access used by the training loop's running sums
        return getattr(self, k)


def surrogate(lp: torch.Tensor, A: float, old_lp: torch.Tensor = None, eps: float = 0.2):
    """Per-sequence policy-gradient surrogate (to be maximized) and the number of clipped tokens."""
    if old_lp is None:
        return A * lp.sum(), 0
    rho = torch.exp(lp - old_lp)
    clipped = torch.clamp(rho, 1.0 - eps, 1.0 + eps)
    obj = torch.minimum(rho * A, clipped * A).sum()
    return obj, int((rho != clipped).sum())


def seq_pg(model, ids, pos, A: float, chunk: int = 1024, grad: bool = True, old=None, eps: float = 0.2):
    """Surrogate of one rollout. ``ids`` [L] token ids; ``pos`` [n] positions of the generated tokens, each scored
    from the hidden state one position earlier; ``old`` optional behaviour-policy log-probs [n] (PPO).
    Returns (objective tensor, :class:`PGStats`)."""
    dev = model.device
    ids = torch.as_tensor(ids, dtype=torch.long, device=dev)
    at = torch.as_tensor(pos, dtype=torch.long, device=dev)
    ctx = torch.enable_grad() if grad else torch.no_grad()
    with ctx:
        h = model.hidden(ids, ckpt=grad)
        rows = h.index_select(0, at - 1)
        lp = VocabLogProb.apply(rows, model.lm_head, ids.index_select(0, at), max(1, chunk))
        old_lp = torch.as_tensor(old, dtype=torch.float32, device=dev) if old is not None else None
        obj, n_clip = surrogate(lp, A, old_lp, eps)
    ent = token_entropy(rows.detach(), model.lm_head, max(1, chunk))
    return obj, PGStats(lp=float(lp.detach().sum()), ent=float(ent.sum()), n=int(at.numel()), clipped=n_clip, A=A,
                        token_lp=lp.detach())


def lr_factor(step: int, total: int, warmup: int) -> float:
    """Linear warm-up over ``warmup`` steps, then a cosine from 1 to 0 over the remaining steps."""
    if step < warmup:
        return (step + 1) / max(1, warmup)
    if total <= warmup:
        return 1.0
    frac = min(1.0, (step - warmup) / max(1, total - warmup))
    return 0.5 + 0.5 * math.cos(math.pi * frac)

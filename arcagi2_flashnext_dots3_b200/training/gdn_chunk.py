"""Chunked gated delta rule for training (autograd through plain torch ops).

Recurrence (per value head): S_t = e^{g_t} S_{t-1} + k_t (beta_t (v_t - e^{g_t} S_{t-1}^T k_t))^T, o_t = S_t^T q_t.
The reference trains through the fla library's chunked kernel (flashnext/training/student/student_fn.py:251
`GDN`); this is the same chunk decomposition written out: within a chunk of C tokens the WY form
T = (I + strictly_lower(diag(beta) K K^T * Gamma))^{-1} (a unit-lower triangular solve) turns the sequential
updates into matrix products, and the state is carried across chunks. Decay factors are formed from masked
log-differences, so every exponent is <= 0.
"""
from __future__ import annotations

import torch


def chunk_gated_delta_rule(q, k, v, g, beta, chunk: int = 64, initial_state=None, return_state=False):
    """q, k [H, T, dk] (q pre-scaled, k L2-normalized), v [H, T, dv], g [H, T] (log decay <= 0), beta [H, T].
    Returns o [H, T, dv] (and the final state [H, dk, dv])."""
    Hh, T, dk = q.shape
    dv = v.shape[-1]
    C = chunk
    N = (T + C - 1) // C
    pad = N * C - T
    if pad:
        q = torch.cat([q, q.new_zeros(Hh, pad, dk)], 1)
        k = torch.cat([k, k.new_zeros(Hh, pad, dk)], 1)
        v = torch.cat([v, v.new_zeros(Hh, pad, dv)], 1)
        g = torch.cat([g, g.new_zeros(Hh, pad)], 1)
        beta = torch.cat([beta, beta.new_zeros(Hh, pad)], 1)
    q, k, v = q.view(Hh, N, C, dk), k.view(Hh, N, C, dk), v.view(Hh, N, C, dv)
    gc = g.view(Hh, N, C).cumsum(-1)
    beta = beta.view(Hh, N, C)
    kb = k * beta[..., None]
    vb = v * beta[..., None]
    lower_incl = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    diff = (gc[..., :, None] - gc[..., None, :]).masked_fill(~lower_incl, float("-inf"))
    gamma = diff.exp()                                                  # [H, N, C, C], zero above the diagonal
    strict = torch.ones(C, C, dtype=torch.bool, device=q.device).tril(-1)
    L = ((kb @ k.transpose(-1, -2)) * gamma).masked_fill(~strict, 0.0)
    eye = torch.eye(C, dtype=q.dtype, device=q.device)
    Tm = torch.linalg.solve_triangular(eye + L, eye.expand_as(L), upper=False, unitriangular=True)
    u = Tm @ vb
    w = Tm @ (kb * gc.exp()[..., None])
    S = q.new_zeros(Hh, dk, dv) if initial_state is None else initial_state.to(q.dtype)
    outs = []
    for n in range(N):
        qn, kn, gn = q[:, n], k[:, n], gc[:, n]
        attn = (qn @ kn.transpose(-1, -2)) * gamma[:, n]
        v_new = u[:, n] - w[:, n] @ S
        outs.append((qn * gn.exp()[..., None]) @ S + attn @ v_new)
        last = gn[:, -1:]
        S = S * last.exp()[..., None] + (kn * (last - gn).exp()[..., None]).transpose(-1, -2) @ v_new
    o = torch.stack(outs, 1).view(Hh, N * C, dv)[:, :T]
    return (o, S) if return_state else o

"""Offline expert compression: routing capture, saliency-based expert selection, GPTQ low-bit quantization.

Pipeline of the reference (flashnext/training/prune_gptq/gptq_fn.py: `mode_keep` :96, grids :140, `gptq` :152,
`mode_build` :213; flashnext/training/README.md:111-197):

1. capture: run calibration tokens through the model, record per MoE layer the gate inputs x and router logits;
2. keep: score every expert by REAP saliency, sum over routed tokens of gate weight x ||expert output||, keep the
   top-K per layer (keep.json), report the routed-weight coverage;
3. quantize: per kept expert and projection, a per-(row, 128-column group) asymmetric grid chosen by an MSE clip
   search over 10 ratios (1.0 .. 0.55), then GPTQ (second-order error compensation against the Hessian
   H = 2 X^T X / n of the projection's inputs) with activation order and static groups, damping
   lambda = mean(diag H) * (damp + 4 / n_tokens);
4. pack into the planar checkpoint (lowbit-LNN.pt / router-LNN.pt), sliced routers over the kept experts.

Everything is plain torch (GPU when the tensors are on a GPU).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..formats import lowbit_file
from ..formats.planar import pack_planar

G = 128


def clip_grid(W: torch.Tensor, bits: int, ratios=None):
    """Asymmetric per-(row, group) scale (fp16-representable) and zero minimizing the group's squared error over
    clip ratios. W [R, K] -> s [R, K/G] fp32, z [R, K/G] fp32 (integers)."""
    R, K = W.shape
    Wg = W.float().view(R, K // G, G)
    qmax = 2 ** bits - 1
    ratios = ratios if ratios is not None else torch.linspace(1.0, 0.55, 10).tolist()
    lo0, hi0 = Wg.amin(-1).clamp(max=0), Wg.amax(-1).clamp(min=0)
    best_err = None
    for c in ratios:
        lo, hi = lo0 * c, hi0 * c
        s = ((hi - lo) / qmax).clamp_min(1e-10)
        z = torch.round(-lo / s).clamp(0, qmax)
        q = torch.clamp(torch.round(Wg / s[..., None]) + z[..., None], 0, qmax)
        err = ((q - z[..., None]) * s[..., None] - Wg).pow(2).sum(-1)
        if best_err is None:
            best_s, best_z, best_err = s, z, err
        else:
            better = err < best_err
            best_s = torch.where(better, s, best_s)
            best_z = torch.where(better, z, best_z)
            best_err = torch.where(better, err, best_err)
    return best_s.half().float().clamp_min(6e-8), best_z


def rtn(W: torch.Tensor, bits: int):
    s, z = clip_grid(W, bits)
    R, K = W.shape
    qmax = 2 ** bits - 1
    q = torch.clamp(torch.round(W.float().view(R, K // G, G) / s[..., None]) + z[..., None], 0, qmax)
    return q.view(R, K).to(torch.uint8), s, z


class Hessian:
    """Running H = 2 / n * sum x x^T of one projection's inputs."""

    def __init__(self, K: int, device="cpu"):
        self.H = torch.zeros(K, K, dtype=torch.float64, device=device)
        self.n = 0

    def add(self, x: torch.Tensor):
        x = x.reshape(-1, x.shape[-1]).double()
        self.H += x.t() @ x
        self.n += x.shape[0]

    def value(self) -> torch.Tensor:
        return (2.0 / max(1, self.n)) * self.H


def gptq(W: torch.Tensor, H: torch.Tensor, bits: int, n_tokens: int, damp: float = 0.01, block: int = 128,
         act_order: bool = True):
    """GPTQ with static groups. W [R, K], H [K, K]. Returns (codes uint8 [R, K], s [R, K/G], z [R, K/G],
    dequantized fp32 [R, K])."""
    R, K = W.shape
    qmax = 2 ** bits - 1
    s, z = clip_grid(W, bits)          # static group grids (original column order)
    W = W.double().clone()
    H = H.double().clone()
    d = torch.diagonal(H)
    dead = d <= 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    lam = float(torch.diagonal(H).mean()) * (damp + 4.0 / max(1, n_tokens))
    H += lam * torch.eye(K, dtype=H.dtype, device=H.device)
    perm = torch.argsort(torch.diagonal(H), descending=True) if act_order else torch.arange(K, device=W.device)
    W, H = W[:, perm], H[perm][:, perm]
    group = perm // G
    Hinv = None
    for attempt in range(12):
        try:
            L = torch.linalg.cholesky(H)
            Hinv = torch.linalg.cholesky(torch.cholesky_inverse(L), upper=True)
            break
        except RuntimeError:  # not positive definite after damping: add more
            H += float(torch.diagonal(H).mean()) * 0.01 * 2 ** attempt * torch.eye(K, dtype=H.dtype, device=H.device)
    if Hinv is None:
        raise RuntimeError("Hessian could not be made positive definite")
    codes = torch.zeros(R, K, dtype=torch.uint8, device=W.device)
    Q = torch.zeros_like(W)
    sd, zd = s.double(), z.double()
    for b0 in range(0, K, block):
        b1 = min(K, b0 + block)
        Wb = W[:, b0:b1].clone()
        Eb = torch.zeros_like(Wb)
        Hb = Hinv[b0:b1, b0:b1]
        for i in range(b1 - b0):
            gi = group[b0 + i]
            sc, zc = sd[:, gi], zd[:, gi]
            w = Wb[:, i]
            q = torch.clamp(torch.round(w / sc) + zc, 0, qmax)
            dq = (q - zc) * sc
            codes[:, b0 + i] = q.to(torch.uint8)
            Q[:, b0 + i] = dq
            e = (w - dq) / Hb[i, i]
            Wb[:, i:] -= e[:, None] * Hb[i, i:][None, :]
            Eb[:, i] = e
        W[:, b1:] -= Eb @ Hinv[b0:b1, b1:]
    inv = torch.argsort(perm)
    return codes[:, inv], s, z, Q[:, inv].float()


# ------------------------------------------------------------------------------------------ expert selection
def expert_forward(x, wgu, wd):
    g, u = (x @ wgu.t()).chunk(2, -1)
    return (F.silu(g) * u) @ wd.t()


def reap_scores(x: torch.Tensor, logits: torch.Tensor, experts, top_k: int, scoring: str = "softmax",
                bias: torch.Tensor = None) -> torch.Tensor:
    """REAP saliency per expert: sum over routed tokens of (renormalized gate weight) x ||expert(x)||.
    experts: list of (W_gu [2I, H], W_d [H, I]) dense fp32."""
    if scoring == "softmax":
        pr = torch.softmax(logits.float(), -1)
        w, ids = torch.topk(pr, top_k, -1)
    else:  # sigmoid scores, selection by score + correction bias
        sc = torch.sigmoid(logits.float())
        ids = torch.topk(sc + (bias if bias is not None else 0), top_k, -1).indices
        w = sc.gather(1, ids)
    w = w / w.sum(-1, keepdim=True)
    scores = torch.zeros(len(experts), dtype=torch.float64)
    for e, (wgu, wd) in enumerate(experts):
        tok, slot = (ids == e).nonzero(as_tuple=True)
        if len(tok):
            y = expert_forward(x[tok].float(), wgu.float(), wd.float())
            scores[e] = float((w[tok, slot].double() * y.norm(dim=-1).double()).sum())
    return scores


def select_keep(scores: torch.Tensor, k: int, wsum: torch.Tensor = None):
    """Top-k experts by score; returns (sorted kept ids, routed-weight coverage or None)."""
    keep = sorted(torch.argsort(scores, descending=True)[:k].tolist())
    cov = None
    if wsum is not None:
        cov = float(wsum[keep].sum() / wsum.sum().clamp_min(1e-12))
    return keep, cov


# ------------------------------------------------------------------------------------------ layer build
def quantize_layer(experts, router: torch.Tensor, keep: list, bits: list, x_calib: torch.Tensor = None,
                   logits: torch.Tensor = None, top_k: int = 8, method: str = "gptq") -> lowbit_file.LowbitLayer:
    """Quantize the kept experts of one MoE layer. Hessians come from the calibration tokens routed to each
    expert (gate_up: its inputs x; down: silu(g)*u); experts without calibration tokens fall back to RTN."""
    routed = None
    if x_calib is not None and logits is not None:
        ids = torch.topk(torch.softmax(logits.float(), -1), top_k, -1).indices
        routed = {e: (ids == e).any(-1).nonzero().flatten() for e in keep}
    blobs = []
    for j, e in enumerate(keep):
        wgu, wd = experts[e]
        b = bits[j]
        tok = routed[e] if routed is not None else None
        if method == "gptq" and tok is not None and len(tok) > 0:
            xe = x_calib[tok].float()
            h1 = Hessian(wgu.shape[1], xe.device)
            h1.add(xe)
            qg, sg, zg, dq_gu = gptq(wgu.float(), h1.value(), b, len(tok))
            gg, uu = (xe @ dq_gu.t()).chunk(2, -1)
            h2 = Hessian(wd.shape[1], xe.device)
            h2.add(F.silu(gg) * uu)
            qd, sdn, zdn, _ = gptq(wd.float(), h2.value(), b, len(tok))
        else:
            qg, sg, zg = rtn(wgu, b)
            qd, sdn, zdn = rtn(wd, b)
        blobs.append(lowbit_file.ExpertBlob(b, pack_planar(qg.to(torch.int32).cpu(), b), sg.half().cpu(),
                                            zg.to(torch.uint8).cpu(), pack_planar(qd.to(torch.int32).cpu(), b),
                                            sdn.half().cpu(), zdn.to(torch.uint8).cpu()))
    n_orig = len(experts)
    keep_mask = [e in set(keep) for e in range(n_orig)]
    return lowbit_file.LowbitLayer(list(keep), blobs, router[keep].to(torch.bfloat16).cpu(), keep_mask)


def recon_error(W: torch.Tensor, Wq: torch.Tensor, x: torch.Tensor) -> float:
    """Relative output error ||x W^T - x Wq^T|| / ||x W^T|| on inputs x."""
    y = x.float() @ W.float().t()
    return float((y - x.float() @ Wq.float().t()).norm() / y.norm().clamp_min(1e-12))


def bits_for(n_keep: int, tiers: str) -> list:
    """Bit widths by rank: tiers 'end:bits,...' ('160:4,all:3' = first 160 kept experts at 4 bits, rest 3)."""
    out = []
    for t in tiers.split(","):
        end, b = t.split(":")
        end = n_keep if end == "all" else int(end)
        out += [int(b)] * (end - len(out))
    return out[:n_keep] + [out[-1]] * max(0, n_keep - len(out))


__all__ = ["clip_grid", "rtn", "Hessian", "gptq", "reap_scores", "select_keep", "quantize_layer", "recon_error",
           "bits_for", "math"]

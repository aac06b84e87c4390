"""Draft-head (MTP) training for the FN-shaped model.

The reference fine-tunes its MTP layer (layer 48) as the speculative-decoding draft head: an
expected-accepted-length objective, -E + 0.3 * KL, over 4 unrolled draft steps, with the LM head restricted
to the hottest 32k tokens (flashnext/training/draft_head/train.py; docs/appendix.tex:270-293). The trained
dense tensors ship as an override file next to scale/router deltas of layer 48.

Here :class:`DraftHeadTrain` is the head in autograd form. It mirrors :meth:`..models.fn_mtp.MTPHead.step`
(normalize the main hidden state and the next token's embedding, project [e; x] with `fc`, one attention + MoE
layer, stream mixer, the main model's LM head), with the layer computed by the student machinery of
:mod:`.student`. Trainable: fc, the two input norms, optionally the attention projections, and the MoE router
rows and log-scale offsets. Unrolled step k reads the previous step's output at every position q and the true
token t_{q+k}, uses rotary position q + k - 1 (the position the serving head writes for that chain step), and
attends causally to the same step's entries. That is the parallel form of the chain; the serving cache
instead holds step-1 entries for past positions.

Objective per start position q: alpha_k = sum_v min(q_k(v), p_k(v)), the probability that draft k is accepted
when drafts are sampled from q_k and verified against the target distribution p_k (the main model's next-token
distribution at position q + k, renormalized over the hot vocabulary). E = sum_k prod_{j <= k} alpha_j is the
expected number of accepted drafts. loss = -mean(E) + kl_weight * mean_k KL(p_k || q_k).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..models import fn_reference as R
from ..models.fn_mtp import mtp_config
from .student import FNStudent


def hot_vocab(token_counts: torch.Tensor, n: int) -> torch.Tensor:
    """The n most frequent token ids (ties: lower id), sorted ascending."""
    order = torch.sort(token_counts.float(), descending=True, stable=True).indices[:n]
    return torch.sort(order).values


class DraftHeadTrain(nn.Module):
    def __init__(self, cfg, main_dense: dict, mtp_dense: dict, device, hot_ids: torch.Tensor = None,
                 train_attn: bool = True):
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        mc = mtp_config(cfg)
        self.inner = FNStudent(mc, {"embed": main_dense["embed"], "lm_head": main_dense["lm_head"],
                                    "mixer": mtp_dense["mixer"], "layers": [mtp_dense["layer"]]}, self.device)
        self.fc = nn.Parameter(mtp_dense["fc"].float().to(self.device).clone())
        self.pe = nn.Parameter(mtp_dense["pe"].float().to(self.device).clone())
        self.ph = nn.Parameter(mtp_dense["ph"].float().to(self.device).clone())
        self.attn = nn.ParameterDict()
        if train_attn:
            mix = self.inner.W["layers"][0]["mix"]
            for k, v in list(mix.items()):
                if torch.is_tensor(v) and v.dim() == 2 and v.is_floating_point():
                    p = nn.Parameter(v.float().clone())
                    mix[k] = p
                    self.attn[k] = p
        self.register_buffer("hot", hot_ids.to(self.device).long() if hot_ids is not None else None)
        self._src_layer, self._src_mixer = mtp_dense["layer"], mtp_dense["mixer"]

    def step(self, x_prev: torch.Tensor, ids_next: torch.Tensor, pos0: int) -> torch.Tensor:
        """x_prev [Q, H] (main final hidden or the previous step's output), ids_next [Q] -> [Q, H]; rows are the
        consecutive positions pos0, pos0 + 1, ... of one sequence."""
        cfg = self.cfg
        H, hc = cfg.hidden_size, cfg.hc_count
        W = self.inner.W
        e = W["embed"][ids_next.to(self.device).long()].float()
        u = torch.cat([R.rms1p(e, self.pe, cfg.rms_eps), R.rms1p(x_prev.float(), self.ph, cfg.rms_eps)], -1)
        h = (u @ self.fc.t()).repeat(1, hc)
        Q = ids_next.shape[0]
        cos, sin = R.rope_cos_sin(torch.arange(pos0, pos0 + Q), cfg.rope_dim, cfg.rope_theta)
        h = self.inner._layer(0, h, None, cos.to(self.device), sin.to(self.device))
        return R.gated_residual(h, W["mixer"], hc, H, cfg.rms_eps, combine=False)

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        head = self.inner.lm_head.float()
        if self.hot is not None:
            head = head[self.hot]
        return x @ head.t()

    def param_groups(self, lr_dense: float = 1e-4, lr_scales: float = 3e-4, lr_router: float = 1.5e-5):
        g = [{"params": [self.fc, self.pe, self.ph] + list(self.attn.values()), "lr": lr_dense, "name": "dense"}]
        return g + [x for x in self.inner.param_groups(lr_scales, lr_router) if x["name"] in ("scales", "router")]

    def export(self) -> dict:
        """{"dense": the MTP weights in the dense layout with the trained fc, norms and attention projections (serve
        with fn_mtp.mtp_to_engine), "moe": the layer's trained scales and router rows in the student's delta
        format (the reference ships these as the layer-48 scale / router delta)}."""
        with torch.no_grad():
            layer = dict(self._src_layer)
            layer["mix"] = {k: (self.attn[k].detach().cpu().clone() if k in self.attn else v)
                            for k, v in self._src_layer["mix"].items()}
            dense = {"fc": self.fc.detach().cpu().clone(), "pe": self.pe.detach().cpu().clone(),
                     "ph": self.ph.detach().cpu().clone(), "layer": layer, "mixer": self._src_mixer}
            return {"dense": dense, "moe": self.inner.export_scales()[0]}


def draft_objective(model: DraftHeadTrain, h_main: torch.Tensor, ids: torch.Tensor, target_logits: torch.Tensor,
                    K: int = 4, kl_weight: float = 0.3):
    """(loss, mean E) for one sequence. h_main [T, H]: the main model's final hidden states; ids [T] the tokens;
    target_logits [T, V]: the main model's logits (row q predicts t_{q+1})."""
    T = ids.shape[0]
    Q = T - K
    if Q <= 0:
        raise ValueError("sequence shorter than the number of unrolled steps")
    dev = model.device
    ids = ids.to(dev)
    tl = target_logits.to(dev).float()
    if model.hot is not None:
        tl = tl[:, model.hot]
    x = h_main[:Q].to(dev).float()
    prod = torch.ones(Q, device=dev)
    E = torch.zeros(Q, device=dev)
    kl = x.new_zeros(())
    for k in range(1, K + 1):
        x = model.step(x, ids[k:k + Q], k - 1)
        lq = torch.log_softmax(model.logits(x), -1)
        lp = torch.log_softmax(tl[k:k + Q], -1)
        p = lp.exp()
        prod = prod * torch.minimum(lq.exp(), p).sum(-1)
        E = E + prod
        kl = kl + (p * (lp - lq)).sum(-1).mean()
    return -E.mean() + kl_weight * kl / K, E.mean().detach()


def train_draft_head(model: DraftHeadTrain, batches, steps: int, K: int = 4, kl_weight: float = 0.3, **lrs):
    """Adam over `steps` batches; every batch is an iterable of (h_main, ids, target_logits) sequences.
    Returns the per-step history of (loss, E)."""
    opt = torch.optim.Adam(model.param_groups(**lrs))
    hist = []
    it = iter(batches)
    for _ in range(steps):
        seqs = next(it)
        opt.zero_grad(set_to_none=True)
        tot, e_sum = 0.0, 0.0
        for h, ids, tl in seqs:
            loss, e = draft_objective(model, h, ids, tl, K, kl_weight)
            (loss / len(seqs)).backward()
            tot += float(loss.detach()) / len(seqs)
            e_sum += float(e) / len(seqs)
        opt.step()
        hist.append((tot, e_sum))
    return hist


__all__ = ["DraftHeadTrain", "draft_objective", "train_draft_head", "hot_vocab"]

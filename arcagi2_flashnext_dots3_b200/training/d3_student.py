"""Differentiable Dots3-Note-shaped student and the SFT / distillation objectives.

The reference trains its D3 build's expert scales, RMSNorm weights and router rows with cross-entropy on selected
SFT samples or top-k distillation against the teacher (dotsnote/training/finetune/student.py: `Attn` :177-259,
`MoE` :290-343, `Layer` :345-362, `Student` :364; train.py:10-64 losses; dotsnote/training/README.md:341-412).
Here the layer math is :mod:`..models.d3_reference` with attention as one masked scaled-dot-product call and the
experts in :class:`.lowbit.GroupedExperts` (sigmoid scores, top-k by score + correction bias, renormalized,
times the routed scaling factor), so the trainable tensors and the export format are the FN student's.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from ..models import d3_reference as R
from .lowbit import ExpertBank, grouped_experts
from .student import _to


def mla_train(x, p, cfg, l, cos, sin):
    """d3_reference.mla with SDPA; the DSA selection is computed without gradient (as in the reference)."""
    T = x.shape[0]
    H, kvr = cfg.heads_of(l), cfg.latent_of(l)
    dn, dr, dv, qr = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.q_lora_rank
    qs = (cfg.hidden_size / qr) ** 0.5 if cfg.kv_rescale else 1.0
    kvs = (cfg.hidden_size / kvr) ** 0.5 if cfg.kv_rescale else 1.0
    qc = R.rms(x @ p["q_a"].t(), p["q_ln"], cfg.rms_eps) * qs
    kvc, kpe = (x @ p["kv_a"].t()).split([kvr, dr], -1)
    kvc = R.rms(kvc, p["kv_ln"], cfg.rms_eps) * kvs
    kvc = kvc + (kvc.to(torch.float8_e4m3fn).float() - kvc).detach()          # FP8 cache round trip, straight-through
    kpe = R.rms(kpe, p["kr_ln"], cfg.rms_eps)
    q = (qc @ p["q_b"].t()).view(T, H, dn + dr)
    q = torch.cat([q[..., :dn], R.rope_inter(q[..., dn:], cos, sin)], -1)
    kpe = R.rope_inter(kpe[:, None, :], cos, sin)
    kpe = kpe + (kpe.to(torch.float8_e4m3fn).float() - kpe).detach()
    kv = (kvc @ p["kv_b"].t()).view(T, H, dn + dv)
    k = torch.cat([kv[..., :dn], kpe.expand(T, H, dr)], -1)
    v = kv[..., dn:]
    ar = torch.arange(T, device=x.device)
    allowed = ar[None, :] <= ar[:, None]
    if cfg.layer_kind(l) == "swa":
        allowed = allowed & (ar[:, None] - ar[None, :] < cfg.swa_window)
    else:
        with torch.no_grad():
            M = R.dsa_mask(x.detach(), qc.detach(), p, cfg, cos, sin)
        if M is not None:
            allowed = M
    o = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                       attn_mask=allowed[None], scale=(dn + dr) ** -0.5)
    gate = torch.sigmoid(x @ p["g"].t())
    return (o.transpose(0, 1) * gate[..., None]).reshape(T, H * dv) @ p["o"].t()


class D3MoETrain(nn.Module):
    def __init__(self, moe: dict, cfg, device):
        super().__init__()
        self.cfg = cfg
        self.bank = ExpertBank.from_lowbit(moe["lowbit"], device)
        self.router = nn.Parameter(moe["gate"].float().to(device).clone())
        self.t_gu = nn.Parameter(torch.zeros_like(self.bank.s0["gu"]))
        self.t_d = nn.Parameter(torch.zeros_like(self.bank.s0["d"]))
        self.register_buffer("bias", moe["bias"].float().to(device))
        self.shared = {k: v.float().to(device) for k, v in moe["shared"].items()}

    def scales(self):
        return self.bank.s0["gu"] * self.t_gu.exp(), self.bank.s0["d"] * self.t_d.exp()

    def forward(self, x):
        cfg, k = self.cfg, self.cfg.top_k
        T, H = x.shape
        sc = torch.sigmoid(x @ self.router.t())
        ids = torch.topk((sc + self.bias).detach(), k, -1).indices
        w = sc.gather(1, ids)
        w = w / w.sum(-1, keepdim=True) * cfg.route_scale
        flat = ids.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=self.bank.E).tolist()
        s_gu, s_d = self.scales()
        ys = grouped_experts(x.repeat_interleave(k, 0)[order], s_gu, s_d, counts, self.bank)
        y = torch.zeros(T * k, H, dtype=ys.dtype, device=x.device).index_copy(0, order, ys)
        return (y.view(T, k, H) * w[..., None]).sum(1) + R.mlp(x, self.shared)


class D3Student(nn.Module):
    def __init__(self, cfg, W: dict, device, train_norms: bool = False):
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        Wd = _to({k: v for k, v in W.items() if k != "layers"}, self.device)
        Wd["layers"] = [_to({k: v for k, v in L.items() if k != "moe"}, self.device) for L in W["layers"]]
        self.W = Wd
        self.moe = nn.ModuleDict({str(l): D3MoETrain(L["moe"], cfg, self.device)
                                  for l, L in enumerate(W["layers"]) if cfg.is_moe(l)})
        self.norms = nn.ParameterList()
        if train_norms:
            for L in self.W["layers"]:
                for key in ("ln1", "ln2"):
                    prm = nn.Parameter(L[key].float().clone())
                    L[key] = prm
                    self.norms.append(prm)

    def _layer(self, l, h, cos, sin):
        cfg, L = self.cfg, self.W["layers"][l]
        h = h + mla_train(R.rms(h, L["ln1"], cfg.rms_eps), L["attn"], cfg, l, cos, sin)
        x = R.rms(h, L["ln2"], cfg.rms_eps)
        return h + (self.moe[str(l)](x) if cfg.is_moe(l) else R.mlp(x, L["mlp"]))

    def hidden(self, ids, ckpt: bool = False):
        cfg = self.cfg
        ids = ids.to(self.device)
        T = ids.shape[0]
        cos, sin = R.rope_tab(torch.arange(T, device=self.device), cfg.qk_rope_dim, cfg.rope_theta)
        h = self.W["embed"][ids].float()
        for l in range(len(self.W["layers"])):
            if ckpt and torch.is_grad_enabled():
                h = checkpoint(self._layer, l, h, cos, sin, use_reentrant=False)
            else:
                h = self._layer(l, h, cos, sin)
        return R.rms(h, self.W["norm"], cfg.rms_eps)

    @property
    def lm_head(self):
        return self.W["lm_head"]

    def logits(self, ids):
        return self.hidden(ids) @ self.lm_head.float().t()

    def param_groups(self, lr_scales=3e-4, lr_router=1.5e-5, lr_norms=1e-5):
        g = [{"params": [p for m in self.moe.values() for p in (m.t_gu, m.t_d)], "lr": lr_scales, "name": "scales"},
             {"params": [m.router for m in self.moe.values()], "lr": lr_router, "name": "router"}]
        if len(self.norms):
            g.append({"params": list(self.norms), "lr": lr_norms, "name": "norms"})
        return g

    def export_scales(self) -> dict:
        """{layer: {"gu_s", "d_s"} fp16} of the MoE layers (same export as the FN student)."""
        out = {}
        with torch.no_grad():
            for l, m in self.moe.items():
                s_gu, s_d = m.scales()
                out[int(l)] = {"gu_s": s_gu.half().cpu(), "d_s": s_d.half().cpu()}
        return out


# ------------------------------------------------------------------------------------------- objectives
def sft_loss(model, ids: torch.Tensor, resp_start: int, chunk: int = 1024) -> torch.Tensor:
    """Mean cross-entropy of the response tokens ids[resp_start:] (reference train.py CE objective)."""
    ids = ids.to(model.device)
    h = model.hidden(ids, ckpt=True)
    tgt = ids[resp_start:]
    tot = h.new_zeros(())
    for a in range(resp_start, ids.shape[0], chunk):
        b = min(ids.shape[0], a + chunk)
        lg = h[a - 1:b - 1] @ model.lm_head.float().t()
        tot = tot + F.cross_entropy(lg.float(), ids[a:b].long(), reduction="sum")
    return tot / max(1, tgt.numel())


def kd_topk_loss(student_logits: torch.Tensor, t_ids: torch.Tensor, t_logprobs: torch.Tensor) -> torch.Tensor:
    """KL(teacher || student) over the teacher's top-k tokens plus one tail bin (the reference's 21-bin top-20
    KL, flashnext/training/kd/train_kd.py). student_logits [n, V]; t_ids, t_logprobs [n, k]."""
    ls = torch.log_softmax(student_logits.float(), -1)
    ps_top = ls.gather(1, t_ids.long())
    pt_top = t_logprobs.float().exp()
    tail_t = (1 - pt_top.sum(-1)).clamp_min(1e-8)
    tail_s = (1 - ps_top.exp().sum(-1)).clamp_min(1e-8)
    kl = (pt_top * (t_logprobs.float() - ps_top)).sum(-1) + tail_t * (tail_t.log() - tail_s.log())
    return kl.mean()

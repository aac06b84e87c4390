"""Differentiable low-bit experts: frozen integer codes, trainable per-group scales.

The reference trains the fp16 group scales of its GPTQ experts (w = s * (q - z)) through a torch autograd
function whose backward forms dL/dW with a grouped GEMM and reduces it against (q - z) per 128-column group
(flashnext/training/student/student_fn.py:110-131 `LowbitLinear`, :133-189 `Bank`, :191-228 `GroupedExperts`).

Here the experts stay in the runtime tile-block layout the serving kernels use (one packed buffer per
projection, all experts and bit widths together), and:

* forward: ``blk_set_scales`` writes the current scales into the blocks (fp16, exactly what serving will see
  after export), then the tcgen05 weight-dequant GEMM (``wgemm.grouped``) runs gate_up and down for all experts
  in one launch each;
* backward: per chunk of experts, ``blk_dequant`` materializes bf16 W for the data-gradient GEMMs, the weight
  gradient GEMMs run per expert (cuBLAS), and ``blk_scale_grad`` reduces dL/dW against the packed codes into
  dL/ds without a dequantized (q - z) tensor.

CPU tensors take plain torch paths with identical math (tests compare the two).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..formats import runtime as rt
from ..ops import native, wgemm

CHUNK = 64  # experts per dequantized chunk in backward


class ExpertBank:
    """Frozen codes of one MoE layer (runtime blocks, natural row order: gate_up rows = [gate I; up I]) plus the
    base scales s0 [E, R, K/128] read from the blocks."""

    def __init__(self, gu: wgemm.WeightSet, d: wgemm.WeightSet):
        if any(f > 4 for f in gu.fmts + d.fmts):
            raise ValueError("trainable experts must be 2/3/4-bit")
        self.ws = {"gu": gu, "d": d}
        self.s0 = {n: torch.stack([rt.block_scales(self._blob(n, e), ws.fmts[e], ws.rows)
                                   for e in range(ws.n_experts)]) for n, ws in self.ws.items()}
        self.E = gu.n_experts

    @staticmethod
    def from_lowbit(layer, device) -> "ExpertBank":
        gu, d, fmts = [], [], []
        for b in layer.blobs:
            gu.append(rt.pack_planar_blob(b.gu, b.gu_s, b.gu_z, b.bits))
            d.append(rt.pack_planar_blob(b.d, b.d_s, b.d_z, b.bits))
            fmts.append(b.bits)
        I2, H = layer.blobs[0].gu_s.shape[0], layer.blobs[0].gu_s.shape[1] * rt.G
        return ExpertBank(wgemm.build_weight_set(gu, fmts, I2, H, device=device),
                          wgemm.build_weight_set(d, fmts, H, I2 // 2, device=device))

    def _blob(self, name, e):
        ws = self.ws[name]
        f = ws.fmts[e]
        n = ws.row_tiles * ws.kg * rt.block_bytes(f)
        off = int(ws.exp_off[e])
        return ws.blob[off: off + n].view(ws.row_tiles, ws.kg, rt.block_bytes(f))

    # -------------------------------------------------------------------------------------- primitives
    def set_scales(self, name: str, s: torch.Tensor) -> None:
        """Store fp16(s) [E, R, KG] in the blocks of projection `name`."""
        ws = self.ws[name]
        s = s.detach().float().contiguous()
        if ws.blob.is_cuda:
            native.C().blk_set_scales(ws.blob, ws.exp_off, ws.exp_fmt, s, ws.row_tiles, ws.kg)
            return
        Rp = ws.row_tiles * rt.TILE
        for e in range(ws.n_experts):
            blk = self._blob(name, e)
            nw = rt.FMT_WORDS[ws.fmts[e]]
            sp = torch.zeros(Rp, ws.kg)
            sp[: ws.rows] = s[e]
            h = sp.half().view(ws.row_tiles, rt.TILE, ws.kg).permute(0, 2, 1).contiguous()
            blk[..., nw * 512: nw * 512 + 256] = h.view(torch.uint8).view(ws.row_tiles, ws.kg, 256)

    def dequant(self, name: str, sel: list, s_sel: torch.Tensor) -> torch.Tensor:
        """W = s * (q - z) for experts `sel`: [n, R, K] (bf16 on GPU, fp32 on CPU)."""
        ws = self.ws[name]
        if ws.blob.is_cuda:
            out = torch.empty(len(sel), ws.rows, ws.K, dtype=torch.bfloat16, device=ws.blob.device)
            idx = torch.tensor(sel, dtype=torch.int32, device=ws.blob.device)
            native.C().blk_dequant(ws.blob, ws.exp_off, ws.exp_fmt, idx, s_sel.float().contiguous(), ws.row_tiles,
                                   ws.kg, out)
            return out
        return torch.stack([self.qz(name, e) * s_sel[i].float().repeat_interleave(rt.G, 1)
                            for i, e in enumerate(sel)])

    def scale_grad(self, name: str, sel: list, dW: torch.Tensor) -> torch.Tensor:
        """dL/ds [n, R, KG] = sum over each 128-column group of dL/dW * (q - z)."""
        ws = self.ws[name]
        if ws.blob.is_cuda:
            ds = torch.empty(len(sel), ws.rows, ws.kg, dtype=torch.float32, device=ws.blob.device)
            idx = torch.tensor(sel, dtype=torch.int32, device=ws.blob.device)
            native.C().blk_scale_grad(ws.blob, ws.exp_off, ws.exp_fmt, idx, dW.contiguous(), ws.row_tiles, ws.kg, ds)
            return ds
        return torch.stack([(dW[i].float() * self.qz(name, e)).view(ws.rows, ws.kg, rt.G).sum(-1)
                            for i, e in enumerate(sel)])

    def qz(self, name: str, e: int) -> torch.Tensor:
        ws = self.ws[name]
        return rt.unpack_qz(self._blob(name, e), ws.fmts[e], ws.rows, ws.K)


def _items(counts: list, n_tile: int, device):
    """Host-side plan of the grouped GEMM (token counts per expert are known on the host in training)."""
    items, start = [], 0
    for e, c in enumerate(counts):
        for s0 in range(0, c, n_tile):
            items.append([e, start + s0, min(n_tile, c - s0), 0])
        start += c
    it = torch.tensor(items or [[0, 0, 0, 0]], dtype=torch.int32, device=device)
    return it, torch.tensor([len(items)], dtype=torch.int32, device=device)


def _silu_mul(h):
    g, u = h.chunk(2, -1)
    return F.silu(g) * u


class GroupedExperts(torch.autograd.Function):
    """y[rows of expert e] = (silu(x W_gu,e^T)_gate * (x W_gu,e^T)_up) W_d,e^T for expert-sorted rows xs."""

    @staticmethod
    def forward(ctx, xs, s_gu, s_d, counts, bank: ExpertBank):
        ctx.counts, ctx.bank = list(counts), bank
        P = xs.shape[0]
        gu, d = bank.ws["gu"], bank.ws["d"]
        if xs.is_cuda:
            bank.set_scales("gu", s_gu)
            bank.set_scales("d", s_d)
            n_tile = 64 if P >= 64 * bank.E else 16
            items, n_items = _items(ctx.counts, n_tile, xs.device)
            h = torch.empty(P, gu.rows, dtype=torch.float32, device=xs.device)
            wgemm.grouped(xs.half().contiguous(), gu, items, n_items, items.shape[0], h, n_tile=n_tile)
            act = _silu_mul(h)
            y = torch.empty(P, d.rows, dtype=torch.float32, device=xs.device)
            wgemm.grouped(act.half().contiguous(), d, items, n_items, items.shape[0], y, n_tile=n_tile)
        else:
            h = torch.empty(P, gu.rows)
            y = torch.empty(P, d.rows)
            a = 0
            for e, c in enumerate(ctx.counts):
                if c:
                    Wg = bank.dequant("gu", [e], s_gu[e:e + 1])[0]
                    Wd = bank.dequant("d", [e], s_d[e:e + 1])[0]
                    h[a:a + c] = xs[a:a + c].float() @ Wg.t()
                    y[a:a + c] = _silu_mul(h[a:a + c]) @ Wd.t()
                a += c
        ctx.save_for_backward(xs, h, s_gu, s_d)
        return y

    @staticmethod
    def backward(ctx, dy):
        xs, h, s_gu, s_d = ctx.saved_tensors
        bank, counts = ctx.bank, ctx.counts
        cuda = xs.is_cuda
        cdt = torch.bfloat16 if cuda else torch.float32
        dy = dy.to(cdt).contiguous()
        xs_c = xs.to(cdt)
        g, u = h.float().chunk(2, -1)
        sg = torch.sigmoid(g)
        act = (g * sg * u).to(cdt)
        dx = torch.zeros(xs.shape, dtype=torch.float32, device=xs.device)
        ds_gu = torch.zeros_like(s_gu, dtype=torch.float32)
        ds_d = torch.zeros_like(s_d, dtype=torch.float32)
        starts = [0]
        for c in counts:
            starts.append(starts[-1] + c)
        live = [e for e, c in enumerate(counts) if c]
        for a in range(0, len(live), CHUNK):
            sel = live[a:a + CHUNK]
            Wd = bank.dequant("d", sel, s_d[sel])
            Wgu = bank.dequant("gu", sel, s_gu[sel])
            dWd = torch.empty(len(sel), *Wd.shape[1:], dtype=cdt, device=xs.device)
            dWgu = torch.empty(len(sel), *Wgu.shape[1:], dtype=cdt, device=xs.device)
            for i, e in enumerate(sel):
                r0, r1 = starts[e], starts[e + 1]
                dact = (dy[r0:r1] @ Wd[i].to(cdt)).float()
                dWd[i] = dy[r0:r1].t() @ act[r0:r1]
                gg, uu, ss = g[r0:r1], u[r0:r1], sg[r0:r1]
                dg = dact * uu * (ss * (1 + gg * (1 - ss)))
                du = dact * gg * ss
                dh = torch.cat([dg, du], -1).to(cdt)
                dx[r0:r1] = (dh @ Wgu[i].to(cdt)).float()
                dWgu[i] = dh.t() @ xs_c[r0:r1]
            if ctx.needs_input_grad[2]:
                ds_d[sel] = bank.scale_grad("d", sel, dWd)
            if ctx.needs_input_grad[1]:
                ds_gu[sel] = bank.scale_grad("gu", sel, dWgu)
        return dx.to(xs.dtype), ds_gu, ds_d, None, None


def grouped_experts(xs, s_gu, s_d, counts, bank):
    return GroupedExperts.apply(xs, s_gu, s_d, counts, bank)

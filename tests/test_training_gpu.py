"""Training kernels on the GPU against the CPU torch path: scale refresh, dequant, scale gradient, and the
grouped-expert autograd (forward on the tcgen05 GEMM)."""
import pytest
import torch

from arcagi2_flashnext_dots3_b200.config import fn_small_config
from arcagi2_flashnext_dots3_b200.models import fn_weights
from arcagi2_flashnext_dots3_b200.training.lowbit import ExpertBank, grouped_experts

pytestmark = pytest.mark.gpu


def _banks():
    cfg = fn_small_config(num_layers=1, ple_layers=(), n_experts=8, top_k=2)
    W = fn_weights.random_dense(cfg, seed=2, symmetric=False)
    lay = W["layers"][0]["moe"]["lowbit"]
    return cfg, ExpertBank.from_lowbit(lay, "cpu"), ExpertBank.from_lowbit(lay, "cuda")


def test_blk_kernels_match_cpu():
    cfg, bc, bg = _banks()
    g = torch.Generator().manual_seed(0)
    for name in ("gu", "d"):
        s = bc.s0[name] * (torch.randn(bc.s0[name].shape, generator=g) * 0.1).exp()
        sel = [5, 0, 3]
        wc = bc.dequant(name, sel, s[sel])
        wg = bg.dequant(name, sel, s[sel].cuda())
        assert torch.allclose(wg.float().cpu(), wc, rtol=1e-2, atol=1e-5)
        dW = torch.randn(wc.shape, generator=g)
        for dt in (torch.float32, torch.bfloat16):
            dsc = bc.scale_grad(name, sel, dW.to(dt).float())
            dsg = bg.scale_grad(name, sel, dW.to(dt).cuda())
            assert torch.allclose(dsg.cpu(), dsc, rtol=1e-4, atol=1e-3)
        bg.set_scales(name, s.cuda())
        bc.set_scales(name, s)
        assert torch.equal(bg.ws[name].blob.cpu(), bc.ws[name].blob)


def test_grouped_experts_gpu_vs_cpu():
    cfg, bc, bg = _banks()
    counts = [7, 0, 20, 3, 1, 33, 0, 9]
    P = sum(counts)
    g = torch.Generator().manual_seed(1)
    xs = torch.randn(P, cfg.hidden_size, generator=g)
    t_gu = torch.randn(bc.s0["gu"].shape, generator=g) * 0.05
    t_d = torch.randn(bc.s0["d"].shape, generator=g) * 0.05
    dy = torch.randn(P, cfg.hidden_size, generator=g)
    res = []
    for bank, dev in ((bc, "cpu"), (bg, "cuda")):
        x = xs.detach().clone().to(dev).requires_grad_()
        a = t_gu.detach().clone().to(dev).requires_grad_()
        b = t_d.detach().clone().to(dev).requires_grad_()
        y = grouped_experts(x, bank.s0["gu"].to(dev) * a.exp(), bank.s0["d"].to(dev) * b.exp(), counts, bank)
        (y * dy.to(dev)).sum().backward()
        res.append([t.detach().float().cpu() for t in (y, x.grad, a.grad, b.grad)])
    for c, gp in zip(*res):
        scale = c.abs().max()
        assert (gp - c).abs().max() <= 3e-2 * scale, ((gp - c).abs().max(), scale)


def test_smoke_entry():
    from arcagi2_flashnext_dots3_b200.launch.smoke import run_smoke
    r = run_smoke()
    assert r["grad_norm"] > 0 and len(r["decoded"]) == 2

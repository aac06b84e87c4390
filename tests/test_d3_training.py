"""D3 student on CPU: logits equal the oracle's, SFT and top-k distillation losses backpropagate into the
trainable scales, router and norms."""
import torch

from arcagi2_flashnext_dots3_b200.config import d3_small_config
from arcagi2_flashnext_dots3_b200.models import d3_reference as R
from arcagi2_flashnext_dots3_b200.models.d3_weights import random_dense
from arcagi2_flashnext_dots3_b200.training.d3_student import D3Student, kd_topk_loss, sft_loss


def test_d3_student_matches_oracle_and_trains():
    cfg = d3_small_config(num_layers=3)
    W = random_dense(cfg, seed=1)
    st = D3Student(cfg, W, "cpu", train_norms=True)
    ids = torch.randint(0, cfg.vocab_size, (26,), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        a = st.logits(ids)
    b = R.forward(W, cfg, ids)
    assert (a - b).abs().max() <= 2e-3 * b.abs().max()
    loss = sft_loss(st, ids, 10, chunk=7)
    loss.backward()
    for p in st.parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all()
    assert any(float(m.t_gu.grad.abs().sum()) > 0 for m in st.moe.values())


def test_kd_topk_loss_zero_at_teacher():
    g = torch.Generator().manual_seed(0)
    lg = torch.randn(5, 50, generator=g)
    lp = torch.log_softmax(lg, -1)
    top = lp.topk(20, -1)
    assert kd_topk_loss(lg, top.indices, top.values).abs() < 1e-5
    assert kd_topk_loss(lg + torch.randn(5, 50, generator=g), top.indices, top.values) > 1e-3

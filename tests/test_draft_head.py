"""Draft-head (MTP) training on CPU: the objective rises under training, and the exported head served by the
engine's MTPHead gives the same logits as the training module."""
import torch

from arcagi2_flashnext_dots3_b200.config import fn_small_config
from arcagi2_flashnext_dots3_b200.models import fn_weights
from arcagi2_flashnext_dots3_b200.models.fn_mtp import MTPHead, mtp_to_engine, random_mtp_dense
from arcagi2_flashnext_dots3_b200.training.draft_head import DraftHeadTrain, draft_objective, hot_vocab, \
    train_draft_head
from arcagi2_flashnext_dots3_b200.training.student import FNStudent


def _setup(hot=None):
    cfg = fn_small_config(num_layers=2, ple_layers=())
    main = fn_weights.random_dense(cfg, seed=3, symmetric=False)
    mtp = random_mtp_dense(cfg, seed=9)
    student = FNStudent(cfg, main, "cpu")
    ids = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        h = student.hidden(ids)
        tl = h @ student.lm_head.float().t()
    return cfg, main, mtp, ids, h, tl


def test_draft_head_training_raises_expected_accepted_length():
    cfg, main, mtp, ids, h, tl = _setup()
    hot = hot_vocab(torch.bincount(ids, minlength=cfg.vocab_size) + torch.rand(cfg.vocab_size), 512)
    m = DraftHeadTrain(cfg, main, mtp, "cpu", hot_ids=hot)
    _, e0 = draft_objective(m, h, ids, tl)
    hist = train_draft_head(m, iter(lambda: [(h, ids, tl)], None), steps=12, lr_dense=3e-3)
    assert hist[-1][1] > float(e0) * 1.2, (float(e0), hist[-1])
    assert hist[-1][0] < hist[0][0]


def test_exported_head_serves_like_training_module():
    cfg, main, mtp, ids, h, _ = _setup()
    m = DraftHeadTrain(cfg, main, mtp, "cpu")
    with torch.no_grad():
        # a changed parameter must survive the export; it is kept on the FP8 grid the export stores it in, so
        # both sides multiply the same values
        from arcagi2_flashnext_dots3_b200.models.fn_mtp import mtp_config
        g = torch.Generator().manual_seed(11)
        m.fc.copy_(fn_weights._round_dense(m.fc + 0.01 * torch.randn(m.fc.shape, generator=g), mtp_config(cfg)))
        x_train = m.step(h[:20], ids[1:21], 0)
        lg_train = m.logits(x_train)
    ex = m.export()
    main_eng = fn_weights.to_engine(main, cfg, "cpu")
    head = MTPHead(cfg, main_eng, mtp_to_engine(ex["dense"], cfg, main, "cpu"), "cpu", n_slots=1, max_len=64,
                   block_size=16)
    from arcagi2_flashnext_dots3_b200.engine.block_manager import BlockAllocator
    head.assign_blocks(0, 40, BlockAllocator(head.caches.n_blocks, 1))
    x_eng = head.step(h[:20], ids[1:21].to(torch.int32), torch.tensor([0], dtype=torch.int32),
                      torch.tensor([0], dtype=torch.int32), 20)
    lg_eng = head.logits(x_eng).float()
    err = (lg_eng - lg_train).abs().max() / lg_train.abs().max()
    assert err < 3e-2, float(err)

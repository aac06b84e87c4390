"""Dots3-shaped model on CPU: the engine path (absorbed latent attention over the paged FP8 cache, DSA top-k,
sliding window, sigmoid routing) against the dense oracle, in chunked prefill and in decode."""
import torch

from arcagi2_flashnext_dots3_b200.config import d3_small_config
from arcagi2_flashnext_dots3_b200.engine.block_manager import BlockAllocator
from arcagi2_flashnext_dots3_b200.models import d3_reference as R
from arcagi2_flashnext_dots3_b200.models.d3 import D3Model, allocate_caches
from arcagi2_flashnext_dots3_b200.models.d3_weights import random_dense, to_engine
from arcagi2_flashnext_dots3_b200.ops import d3_ops


def _model(cfg, W, slots=2, max_len=64):
    c = allocate_caches(cfg, "cpu", slots, max_len, block_size=8)
    m = D3Model(cfg, to_engine(W, cfg, "cpu"), c, "cpu")
    return m, BlockAllocator(c.n_blocks, slots)


def test_route_matches_oracle_rule():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(7, 12, generator=g)
    bias = torch.randn(12, generator=g) * 0.1
    ids, w = d3_ops.route(logits, 12, bias, 3, 2.5)
    sc = torch.sigmoid(logits)
    ref = torch.topk(sc + bias, 3, -1).indices
    assert torch.equal(ids.long().sort(-1).values, ref.sort(-1).values)
    assert torch.allclose(w.sum(-1), torch.full((7,), 2.5))


def test_d3_engine_prefill_decode_matches_oracle():
    cfg = d3_small_config()
    W = random_dense(cfg, seed=0)
    m, alloc = _model(cfg, W)
    T = 30
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(1))
    m.assign_blocks(0, T + 4, alloc)
    s0 = torch.tensor([0], dtype=torch.int32)
    xs = [m.step(ids[:17], s0, torch.tensor([0], dtype=torch.int32), 17)]
    xs.append(m.step(ids[17:25], s0, torch.tensor([17], dtype=torch.int32), 8))
    for t in range(25, T):  # decode one token at a time
        xs.append(m.step(ids[t:t + 1], s0, torch.tensor([t], dtype=torch.int32), 1))
    lg = m.logits(torch.cat(xs))
    ref = R.forward(W, cfg, ids)
    err = (lg - ref).abs().max() / ref.abs().max()
    assert err < 2e-3, err
    assert cfg.index_topk < T and cfg.swa_window < T


def test_d3_two_sequences_batched_decode():
    cfg = d3_small_config()
    W = random_dense(cfg, seed=2)
    m, alloc = _model(cfg, W)
    g = torch.Generator().manual_seed(3)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (21, 26)]
    for s, q in enumerate(seqs):
        m.assign_blocks(s, 40, alloc)
        m.step(q[:-1], torch.tensor([s], dtype=torch.int32), torch.tensor([0], dtype=torch.int32), len(q) - 1)
    x = m.step(torch.stack([q[-1] for q in seqs]), torch.tensor([0, 1], dtype=torch.int32),
               torch.tensor([len(q) - 1 for q in seqs], dtype=torch.int32), 1)
    lg = m.logits(x)
    for i, q in enumerate(seqs):
        ref = R.forward(W, cfg, q)[-1]
        assert (lg[i] - ref).abs().max() < 2e-3 * ref.abs().max()


def test_index_share_reuses_topk_and_overlap_stats():
    """Index sharing: an 'S' DSA layer keeps no index-key cache and attends to the latest 'F' layer's top-k; the
    overlap statistic reads 1.0 between them and stays in [0, 1] between independent indexers."""
    import dataclasses
    from arcagi2_flashnext_dots3_b200.utils.observe import TopkOverlap
    base = d3_small_config()
    dsa = base.dsa_layers()
    assert len(dsa) == 2
    W = random_dense(base, seed=0)
    ids = torch.randint(0, base.vocab_size, (40,), generator=torch.Generator().manual_seed(2))
    res = {}
    for name, cfg in (("own", base), ("share", dataclasses.replace(base, index_share=True, dsa_pattern="FS"))):
        m, alloc = _model(cfg, W)
        m.overlap = TopkOverlap()
        m.assign_blocks(0, 44, alloc)
        x = m.step(ids, torch.tensor([0], dtype=torch.int32), torch.tensor([0], dtype=torch.int32), 40)
        m.overlap.end_step()
        res[name] = (x, m.overlap.table(), m)
    assert res["share"][2].c.idx[dsa[1]] is None and res["own"][2].c.idx[dsa[1]] is not None
    shared = res["share"][1][(dsa[0], dsa[1])]
    assert all(v == 1.0 for v in shared if v == v) and any(v == v for v in shared)
    own = [v for v in res["own"][1][(dsa[0], dsa[1])] if v == v]
    assert own and all(0.0 <= v <= 1.0 for v in own)
    try:
        dataclasses.replace(base, index_share=True, dsa_pattern="SF").shared_index_layers()
        raise AssertionError("pattern starting with S accepted")
    except ValueError:
        pass

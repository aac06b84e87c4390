"""BASELINE config 1 on CPU: tiny hybrid (GDN + attention) MoE with 4-bit GPTQ experts. The engine's incremental
path (prefill + 64-token greedy decode over paged KV / recurrent caches) must reproduce the dense fp32 oracle."""
import torch

from arcagi2_flashnext_dots3_b200.config import tiny_config
from arcagi2_flashnext_dots3_b200.engine.block_manager import PyBlockAllocator
from arcagi2_flashnext_dots3_b200.models import fn_reference as ref
from arcagi2_flashnext_dots3_b200.models import fn_weights
from arcagi2_flashnext_dots3_b200.models.fn import FNModel, allocate_caches


def _engine(cfg, W, n_slots=2, max_len=512):
    E = fn_weights.to_engine(W, cfg, "cpu")
    c = allocate_caches(cfg, "cpu", n_slots, max_len, block_size=16)
    return FNModel(cfg, E, c, "cpu"), PyBlockAllocator(c.n_blocks, n_slots)


def test_prefill_logits_match_oracle():
    cfg = tiny_config(num_layers=2)
    W = fn_weights.random_dense(cfg, seed=0)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (40,), generator=g)
    want = ref.forward(W, cfg, ids)
    m, alloc = _engine(cfg, W, 1)
    m.assign_blocks(0, 40, alloc)
    x = m.step(ids, torch.tensor([0]), torch.tensor([0]), n_tok=40)
    got = m.logits(x)
    assert torch.allclose(got, want, atol=2e-3, rtol=2e-3), (got - want).abs().max()


def test_sparse_indexer_matches_oracle():
    # budget small enough that later queries use the block indexer
    cfg = tiny_config(num_layers=2, indexer_budget=16, indexer_ratio=4)
    W = fn_weights.random_dense(cfg, seed=3)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (48,), generator=g)
    want = ref.forward(W, cfg, ids)
    m, alloc = _engine(cfg, W, 1)
    m.assign_blocks(0, 64, alloc)
    x = m.step(ids[:40], torch.tensor([0]), torch.tensor([0]), n_tok=40)
    got = [m.logits(x)]
    for p in range(40, 48):
        x = m.step(ids[p:p + 1], torch.tensor([0]), torch.tensor([p]), n_tok=1)
        got.append(m.logits(x))
    got = torch.cat(got)
    assert torch.allclose(got, want, atol=2e-3, rtol=2e-3), (got - want).abs().max()


def test_config1_greedy_decode_batch2():
    """Prefill then 64-token greedy decode for a batch of two 256-token prompts (ids uniform over [0, 32000))."""
    cfg = tiny_config()
    W = fn_weights.random_dense(cfg, seed=0)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 32000, (256,), generator=g) for _ in range(2)]
    n_new = 64
    m, alloc = _engine(cfg, W, 2, max_len=512)
    nxt = []
    for s, p in enumerate(prompts):
        m.assign_blocks(s, 256 + n_new, alloc)
        x = m.step(p, torch.tensor([s]), torch.tensor([0]), n_tok=256)
        nxt.append(int(m.logits(x)[-1].argmax()))
    outs = [[t] for t in nxt]
    slots = torch.tensor([0, 1])
    for i in range(1, n_new):
        ids = torch.tensor([o[-1] for o in outs])
        pos = torch.tensor([256 + i - 1] * 2)
        lg = m.logits(m.step(ids, slots, pos))
        for s in range(2):
            outs[s].append(int(lg[s].argmax()))
    # oracle: full recomputation; compare the greedy tokens and the last-step logits
    for s, p in enumerate(prompts):
        seq = torch.cat([p, torch.tensor(outs[s][:-1])])
        want_logits = ref.forward(W, cfg, seq)
        want_tokens = want_logits[255:].argmax(-1).tolist()
        assert want_tokens == outs[s], (s, [i for i, (a, b) in enumerate(zip(want_tokens, outs[s])) if a != b][:5])


def test_ple_engine_matches_oracle():
    """PLE layers (n-gram ids with eos restarts, FP8 table, gated dilated conv over the ring) in chunked prefill and
    decode against the full-sequence oracle."""
    from arcagi2_flashnext_dots3_b200.config import fn_small_config
    cfg = fn_small_config(num_layers=2, ple_layers=(0, 1), indexer_budget=1 << 20)
    W = fn_weights.random_dense(cfg, seed=6, symmetric=False)
    E = fn_weights.to_engine(W, cfg, "cpu")
    c = allocate_caches(cfg, "cpu", 2, 64, block_size=16)
    m = FNModel(cfg, E, c, "cpu")
    alloc = PyBlockAllocator(c.n_blocks, 2)
    ids = torch.randint(3, cfg.vocab_size, (23,), generator=torch.Generator().manual_seed(8))
    ids[9] = cfg.eos_token_id  # n-grams restart after an eos
    m.reset_slot(1)
    m.assign_blocks(1, 30, alloc)
    s = torch.tensor([1], dtype=torch.int32)
    xs = [m.step(ids[:6], s, torch.tensor([0], dtype=torch.int32), 6),
          m.step(ids[6:14], s, torch.tensor([6], dtype=torch.int32), 8)]
    for t in range(14, 23):
        xs.append(m.step(ids[t:t + 1], s, torch.tensor([t], dtype=torch.int32), 1))
    lg = m.logits(torch.cat(xs))
    want = ref.forward(W, cfg, ids)
    assert (lg - want).abs().max() <= 2e-3 * want.abs().max()

"""Speculative decoding on CPU: verify + commit reproduce plain greedy decoding exactly with any drafter (full
acceptance with an oracle drafter, partial with prompt lookup, MTP head drafts), including recurrent-state and
PLE-history rollback."""
import pytest
import torch

from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config, tiny_config
from arcagi2_flashnext_dots3_b200.engine.llm import LLM
from arcagi2_flashnext_dots3_b200.engine.spec import MTPDrafter, NgramDrafter, OracleDrafter, SpecDecoder
from arcagi2_flashnext_dots3_b200.models import fn_weights
from arcagi2_flashnext_dots3_b200.models.fn_mtp import MTPHead, random_mtp


def _setup(cfg, seed=0):
    W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=seed, symmetric=False), cfg, "cpu")
    ec = EngineConfig(max_seqs=3, max_model_len=160, block_size=16, graph_batch_sizes=(1, 2, 4))
    return W, ec


PROMPTS = [[5, 9, 11, 40, 7, 9, 11], [3, 8, 21, 13, 8, 21, 13, 8]]


@pytest.mark.parametrize("drafter", ["oracle", "ngram", "mtp"])
def test_spec_equals_greedy(drafter):
    cfg = fn_small_config(num_layers=2, ple_layers=(0,), indexer_budget=1 << 20)
    W, ec = _setup(cfg)
    want = LLM(cfg, W, "cpu", ec).generate(PROMPTS, max_new_tokens=12)
    llm = LLM(cfg, W, "cpu", ec)
    if drafter == "oracle":
        d = OracleDrafter({})
    elif drafter == "ngram":
        d = NgramDrafter()
    else:
        d = MTPDrafter(MTPHead(cfg, W, random_mtp(cfg, "cpu"), "cpu", 4, 160, block_size=16))
    sd = SpecDecoder(llm, d, k=3)
    if drafter == "oracle":
        d.cont = {tuple(p): w for p, w in zip(PROMPTS, want)}
    got = sd.generate(PROMPTS, max_new_tokens=12)
    assert got == want
    if drafter == "oracle":
        assert sd.stats["accepted"] == sd.stats["drafted"] or sd.acceptance > 3.0
    assert sd.stats["steps"] <= 12


def test_spec_hybrid_gdn_rollback():
    """tiny hybrid config (GDN layers): partial acceptance must roll back recurrent state exactly."""
    cfg = tiny_config(num_layers=4)
    W, ec = _setup(cfg, seed=3)
    want = LLM(cfg, W, "cpu", ec).generate(PROMPTS, max_new_tokens=10)
    got = SpecDecoder(LLM(cfg, W, "cpu", ec), NgramDrafter(), k=4).generate(PROMPTS, max_new_tokens=10)
    assert got == want


@pytest.mark.gpu
@pytest.mark.parametrize("drafter", ["ngram", "mtp"])
def test_spec_gpu_matches_greedy(drafter):
    """On the GPU the verify step (k+1 rows per sequence) and plain decode (1 row) take different GEMM tilings,
    so exact equality can break at near-ties; require a long common prefix and high overall agreement."""
    cfg = fn_small_config(num_layers=4, ple_layers=(0,))
    W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=0, symmetric=False), cfg, "cuda")
    ec = EngineConfig(max_seqs=3, max_model_len=256, block_size=16, graph_batch_sizes=(1, 2, 4))
    want = LLM(cfg, W, "cuda", ec).generate(PROMPTS, max_new_tokens=24)
    llm = LLM(cfg, W, "cuda", ec)
    d = NgramDrafter() if drafter == "ngram" else MTPDrafter(
        MTPHead(cfg, W, random_mtp(cfg, "cuda"), "cuda", 4, 256, block_size=16))
    got = SpecDecoder(llm, d, k=3).generate(PROMPTS, max_new_tokens=24)
    for g, w in zip(got, want):
        assert g[:4] == w[:4]
        assert sum(a == b for a, b in zip(g, w)) >= 0.8 * len(w)


def test_mtp_hot_vocab_drafts():
    """Hot-vocabulary draft head: with every token hot it drafts what the full head drafts; with a subset every
    draft lies in the subset and the speculative output still equals plain greedy decoding."""
    cfg = fn_small_config(num_layers=2, ple_layers=(0,), indexer_budget=1 << 20)
    W, ec = _setup(cfg)
    mtp = random_mtp(cfg, "cpu")
    x = torch.randn(5, cfg.hidden_size)
    full = MTPHead(cfg, W, mtp, "cpu", 4, 160, block_size=16)
    every = MTPHead(cfg, W, mtp, "cpu", 4, 160, block_size=16, hot_ids=torch.arange(cfg.vocab_size))
    # the hot head holds the fp16 tensor-core operands; the CPU full head dequantizes in fp32, so only near-ties
    # may differ
    assert int((full.draft_ids(x) == every.draft_ids(x)).sum()) >= 4
    hot = torch.arange(0, cfg.vocab_size, 3)
    sub = MTPHead(cfg, W, mtp, "cpu", 4, 160, block_size=16, hot_ids=hot)
    assert set(sub.draft_ids(x).tolist()) <= set(hot.tolist())
    want = LLM(cfg, W, "cpu", ec).generate(PROMPTS, max_new_tokens=8)
    assert SpecDecoder(LLM(cfg, W, "cpu", ec), MTPDrafter(sub), k=3).generate(PROMPTS, max_new_tokens=8) == want


@pytest.mark.gpu
def test_mtp_hot_vocab_drafts_gpu():
    """GPU hot-vocabulary head (FP8 subset of the LM head on the tcgen05 GEMM): drafts stay inside the subset and
    agree with the full-head argmax restricted to the subset."""
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=0, symmetric=False), cfg, "cuda")
    mtp = random_mtp(cfg, "cuda")
    hot = torch.arange(1, cfg.vocab_size, 2)
    head = MTPHead(cfg, W, mtp, "cuda", 2, 64, block_size=16, hot_ids=hot)
    x = (torch.randn(6, cfg.hidden_size, device="cuda")).half()
    got = head.draft_ids(x).cpu()
    assert set(got.tolist()) <= set(hot.tolist())
    full = head.logits(x).float().cpu()
    ref = hot[full[:, hot].argmax(-1)]
    agree = int((got == ref).sum())
    assert agree >= 5, (got.tolist(), ref.tolist())
    # the hot logits are the full head's logits at the hot rows (same operands; only the K-split order may differ)
    sub = head.inner._mm(x, head.ws_hot).float().cpu()
    torch.testing.assert_close(sub, full[:, hot], rtol=1e-4, atol=1e-4)


def test_speculative_accept_preserves_the_sampling_distribution():
    """With a point-mass draft, accept-with-p(d) + residual sampling emits tokens distributed as the model's
    temperature-scaled softmax (first emitted token over 20000 seeds, total variation < 0.015)."""
    from arcagi2_flashnext_dots3_b200.ops import sampling
    V, T = 6, 0.8
    lg = torch.tensor([[1.0, 0.2, -0.5, 2.0, 0.0, 1.5], [0.0] * 6], dtype=torch.float32)[None]   # k = 1
    p = torch.softmax(lg[0, 0] / T, -1)
    n = 20000
    counts = torch.zeros(V)
    # 20000 calls on tensors of a few elements: one intra-op thread (with a pool per parallel test worker, thread
    # hand-offs made each call hundreds of times slower than its ~0.5 ms)
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        for seed in range(n):
            acc, nxt = sampling.speculative_accept(lg, torch.tensor([[3]]), [T], [seed], [0])
            counts[3 if acc[0] == 1 else nxt[0]] += 1
    finally:
        torch.set_num_threads(threads)
    tv = 0.5 * float((counts / n - p).abs().sum())
    assert tv < 0.015, (tv, (counts / n).tolist(), p.tolist())   # sampling noise alone: ~0.005


def test_d3_mtp_speculative_decoding_equals_greedy_and_samples():
    """D3 with its MTP draft layer: speculative greedy decoding emits exactly the plain greedy tokens; sampled
    sequences go through rejection-sampling verification and finish."""
    from arcagi2_flashnext_dots3_b200.config import d3_small_config
    from arcagi2_flashnext_dots3_b200.models import d3_weights
    from arcagi2_flashnext_dots3_b200.models.d3 import D3Model
    from arcagi2_flashnext_dots3_b200.models.d3_mtp import D3MTPHead, random_d3_mtp
    from arcagi2_flashnext_dots3_b200.ops.sampling import SamplingParams
    cfg = d3_small_config()
    W = d3_weights.to_engine(d3_weights.random_dense(cfg, seed=3), cfg, "cpu")
    ec = EngineConfig(max_seqs=3, max_model_len=160, block_size=16, graph_batch_sizes=(1, 2, 4))
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (12, 19)]
    want = LLM(cfg, W, "cpu", ec, model_cls=D3Model).generate(prompts, max_new_tokens=10)
    llm = LLM(cfg, W, "cpu", ec, model_cls=D3Model)
    head = D3MTPHead(cfg, llm.model, random_d3_mtp(cfg, "cpu"), "cpu", 4, 160, block_size=16)
    sd = SpecDecoder(llm, MTPDrafter(head), k=3)
    assert sd.generate(prompts, max_new_tokens=10) == want
    llm2 = LLM(cfg, W, "cpu", ec, model_cls=D3Model)
    head2 = D3MTPHead(cfg, llm2.model, random_d3_mtp(cfg, "cpu"), "cpu", 4, 160, block_size=16)
    out = SpecDecoder(llm2, MTPDrafter(head2), k=2).generate(prompts, max_new_tokens=8,
                                                               sp=SamplingParams(temperature=0.9, seed=5))
    assert [len(o) for o in out] == [8, 8]


@pytest.mark.gpu
def test_d3_mtp_speculative_graph_equals_greedy_gpu():
    from arcagi2_flashnext_dots3_b200.config import d3_small_config
    from arcagi2_flashnext_dots3_b200.models import d3_weights
    from arcagi2_flashnext_dots3_b200.models.d3 import D3Model
    from arcagi2_flashnext_dots3_b200.models.d3_mtp import D3MTPHead, random_d3_mtp
    cfg = d3_small_config()
    W = d3_weights.to_engine(d3_weights.random_dense(cfg, seed=3), cfg, "cuda")
    ec = EngineConfig(max_seqs=3, max_model_len=160, block_size=16, graph_batch_sizes=(1, 2, 4))
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (12, 19)]
    want = LLM(cfg, W, "cuda", ec, model_cls=D3Model).generate(prompts, max_new_tokens=10)
    llm = LLM(cfg, W, "cuda", ec, model_cls=D3Model)
    head = D3MTPHead(cfg, llm.model, random_d3_mtp(cfg, "cuda"), "cuda", 4, 160, block_size=16)
    got = SpecDecoder(llm, MTPDrafter(head), k=3).generate(prompts, max_new_tokens=10)
    for g, w in zip(got, want):
        assert g[:4] == w[:4] and sum(a == b for a, b in zip(g, w)) >= 8

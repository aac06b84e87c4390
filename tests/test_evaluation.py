"""Evaluation tooling on CPU: pass@2 scoring and budget-limited replay, paired bootstrap, teacher-forced KL fidelity
between two engine models, degeneration flags and leaf-wise build comparison."""
import random

import torch

from arcagi2_flashnext_dots3_b200.evaluation import compare, degeneration, fidelity, paired, scoring

G1, G2 = [[1, 2]], [[3, 4]]


def _rec(task, grid, used, verified=True):
    return {"task": task, "n_test": 1, "used": used,
            "progs": [{"verified": verified, "tests": [grid], "n_ok": 2 if verified else 1, "n_train": 2}]}


def test_scoring_and_budget_replay():
    truth = {"a": [G1], "b": [G2]}
    recs = [_rec("a", G1, 100), _rec("a", G2, 100), _rec("a", G1, 100), _rec("b", G1, 500)]
    pool = scoring.Pool.from_records(recs, truth)
    s, tok = scoring.expected_scores(pool, pool.tasks, 1e9, draws=5)
    assert s == {"a": 1.0, "b": 0.0} and tok == 400
    s0, _ = scoring.expected_scores(pool, pool.tasks, 50, draws=5)
    assert s0 == {"a": 0.0, "b": 0.0}          # no sample fits: nothing submitted
    sub = {"a": [{"attempt_1": G2, "attempt_2": G1}]}
    assert scoring.score_submission(sub, truth) == {"a": 1.0, "b": 0.0}


def test_paired_bootstrap_interval():
    rng = random.Random(0)
    b = {f"t{i}": rng.random() for i in range(200)}
    a = {t: v + 0.1 for t, v in b.items()}
    diff, lo, hi = paired.paired_bootstrap(a, b)
    assert abs(diff - 10.0) < 1e-9 and lo <= 10.0 + 1e-9 and hi >= 10.0 - 1e-9
    a2 = {t: v + (0.2 if i % 2 else 0.0) for i, (t, v) in enumerate(b.items())}
    d2, lo2, hi2 = paired.paired_bootstrap(a2, b)
    assert lo2 < d2 < hi2 and lo2 > 0


def test_fidelity_zero_for_same_model_positive_for_perturbed():
    from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config
    from arcagi2_flashnext_dots3_b200.engine.llm import LLM
    from arcagi2_flashnext_dots3_b200.models import fn_weights
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.random_dense(cfg, seed=0, symmetric=False)
    ec = EngineConfig(max_seqs=2, max_model_len=128, block_size=16, graph_batch_sizes=(1,))
    ref = LLM(cfg, fn_weights.to_engine(W, cfg, "cpu"), "cpu", ec)
    same = LLM(cfg, fn_weights.to_engine(W, cfg, "cpu"), "cpu", ec)
    seqs = [torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(s)).tolist()
            for s in (1, 2)]
    r = fidelity.fidelity(ref, same, seqs, k=8, chunk=16)
    assert r["n"] == 78 and r["kl"] < 1e-6 and r["agree"] == 1.0
    W2 = dict(W)
    W2["lm_head"] = W["lm_head"] + torch.randn(W["lm_head"].shape, generator=torch.Generator().manual_seed(9)) * 0.05
    other = LLM(cfg, fn_weights.to_engine(W2, cfg, "cpu"), "cpu", ec)
    r2 = fidelity.fidelity(ref, other, seqs, k=8, chunk=16)
    assert r2["kl"] > 1e-4 and r2["kl_topk"] > 0 and r2["bands"][0]["n"] == 78
    assert len(ref.free_slots) == 2      # slots returned


def test_degeneration_flags():
    fine = "The grid rotates by 90 degrees and then the colours swap. " * 80
    dumps = "[[1, 2], [3, 4]]\n" * 300
    run = "1, 2, 3, " * 400
    s = degeneration.summarize([fine, dumps, run])
    assert s["map"] == ".XR" and s["degenerate"] == 2 and s["runaway"] == 1


def test_compare_trees():
    a = {"x": torch.ones(3), "y": [torch.zeros(2), 5], "z": torch.ones(1)}
    b = {"x": torch.ones(3), "y": [torch.tensor([0.0, 0.5]), 5]}
    r = compare.compare_trees(a, b)
    assert r["leaves"] == 4 and r["differ"] == 1 and r["missing"] == 1 and r["max_abs"]["y[0]"] == 0.5

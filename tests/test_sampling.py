"""Sampler: greedy / Gumbel-max / top-k-top-p rules on CPU (empirical frequencies against the target
distribution), and the CUDA kernel against the CPU implementation of the same hash (identical draws)."""
import numpy as np
import pytest
import torch

from arcagi2_flashnext_dots3_b200.ops import sampling


def _vec(B, T, k, p, seed0=0):
    return (torch.full((B,), T, dtype=torch.float32), torch.full((B,), k, dtype=torch.int32),
            torch.full((B,), p, dtype=torch.float32), torch.arange(seed0, seed0 + B, dtype=torch.int64),
            torch.zeros(B, dtype=torch.int64))


def test_greedy_and_logprob():
    x = torch.randn(4, 50, generator=torch.Generator().manual_seed(0))
    ids, lp = sampling.sample(x, *_vec(4, 0.0, 0, 1.0))
    assert torch.equal(ids.long(), x.argmax(-1))
    assert torch.allclose(lp, torch.log_softmax(x, -1).max(-1).values)


@pytest.mark.parametrize("k,p", [(0, 1.0), (5, 1.0), (0, 0.7), (8, 0.8)])
def test_frequencies_follow_the_target(k, p):
    V, N, T = 12, 4000, 0.8
    x = torch.randn(1, V, generator=torch.Generator().manual_seed(1)).repeat(N, 1)
    ids, _ = sampling.sample(x, *_vec(N, T, k, p))
    prob = torch.softmax(x[0] / T, -1).double()
    order = torch.argsort(prob, descending=True)
    keep = torch.zeros(V, dtype=torch.bool)
    kk = k if k > 0 else V
    cum = torch.cumsum(prob[order[:kk]] / prob[order[:kk]].sum(), 0)
    cut = int((cum >= p - 1e-9).nonzero()[0]) if p < 1 else kk - 1
    keep[order[: cut + 1]] = True
    target = torch.where(keep, prob, torch.zeros_like(prob))
    target /= target.sum()
    freq = torch.bincount(ids.long(), minlength=V).double() / N
    assert freq[~keep].sum() == 0
    assert (freq - target).abs().max() < 0.03


def test_uniform_in_open_interval():
    u = sampling.uniform(123, 4, np.arange(100000))
    assert u.min() > 0 and u.max() < 1 and abs(u.mean() - 0.5) < 0.01


@pytest.mark.gpu
@pytest.mark.parametrize("T,k,p", [(0.0, 0, 1.0), (1.0, 0, 1.0), (0.7, 40, 1.0), (1.0, 0, 0.9), (0.9, 100, 0.95)])
def test_gpu_matches_cpu(T, k, p):
    B, V = 64, 151936
    x = torch.randn(B, V, generator=torch.Generator().manual_seed(2)) * 3
    vec = _vec(B, T, k, p, seed0=11)
    a, la = sampling.sample(x, *vec)
    b, lb = sampling.sample(x.cuda(), *[t.cuda() for t in vec])
    mism = int((a != b.cpu()).sum())
    assert mism <= 1, mism
    assert torch.allclose(la, lb.cpu(), atol=2e-3)

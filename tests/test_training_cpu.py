"""Repair-training student on CPU: chunked gated delta rule vs the sequential oracle, student logits vs the
oracle model, and the low-bit expert autograd (dL/ds, dL/dx) vs autograd through a dense dequantization."""
import torch

from arcagi2_flashnext_dots3_b200.config import fn_small_config
from arcagi2_flashnext_dots3_b200.models import fn_reference as R
from arcagi2_flashnext_dots3_b200.models import fn_weights
from arcagi2_flashnext_dots3_b200.training.gdn_chunk import chunk_gated_delta_rule
from arcagi2_flashnext_dots3_b200.training.lowbit import ExpertBank, grouped_experts
from arcagi2_flashnext_dots3_b200.training.student import FNStudent, gdn_train, qsa_select_vec


def _seq_gdn(q, k, v, g, beta):
    H, T, dk = q.shape
    S = torch.zeros(H, dk, v.shape[-1], dtype=torch.float64)
    out = []
    for t in range(T):
        S = S * g[:, t].exp()[:, None, None]
        kv = torch.einsum("hkv,hk->hv", S, k[:, t])
        u = beta[:, t][:, None] * (v[:, t] - kv)
        S = S + k[:, t][:, :, None] * u[:, None, :]
        out.append(torch.einsum("hkv,hk->hv", S, q[:, t]))
    return torch.stack(out, 1), S


def test_chunk_gdn_matches_sequential():
    g0 = torch.Generator().manual_seed(0)
    H, T, dk, dv = 3, 150, 16, 24
    q = torch.randn(H, T, dk, generator=g0, dtype=torch.float64) * 0.3
    k = torch.nn.functional.normalize(torch.randn(H, T, dk, generator=g0, dtype=torch.float64), dim=-1)
    v = torch.randn(H, T, dv, generator=g0, dtype=torch.float64)
    g = -torch.rand(H, T, generator=g0, dtype=torch.float64) * 2
    beta = torch.rand(H, T, generator=g0, dtype=torch.float64)
    o_ref, S_ref = _seq_gdn(q, k, v, g, beta)
    o, S = chunk_gated_delta_rule(q, k, v, g, beta, chunk=32, return_state=True)
    assert torch.allclose(o, o_ref, atol=1e-9, rtol=1e-9)
    assert torch.allclose(S, S_ref, atol=1e-9, rtol=1e-9)


def _small():
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.random_dense(cfg, seed=3, symmetric=False)
    return cfg, W


def test_gdn_train_matches_oracle():
    cfg, W = _small()
    L = W["layers"][0]
    assert cfg.layer_kind(0) == "linear"
    x = torch.randn(37, cfg.hidden_size, generator=torch.Generator().manual_seed(1))
    assert torch.allclose(gdn_train(x, L["mix"], cfg), R.gdn(x, L["mix"], cfg), atol=1e-4, rtol=1e-4)


def test_qsa_select_vectorized_matches_oracle():
    cfg = fn_small_config(num_layers=2, ple_layers=(), indexer_budget=16)
    W = fn_weights.random_dense(cfg, seed=4, symmetric=False)
    p = W["layers"][1]["mix"]
    T = 96
    x = torch.randn(T, cfg.hidden_size, generator=torch.Generator().manual_seed(2))
    cos, sin = R.rope_cos_sin(torch.arange(T), cfg.rope_dim, cfg.rope_theta)
    a = R.qsa_select(x, p, cfg, cos, sin)
    b = qsa_select_vec(x, p, cfg, cos, sin, q_chunk=17)
    assert a is not None and torch.equal(a.sum(1), b.sum(1))
    # rows may differ only among blocks whose scores tie (relu makes exact zeros common)
    iH, iD, r = cfg.indexer_heads, cfg.indexer_dim, cfg.indexer_ratio
    q, kr = (x @ p["iqk"].t()).split([iH * iD, iD], -1)
    q = R.rope_part(R.rms1p(q.view(T, iH, iD), p["iqn"], cfg.rms_eps), cos, sin)
    nb = T // r
    kb = R.rms1p(kr[: nb * r].view(nb, r, iD).mean(1), p["ikn"], cfg.rms_eps)
    kb = R.rope_part(kb[:, None], cos[torch.arange(nb) * r], sin[torch.arange(nb) * r])[:, 0]
    for i in (a != b).any(1).nonzero().flatten().tolist():
        s = torch.relu(torch.einsum("hd,bd->hb", q[i], kb)).sum(0)
        assert torch.allclose(s[a[i]].sort().values, s[b[i]].sort().values, atol=1e-6)


def test_student_logits_match_oracle():
    cfg, W = _small()
    st = FNStudent(cfg, W, "cpu")
    ids = torch.randint(0, cfg.vocab_size, (41,), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        a = st.logits(ids)
    b = R.forward(W, cfg, ids)
    assert (a - b).abs().max() <= 1e-3 * b.abs().max()


def _dense_ref(bank, xs, s_gu, s_d, counts):
    ys, a = [], 0
    for e, c in enumerate(counts):
        Wg = bank.qz("gu", e) * s_gu[e].repeat_interleave(128, 1)
        Wd = bank.qz("d", e) * s_d[e].repeat_interleave(128, 1)
        h = xs[a:a + c] @ Wg.t()
        gg, uu = h.chunk(2, -1)
        ys.append((torch.nn.functional.silu(gg) * uu) @ Wd.t())
        a += c
    return torch.cat(ys)


def test_grouped_experts_grad_cpu():
    cfg, W = _small()
    bank = ExpertBank.from_lowbit(W["layers"][0]["moe"]["lowbit"], "cpu")
    E = bank.E
    counts = [3, 0, 5, 1, 2, 4, 0, 6][:E]
    P = sum(counts)
    g0 = torch.Generator().manual_seed(7)
    xs = torch.randn(P, cfg.hidden_size, generator=g0, requires_grad=True)
    t_gu = (torch.randn(bank.s0["gu"].shape, generator=g0) * 0.05).requires_grad_()
    t_d = (torch.randn(bank.s0["d"].shape, generator=g0) * 0.05).requires_grad_()
    dy = torch.randn(P, cfg.hidden_size, generator=g0)
    y = grouped_experts(xs, bank.s0["gu"] * t_gu.exp(), bank.s0["d"] * t_d.exp(), counts, bank)
    (y * dy).sum().backward()
    grads = [xs.grad.clone(), t_gu.grad.clone(), t_d.grad.clone()]
    for t in (xs, t_gu, t_d):
        t.grad = None
    y2 = _dense_ref(bank, xs, bank.s0["gu"] * t_gu.exp(), bank.s0["d"] * t_d.exp(), counts)
    assert torch.allclose(y, y2, atol=1e-4, rtol=1e-4)
    (y2 * dy).sum().backward()
    for a, b in zip(grads, [xs.grad, t_gu.grad, t_d.grad]):
        assert torch.allclose(a, b, atol=1e-4, rtol=1e-3), (a - b).abs().max()


def test_student_backward_reaches_all_trainables():
    cfg, W = _small()
    st = FNStudent(cfg, W, "cpu", train_norms=True)
    ids = torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(9))
    h = st.hidden(ids, ckpt=True)
    lp = torch.log_softmax(h[:-1] @ st.lm_head.t(), -1).gather(1, ids[1:, None]).sum()
    lp.backward()
    for p in st.parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all()
    assert any(float(m.t_gu.grad.abs().sum()) > 0 for m in st.moe)


def test_routing_capture_replay_feeds_keep_selection(tmp_path):
    """Teacher-forced replay through the engine with the capture hook: per-layer rows and logits on disk, routing
    counts consistent with top-k, and REAP keep selection from the captured rows."""
    from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config
    from arcagi2_flashnext_dots3_b200.engine.llm import LLM
    from arcagi2_flashnext_dots3_b200.models import fn_weights
    from arcagi2_flashnext_dots3_b200.training import capture, compress
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.random_dense(cfg, seed=0, symmetric=False)
    llm = LLM(cfg, fn_weights.to_engine(W, cfg, "cpu"), "cpu",
              EngineConfig(max_seqs=2, max_model_len=128, block_size=16, graph_batch_sizes=(1,)))
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n)).tolist()
            for n in (37, 50)]
    cap = capture.RoutingCapture(tmp_path, cfg.top_k, every=2, flush_rows=16)
    capture.replay(llm, seqs, cap, chunk=20)
    st = capture.load_stats(tmp_path)
    assert st["layers"] == [0, 1] and st["tokens"][0] == 87
    assert int(st["counts"][0].sum()) == 87 * cfg.top_k
    assert abs(float(st["wsum"][1].sum()) - 87) < 1e-4
    x, lg = capture.load_layer(tmp_path, 1)
    assert x.shape == (44, cfg.hidden_size) and lg.shape == (44, cfg.n_experts)
    experts = W["layers"][1]["moe"]["experts_dense"]
    sc = compress.reap_scores(x.float(), lg, experts, cfg.top_k)
    keep, cov = compress.select_keep(sc, cfg.n_experts // 2, st["wsum"][1])
    assert len(keep) == cfg.n_experts // 2 and 0 < cov <= 1 and float(sc.sum()) > 0

"""Tensor-core latent attention (csrc/k_mla.cu) against a plain fp32 PyTorch reference of the same op: DSA top-k
lists (with invalid entries), causal rows, sliding windows, prefill rows, key splits, padded head groups."""
import pytest
import torch

from arcagi2_flashnext_dots3_b200.ops import d3_ops, native

pytestmark = pytest.mark.gpu


def _reference(q_lat, q_pe, cache, block_table, slots, positions, n_tok, sel, window, scale):
    H, T, kvr = q_lat.shape
    bs = cache.shape[1]
    c = cache.float()
    out = torch.zeros(H, T, kvr, device=q_lat.device)
    for t in range(T):
        b = t // n_tok
        pos = int(positions[b]) + t % n_tok
        slot = int(slots[b])
        if sel is not None and int(sel[t, 0]) >= 0:
            p = sel[t].long()
            p = p[(p >= 0) & (p <= pos)]
        else:
            lo = max(0, pos - window + 1) if window > 0 else 0
            p = torch.arange(lo, pos + 1, device=q_lat.device)
        rows = c[block_table[slot, p // bs].long(), p % bs]                     # [n, kvr + dr]
        s = (q_lat[:, t].float() @ rows[:, :kvr].t() + q_pe[t].float() @ rows[:, kvr:].t()) * scale
        out[:, t] = torch.softmax(s, -1) @ rows[:, :kvr]
    return out


def _case(H, kvr, dr, n_slots, n_tok, ctx, bs=64, topk=0, window=0, seed=0, invalid=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = "cuda"
    max_blocks = (ctx + n_tok + bs - 1) // bs + 1
    n_blocks = n_slots * max_blocks
    cache = (torch.randn(n_blocks, bs, kvr + dr, generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
    perm = torch.randperm(n_blocks, generator=g, device=dev).to(torch.int32)
    block_table = perm.view(n_slots, max_blocks).contiguous()
    slots = torch.arange(n_slots, dtype=torch.int32, device=dev)
    positions = torch.randint(ctx // 2, ctx, (n_slots,), generator=g, device=dev).to(torch.int32)
    T = n_slots * n_tok
    q_lat = (torch.randn(H, T, kvr, generator=g, device=dev) * 0.3).bfloat16()
    q_pe = torch.randn(T, H, dr, generator=g, device=dev) * 0.3
    sel = None
    if topk:
        sel = torch.empty(T, topk, dtype=torch.int32, device=dev)
        for t in range(T):
            pos = int(positions[t // n_tok]) + t % n_tok
            k = min(topk, pos + 1)
            idx = torch.randperm(pos + 1, generator=g, device=dev)[:k].to(torch.int32)
            row = torch.full((topk,), -1, dtype=torch.int32, device=dev)
            row[:k] = idx
            if invalid and topk > 4:
                row[1] = -1
                row[3] = pos + 5   # past the row's position: must be ignored
            sel[t] = row
    scale = (128 + 64) ** -0.5
    return q_lat, q_pe, cache, block_table, slots, positions, n_tok, sel, window, scale


CASES = {
    "dsa_decode": dict(H=128, kvr=512, dr=64, n_slots=5, n_tok=1, ctx=400, topk=256, invalid=True),
    "dsa_causal": dict(H=128, kvr=512, dr=64, n_slots=3, n_tok=1, ctx=150),
    "swa_decode": dict(H=64, kvr=1024, dr=64, n_slots=4, n_tok=1, ctx=300, window=129),
    "prefill_rows": dict(H=32, kvr=512, dr=64, n_slots=1, n_tok=9, ctx=90),
    "small_heads": dict(H=4, kvr=128, dr=64, n_slots=2, n_tok=1, ctx=70, bs=16, window=33),
    "tp4_heads": dict(H=16, kvr=1024, dr=64, n_slots=3, n_tok=2, ctx=200, window=70),
}


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("splits", [0, 3])
def test_mla_tc_matches_reference(name, splits, monkeypatch):
    args = _case(**CASES[name])
    monkeypatch.setattr(d3_ops, "_MLA_SPLITS", splits)
    monkeypatch.setattr(d3_ops, "_MLA_CUDA_CORE", False)
    out = d3_ops.mla_attn(*args)
    torch.cuda.synchronize()
    native.check_error(torch.device("cuda"))
    ref = _reference(*args)
    err = (out.float() - ref).abs().max() / ref.abs().max()
    assert err < 2e-2, (name, float(err))


def test_mla_tc_matches_cuda_core_kernel(monkeypatch):
    args = _case(**CASES["dsa_decode"])
    monkeypatch.setattr(d3_ops, "_MLA_CUDA_CORE", False)
    a = d3_ops.mla_attn(*args)
    monkeypatch.setattr(d3_ops, "_MLA_CUDA_CORE", True)
    b = d3_ops.mla_attn(*args)
    torch.cuda.synchronize()
    native.check_error(torch.device("cuda"))
    assert (a.float() - b.float()).abs().max() / b.float().abs().max() < 2e-2


@pytest.mark.parametrize("iH,rows,ctx", [(64, 6, 3000), (16, 3, 300)])
def test_dsa_scores_tc_matches_reference(iH, rows, ctx, monkeypatch):
    """Indexer logits sum_h w_h relu(q_h . k_j) on tcgen05 against fp32 PyTorch; masked past each row's position."""
    g = torch.Generator(device="cuda").manual_seed(iH)
    iD, S, max_len = 128, rows + 1, ctx + 64
    keys = (torch.randn(S, max_len, iD, generator=g, device="cuda") * 0.5).bfloat16()
    iq = torch.randn(rows, iH, iD, generator=g, device="cuda") * 0.3
    iw = torch.rand(rows, iH, generator=g, device="cuda")
    slots = torch.randperm(S, generator=g, device="cuda")[:rows].to(torch.int32)
    positions = torch.randint(1, ctx, (rows,), generator=g, device="cuda").to(torch.int32)
    positions[0] = 5
    ld = (max_len + 255) // 256 * 256
    out = torch.empty(rows, ld, device="cuda")
    native.C().d3_dsa_scores_tc(iq, iw, keys, slots, positions, 1, out, native.err_word(torch.device("cuda")),
                                native.DEFAULT_TIMEOUT_NS)
    torch.cuda.synchronize()
    native.check_error(torch.device("cuda"))
    for r in range(rows):
        p = int(positions[r])
        k = keys[int(slots[r]), : p + 1].float()
        ref = (torch.relu(iq[r].bfloat16().float() @ k.t()) * iw[r][:, None]).sum(0)
        got = out[r, : p + 1]
        assert (got - ref).abs().max() / ref.abs().max() < 1e-3, r
        assert bool((out[r, p + 1:] == -torch.finfo(torch.float32).max).all())
    # the selection the engine builds on it agrees with the CUDA-core logits
    monkeypatch.setattr(d3_ops, "_DSA_CUDA_CORE", False)
    a = d3_ops.dsa_select(iq, iw, keys, slots, positions, 1, 64, max_len)
    monkeypatch.setattr(d3_ops, "_DSA_CUDA_CORE", True)
    b = d3_ops.dsa_select(iq, iw, keys, slots, positions, 1, 64, max_len)
    for r in range(1, rows):
        sa, sb = set(a[r].tolist()), set(b[r].tolist())
        assert len(sa & sb) >= 60, (r, len(sa & sb))

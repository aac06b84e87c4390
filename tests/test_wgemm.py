"""Weight-dequant tcgen05 GEMM vs a plain fp32 torch reference (GPU), and the CPU reference path."""
import pytest
import torch

from arcagi2_flashnext_dots3_b200.formats import runtime as rt
from arcagi2_flashnext_dots3_b200.ops import native, wgemm


def _expert_blob(R, K, bits, g):
    q = torch.randint(0, 1 << bits, (R, K), generator=g, dtype=torch.int32)
    s = (torch.rand(R, K // 128, generator=g) * 0.02 + 2e-3).half()
    z = torch.randint(0, 1 << bits, (R, K // 128), generator=g).to(torch.uint8)
    return rt.pack_q(q, s, z, bits)


def test_cpu_reference_dense():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(192, 256, generator=g) * 0.05
    ws = wgemm.dense_f16(w)
    x = torch.randn(5, 256, generator=g).half()
    y = wgemm.matmul(x, ws)
    assert torch.allclose(y, x.float() @ w.half().float().t(), atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [16, 8])
@pytest.mark.parametrize("T", [1, 7, 16, 40, 100, 300])
def test_dense_gemm(fmt, T):
    g = torch.Generator().manual_seed(T + fmt)
    R, K = 384, 512
    w = torch.randn(R, K, generator=g) * 0.05
    ws = (wgemm.dense_f16(w) if fmt == 16 else wgemm.dense_fp8(w)).to("cuda")
    x = torch.randn(T, K, generator=g).half()
    ref = x.float() @ ws.dense(0).cpu().t()
    # the weight-dequant kind::f16 GEMM (fp16 activations); FP8 weight sets reach it with an explicit launch plan,
    # their default route being the kind::f8f6f4 GEMM (tests/test_f8gemm.py)
    nt, ks = wgemm.dense_plan(T, ws)
    y = wgemm.matmul(x.cuda(), ws, n_tile=nt, k_splits=ks)
    torch.cuda.synchronize()
    native.check_error()
    assert torch.allclose(y.cpu(), ref, atol=2e-3, rtol=2e-3), (y.cpu() - ref).abs().max()


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 3, 2])
def test_grouped_lowbit(bits):
    g = torch.Generator().manual_seed(bits)
    E, R, K = 6, 256, 384
    blobs = [_expert_blob(R, K, bits, g) for _ in range(E)]
    ws = wgemm.build_weight_set(blobs, [bits] * E, R, K).to("cuda")
    counts = [3, 0, 17, 1, 40, 5]
    items, t0 = [], 0
    for e, c in enumerate(counts):
        for s in range(0, c, 16):
            items.append([e, t0 + s, min(16, c - s), 0])
        t0 += c
    P = t0
    x = torch.randn(P, K, generator=g).half()
    out = torch.zeros(P, R, device="cuda")
    it = torch.tensor(items, dtype=torch.int32, device="cuda")
    n = torch.tensor([len(items)], dtype=torch.int32, device="cuda")
    wgemm.grouped(x.cuda(), ws, it, n, len(items), out, n_tile=16)
    torch.cuda.synchronize()
    native.check_error()
    t0 = 0
    for e, c in enumerate(counts):
        ref = x[t0:t0 + c].float() @ ws.dense(e).cpu().t()
        assert torch.allclose(out[t0:t0 + c].cpu(), ref, atol=2e-2, rtol=1e-2), (e, (out[t0:t0 + c].cpu() - ref).abs().max())
        t0 += c


@pytest.mark.gpu
def test_grouped_mixed_bits_silu():
    g = torch.Generator().manual_seed(7)
    E, I, K = 4, 128, 256
    perm = rt.gate_up_perm(I)
    bits = [4, 3, 4, 3]
    blobs = []
    for b in bits:
        q = torch.randint(0, 1 << b, (2 * I, K), generator=g, dtype=torch.int32)[perm]
        s = (torch.rand(2 * I, K // 128, generator=g) * 0.02 + 2e-3).half()
        z = torch.randint(0, 1 << b, (2 * I, K // 128), generator=g).to(torch.uint8)
        blobs.append(rt.pack_q(q, s, z, b))
    ws = wgemm.build_weight_set(blobs, bits, 2 * I, K, silu_pairs=True).to("cuda")
    counts = [2, 5, 0, 9]
    items, t0 = [], 0
    for e, c in enumerate(counts):
        if c:
            items.append([e, t0, c, 0])
        t0 += c
    x = torch.randn(t0, K, generator=g).half()
    out = torch.zeros(t0, I, dtype=torch.float16, device="cuda")
    it = torch.tensor(items, dtype=torch.int32, device="cuda")
    n = torch.tensor([len(items)], dtype=torch.int32, device="cuda")
    wgemm.grouped(x.cuda(), ws, it, n, len(items), out, epi=wgemm.EPI_SILU_MUL, n_tile=16)
    torch.cuda.synchronize()
    native.check_error()
    t0 = 0
    for e, c in enumerate(counts):
        ref = wgemm._ref_apply(x[t0:t0 + c].float() @ ws.dense(e).cpu().t(), wgemm.EPI_SILU_MUL)
        assert torch.allclose(out[t0:t0 + c].float().cpu(), ref, atol=2e-2, rtol=2e-2)
        t0 += c


@pytest.mark.gpu
@pytest.mark.parametrize("R,K,T,ks", [(388, 10240, 64, 0), (2560, 6144, 64, 0), (256, 1024, 20, 3), (300, 2560, 1, 0)])
def test_dense_split_k_deterministic(R, K, T, ks):
    g = torch.Generator().manual_seed(R + T)
    w = torch.randn(R, K, generator=g) * 0.02
    ws = wgemm.dense_fp8(w).to("cuda")
    x = torch.randn(T, K, generator=g).half()
    ref = x.float() @ ws.dense(0).cpu().t()
    nt, ks = wgemm.dense_plan(T, ws) if ks == 0 else (None, ks)   # the kind::f16 GEMM's own plan
    y1 = wgemm.matmul(x.cuda(), ws, n_tile=nt, k_splits=ks)
    y2 = wgemm.matmul(x.cuda(), ws, n_tile=nt, k_splits=ks)
    torch.cuda.synchronize()
    native.check_error()
    assert torch.equal(y1, y2), "split-K result is not reproducible"
    assert torch.allclose(y1.cpu(), ref, atol=3e-3, rtol=3e-3), (y1.cpu() - ref).abs().max()


@pytest.mark.gpu
def test_split_k_silu_epilogue():
    g = torch.Generator().manual_seed(3)
    I, K, T = 128, 4096, 9
    w = torch.randn(2 * I, K, generator=g) * 0.02
    ws = wgemm.dense_f16(w[rt.gate_up_perm(I)], silu_pairs=True).to("cuda")
    x = torch.randn(T, K, generator=g).half()
    ref = wgemm._ref_apply(x.float() @ ws.dense(0).cpu().t(), wgemm.EPI_SILU_MUL)
    y = wgemm.matmul(x.cuda(), ws, epi=wgemm.EPI_SILU_MUL, out_dtype=torch.float32, k_splits=8)
    torch.cuda.synchronize()
    assert torch.allclose(y.cpu(), ref, atol=3e-3, rtol=3e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("epi", [0, 1])
def test_gemv_grouped_matches_reference(epi):
    """CUDA-core grouped GEMV (<= 8 tokens per item) on mixed 4/3/2-bit experts against the torch reference
    (same items, same blocks), store and silu*up epilogues, plus per-row destinations."""
    from arcagi2_flashnext_dots3_b200.formats import lowbit_file
    from arcagi2_flashnext_dots3_b200.formats import runtime as rt
    from arcagi2_flashnext_dots3_b200.ops import fn_ops, wgemm
    g = torch.Generator().manual_seed(3)
    E, H, I = 6, 384, 256
    lay = lowbit_file.random_layer(E, H, I, [4, 3, 2, 4, 3, 4], g, symmetric=False)
    perm = rt.gate_up_perm(I)
    if epi == 1:
        blobs = [rt.pack_planar_blob(b.gu, b.gu_s, b.gu_z, b.bits, row_perm=perm) for b in lay.blobs]
        ws = wgemm.build_weight_set(blobs, [b.bits for b in lay.blobs], 2 * I, H, silu_pairs=True, device="cuda")
        K, cols = H, I
    else:
        blobs = [rt.pack_planar_blob(b.d, b.d_s, b.d_z, b.bits) for b in lay.blobs]
        ws = wgemm.build_weight_set(blobs, [b.bits for b in lay.blobs], H, I, device="cuda")
        K, cols = I, H
    T, k = 13, 3
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32).cuda()
    P = T * k
    pair_pos, items, n_items = fn_ops.moe_plan(ids, E, 8, P // 8 + E + 1)
    xs = (torch.randn(P, K, generator=g) * 0.5).half().cuda()
    out_g = torch.zeros(P, cols, dtype=torch.float16 if epi else torch.float32, device="cuda")
    ref = wgemm.grouped(xs.float().cpu(), ws.to("cpu"), items.cpu(), n_items.cpu(), items.shape[0],
                        torch.zeros(P, cols), epi=epi)
    wgemm.gemv_grouped(xs, ws, items, n_items, items.shape[0], out_g, epi=epi)
    torch.cuda.synchronize()
    err = (out_g.float().cpu() - ref).abs().max() / ref.abs().max()
    assert err < 2e-2, err  # int8 activations per 128-column group
    if epi == 0:  # per-row destinations: rows land in a permuted buffer
        dst = torch.zeros(P, cols, dtype=torch.float32, device="cuda")
        perm_rows = torch.randperm(P, generator=g).cuda()
        addr = dst.data_ptr() + perm_rows.long() * cols * 4
        wgemm.gemv_grouped(xs, ws, items, n_items, items.shape[0], out_g, row_dst=addr)
        torch.cuda.synchronize()
        assert torch.allclose(dst[perm_rows].cpu(), out_g.cpu())


@pytest.mark.gpu
@pytest.mark.parametrize("epi", [0, 1])
@pytest.mark.parametrize("shape", [(6, 384, 256, 13, 3), (24, 2560, 640, 64, 6)])
def test_moe_i8_equals_gemv(epi, shape):
    """The tcgen05 kind::i8 grouped MoE kernel (codes widened into tensor memory, integer MMA) gives the CUDA-core
    GEMV's bits on mixed 4/3/2-bit experts: short rows (fewer groups than its fold lag) and FN-sized rows (20
    groups), items of 1..8 tokens, store and silu*up epilogues, per-row destinations."""
    from arcagi2_flashnext_dots3_b200.formats import lowbit_file
    from arcagi2_flashnext_dots3_b200.formats import runtime as rt
    from arcagi2_flashnext_dots3_b200.ops import fn_ops, wgemm
    E, H, I, T, k = shape
    g = torch.Generator().manual_seed(7 + E)
    lay = lowbit_file.random_layer(E, H, I, [(4, 3, 2)[e % 3] for e in range(E)], g, symmetric=False)
    if epi == 1:
        perm = rt.gate_up_perm(I)
        blobs = [rt.pack_planar_blob(b.gu, b.gu_s, b.gu_z, b.bits, row_perm=perm) for b in lay.blobs]
        ws = wgemm.build_weight_set(blobs, [b.bits for b in lay.blobs], 2 * I, H, silu_pairs=True, device="cuda")
        K, cols = H, I
    else:
        blobs = [rt.pack_planar_blob(b.d, b.d_s, b.d_z, b.bits) for b in lay.blobs]
        ws = wgemm.build_weight_set(blobs, [b.bits for b in lay.blobs], H, I, device="cuda")
        K, cols = I, H
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32).cuda()
    P = T * k
    mi = P // 8 + E + 1
    pair_pos, items, n_items = fn_ops.moe_plan(ids, E, 8, mi)
    xs = (torch.randn(P, K, generator=g) * 0.5).half().cuda()
    dt = torch.float16 if epi else torch.float32
    a = torch.zeros(P, cols, dtype=dt, device="cuda")
    b = torch.zeros(P, cols, dtype=dt, device="cuda")
    wgemm.gemv_grouped(xs, ws, items, n_items, mi, a, epi=epi, kernel="dp4a")
    wgemm.gemv_grouped(xs, ws, items, n_items, mi, b, epi=epi, kernel="i8")
    torch.cuda.synchronize()
    native.check_error()
    assert torch.equal(a, b), (a.float() - b.float()).abs().max()
    if epi == 0:
        dst = torch.zeros(P, cols, dtype=torch.float32, device="cuda")
        perm_rows = torch.randperm(P, generator=g).cuda()
        addr = dst.data_ptr() + perm_rows.long() * cols * 4
        wgemm.gemv_grouped(xs, ws, items, n_items, mi, b, row_dst=addr, kernel="i8")
        torch.cuda.synchronize()
        assert torch.equal(dst[perm_rows], a)


@pytest.mark.gpu
def test_moe_layer_fullsize_error_bound():
    """A full-size FN decode MoE layer (320 experts, hidden 2560, expert FFN 640, top-10, 4/3-bit, 64 tokens) on the
    decode path (int8 activations per 128-column group, fp16 intermediate) against an fp32 oracle on the same
    dequantized weights: the error this precision choice costs, bounded."""
    from arcagi2_flashnext_dots3_b200.config import fn_config
    from arcagi2_flashnext_dots3_b200.models import fn_weights
    from arcagi2_flashnext_dots3_b200.ops import fn_ops, wgemm
    cfg = fn_config()
    E, H, I, k, T = cfg.n_experts, cfg.hidden_size, cfg.moe_inter, cfg.top_k, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    gu, dn = fn_weights._random_experts(cfg, g, torch.device("cuda"))
    x = torch.randn(T, H, generator=g, device="cuda").half()
    ids, w = fn_ops.moe_route(torch.randn(T, E + 1, generator=g, device="cuda"), E, k)
    P = T * k
    n_tile = wgemm.GEMV_MAX_TOK
    max_items = (P + n_tile - 1) // n_tile + E
    pair_pos, items, n_items = fn_ops.moe_plan(ids, E, n_tile, max_items)
    xs = fn_ops.moe_scatter(x, pair_pos)
    act = torch.empty(P, I, dtype=torch.float16, device="cuda")
    ypair = torch.empty(P, H, dtype=torch.float32, device="cuda")
    wgemm.gemv_grouped(xs, gu, items, n_items, max_items, act, epi=wgemm.EPI_SILU_MUL)
    wgemm.gemv_grouped(act, dn, items, n_items, max_items, ypair)
    h = torch.zeros(T, H, dtype=torch.float32, device="cuda")
    fn_ops.moe_combine(h, ypair, pair_pos, w, torch.zeros(T, H, device="cuda"),
                       torch.full((T,), float("-inf"), device="cuda"), torch.ones(T, 1, device="cuda"))
    ref = torch.zeros(T, H, dtype=torch.float64, device="cuda")
    ids_l, x32 = ids.long(), x.float()
    for e in torch.unique(ids_l).tolist():
        t, j = (ids_l == e).nonzero(as_tuple=True)
        a = wgemm._ref_apply(x32[t] @ gu.dense(e).t(), wgemm.EPI_SILU_MUL)
        y = a @ dn.dense(e).t()
        ref.index_add_(0, t, (y * w[t, j, None]).double())
        gu._dense_cache = dn._dense_cache = None
    ref = ref.float()
    err = (h - ref).abs()
    rel_max = float(err.max() / ref.abs().max())
    rel_mean = float(err.mean() / ref.abs().mean())
    # measured on a B200: max 1.5% of max|y|, mean 1.6% of mean|y| (int8 activations; fp16 ones would give ~0.1%)
    assert rel_max < 3e-2 and rel_mean < 2.5e-2, (rel_max, rel_mean)

"""Dense FP8 GEMM on tcgen05 kind::f8f6f4 (csrc/k_f8gemm.cu) against fp32 references of the same op.

`f8_reference` forms the same e4m3 codes and exact products but sums them in fp32 in another order, so the two
agree to fp32 rounding (EMU_TOL, relative to the output's scale). On integer data with exact codes the kernel
must match exactly (`test_f8_linear_exact_on_integers`)."""
import pytest
import torch

EMU_TOL = 1e-4

from arcagi2_flashnext_dots3_b200.formats import runtime as rt
from arcagi2_flashnext_dots3_b200.ops import wgemm


def _ws(R, K, seed=0, silu=False, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(R, K, generator=g) * 0.05
    w[:, :128] *= 8.0                       # block scales differ across groups
    ws = wgemm.dense_fp8(w)
    if silu:
        ws.silu_pairs = True
    return ws.to(device) if device != "cpu" else ws


def test_fp8_rowmajor_matches_blocks():
    ws = _ws(300, 384)
    codes, sc = ws.f8_operands()
    assert codes.shape == (384, 384) and sc.shape == (3, 3)
    dense = codes.view(torch.float8_e4m3fn).float() * sc.repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert torch.equal(dense[:300], ws.dense(0))
    assert not codes[300:].any()


def test_f8_reference_close_to_fp32():
    ws = _ws(256, 512)
    x = torch.randn(5, 512)
    ref = x @ ws.dense(0).t()
    y = wgemm.f8_reference(x, ws)
    assert (y - ref).abs().max() / ref.abs().max() < 0.05


def test_f8_plan_one_wave():
    for R, K in ((16480, 2560), (2560, 6144), (388, 10240), (10240, 384), (321, 2560)):
        ws = _ws(R, K) if R * K < 3e6 else None
        if ws is None:
            ws = wgemm.WeightSet(torch.empty(0, dtype=torch.uint8), None, None, R, K, (8,))
        nt, s = wgemm.f8_plan(64, ws)
        assert nt == 64 and 1 <= s <= 8 and s <= K // 128
        assert ws.row_tiles * s <= 148 or s == 1


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 17, 64, 100, 300])
@pytest.mark.parametrize("R,K", [(388, 1280), (640, 2560), (2560, 640)])
def test_f8_linear_store(T, R, K):
    dev = torch.device("cuda")
    ws = _ws(R, K, seed=T, device=dev)
    x = torch.randn(T, K, device=dev, dtype=torch.float16)
    out = torch.empty(T, R, device=dev)
    wgemm.f8_linear(x, ws, out)
    torch.cuda.synchronize()
    ref = wgemm.f8_reference(x, ws)
    err = ((out - ref).abs().max() / ref.abs().max()).item()
    assert err < EMU_TOL, err
    full = x.float() @ ws.dense(0).t()
    assert ((out - full).abs().max() / full.abs().max()).item() < 0.05


@pytest.mark.gpu
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_f8_linear_splits_same_values(splits):
    dev = torch.device("cuda")
    ws = _ws(512, 2048, device=dev)
    x = torch.randn(64, 2048, device=dev, dtype=torch.bfloat16)
    out = torch.empty(64, 512, device=dev)
    wgemm.f8_linear(x, ws, out, nt=64, splits=splits)
    ref = wgemm.f8_reference(x, ws)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < EMU_TOL
    again = torch.empty_like(out)
    wgemm.f8_linear(x, ws, again, nt=64, splits=splits)
    assert torch.equal(out, again)                   # fixed reduction order: identical bits


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_f8_linear_silu_and_dtypes(out_dtype):
    dev = torch.device("cuda")
    ws = _ws(1280, 2560, silu=True, device=dev)
    x = torch.randn(64, 2560, device=dev, dtype=torch.float16)
    out = torch.empty(64, 640, device=dev, dtype=out_dtype)
    wgemm.f8_linear(x, ws, out, epi=wgemm.EPI_SILU_MUL)
    ref = wgemm.f8_reference(x, ws, epi=wgemm.EPI_SILU_MUL)
    assert ((out.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2


@pytest.mark.gpu
def test_f8_linear_accumulate_alpha_and_matmul_route():
    dev = torch.device("cuda")
    ws = _ws(2560, 1280, device=dev)
    x = torch.randn(40, 1280, device=dev, dtype=torch.float16)
    base = torch.randn(40, 2560, device=dev)
    out = base.clone()
    wgemm.f8_linear(x, ws, out, accumulate=True, alpha=0.5)
    ref = base + 0.5 * wgemm.f8_reference(x, ws)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < EMU_TOL
    y = wgemm.matmul(x, ws)                          # default dense FP8 route
    assert ((y - wgemm.f8_reference(x, ws)).abs().max() / y.abs().max()).item() < EMU_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("T,splits", [(5, 1), (5, 4), (70, 2)])
def test_f8_linear_exact_on_integers(T, splits):
    """Integer weights and activations whose e4m3 codes and scales are exact (every 128 x 128 weight block and
    every (token, group) of the activations holds one 448, so both scales are exactly 1) and whose products and
    sums stay far inside fp32's integer range: the kernel must return the exact integer result, whatever the K
    split or the token tile. Any layout, swizzle, scale or ordering slip shows up as a mismatch."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(T + splits)
    R, K = 256, 512
    w = torch.randint(-8, 9, (R, K), generator=g).float()
    for rb in range(R // 128):
        for kb in range(K // 128):
            w[rb * 128, kb * 128] = 448.0
    x = torch.randint(-4, 5, (T, K), generator=g).float()
    x[:, 1::128] = 448.0
    ws = wgemm.dense_fp8(w).to(dev)
    codes, sc = ws.f8_operands()
    assert torch.all(sc == 1.0)
    out = torch.empty(T, R, device=dev)
    wgemm.f8_linear(x.to(dev).half(), ws, out, nt=64 if T <= 64 else 128, splits=splits)
    torch.cuda.synchronize()
    want = (x.double() @ w.double().t()).float()
    assert torch.equal(out.cpu(), want), (out.cpu() - want).abs().max()

"""Chunked Gated DeltaNet prefill on tcgen05 (csrc/k_gdn_chunk.cu) against the sequential GPU recurrence (itself
checked against the torch statement in tests/test_fn_gpu.py): outputs, recurrent states and conv states after
prefill steps of whole and partial 64-token chunks, starting from a non-zero state."""
import dataclasses

import pytest
import torch

from arcagi2_flashnext_dots3_b200.config import fn_small_config
from arcagi2_flashnext_dots3_b200.ops import fn_ops, native

pytestmark = pytest.mark.gpu


def _case(n_tok, B, seed):
    cfg = dataclasses.replace(fn_small_config(), lin_v_heads=6)
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    C = 2 * nk * dk + nv * dv
    g = torch.Generator().manual_seed(seed)
    dev = "cuda"
    proj = torch.randn(B * n_tok, C + nv * dv + 2 * nv, generator=g).to(dev)
    conv_w = (torch.randn(C, cfg.conv_kernel, generator=g) * 0.4).to(dev)
    conv_state = torch.randn(B + 1, C, cfg.conv_kernel - 1, generator=g).to(dev)
    ssm = (torch.randn(B + 1, nv, dk, dv, generator=g) * 0.05).to(dev).bfloat16()
    A_log = torch.log(torch.rand(nv, generator=g) * 0.2 + 0.01).to(dev)
    dt_bias = (torch.randn(nv, generator=g) * 0.3).to(dev)
    norm_w = (torch.rand(dv, generator=g) + 0.5).to(dev)
    slots = torch.tensor([B - i for i in range(B)], dtype=torch.int32, device=dev)
    return cfg, proj, conv_w, conv_state, ssm, A_log, dt_bias, norm_w, slots


@pytest.mark.parametrize("n_tok,B", [(64, 1), (200, 2), (130, 1)])
def test_chunked_prefill_matches_sequential(n_tok, B):
    cfg, proj, conv_w, conv_state, ssm, A_log, dt_bias, norm_w, slots = _case(n_tok, B, n_tok + B)
    cs1, ss1 = conv_state.clone(), ssm.clone()
    cs2, ss2 = conv_state.clone(), ssm.clone()
    saved = fn_ops.GDN_CHUNK
    try:
        fn_ops.GDN_CHUNK = True
        got = fn_ops.gdn_step(proj, conv_w, cs1, ss1, A_log, dt_bias, norm_w, slots, cfg, n_tok)
        fn_ops.GDN_CHUNK = False
        want = fn_ops.gdn_step(proj, conv_w, cs2, ss2, A_log, dt_bias, norm_w, slots, cfg, n_tok)
    finally:
        fn_ops.GDN_CHUNK = saved
    torch.cuda.synchronize()
    native.check_error()
    rel = lambda x, y: ((x.float() - y.float()).abs().max() / y.float().abs().max()).item()
    assert rel(got, want) < 3e-2, rel(got, want)
    assert rel(ss1, ss2) < 3e-2, rel(ss1, ss2)
    assert torch.equal(cs1, cs2)
    # untouched slot keeps its state
    assert torch.equal(ss1[0], ssm[0]) if B == 1 else True


def test_chunked_prefill_then_decode_continues():
    """A chunked prefill followed by single-token decode steps gives the same outputs as a fully sequential run."""
    cfg, proj, conv_w, conv_state, ssm, A_log, dt_bias, norm_w, slots = _case(136, 1, 7)
    n_pre = 128
    outs = {}
    saved = fn_ops.GDN_CHUNK
    try:
        for chunked in (True, False):
            fn_ops.GDN_CHUNK = chunked
            cs, ss = conv_state.clone(), ssm.clone()
            o = [fn_ops.gdn_step(proj[:n_pre].contiguous(), conv_w, cs, ss, A_log, dt_bias, norm_w, slots, cfg,
                                 n_pre)]
            for t in range(n_pre, 136):
                o.append(fn_ops.gdn_step(proj[t:t + 1].contiguous(), conv_w, cs, ss, A_log, dt_bias, norm_w, slots,
                                         cfg, 1))
            outs[chunked] = torch.cat(o).float()
    finally:
        fn_ops.GDN_CHUNK = saved
    torch.cuda.synchronize()
    native.check_error()
    a, b = outs[True], outs[False]
    assert ((a - b).abs().max() / b.abs().max()).item() < 3e-2

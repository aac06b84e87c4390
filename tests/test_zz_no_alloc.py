"""The allocation-free indexer select (`fw_qsa_select_noalloc`, exported C symbol of the `_C` library).

Some callers cannot allocate device memory themselves (a host runtime that owns every allocation, a plugin
sandbox that forbids cudaMalloc). This entry point takes their input and output buffers and keeps its scratch
in a fixed file-scope device array. The test calls it through ctypes, as such a caller would, and checks it
against the regular (allocating) entry point on two calls in a row, so the reused scratch array is exercised.
It is collected last so a failure here cannot hide the results of the other tests.
"""
import ctypes

import pytest
import torch

from arcagi2_flashnext_dots3_b200.config import fn_small_config
from arcagi2_flashnext_dots3_b200.ops import fn_ops, native

pytestmark = pytest.mark.gpu


def _fn():
    lib = ctypes.CDLL(native.C().__file__)
    f = lib.fw_qsa_select_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 7 + [ctypes.c_void_p]
    cap = lib.fw_qsa_select_noalloc_max_floats
    cap.restype = ctypes.c_size_t
    return f, int(cap())


def _inputs(cfg, rows, n_tok, max_comp, seed):
    g = torch.Generator().manual_seed(seed)
    S = 4
    iq = torch.randn(rows, cfg.indexer_heads, cfg.indexer_dim, generator=g).cuda()
    comp = torch.randn(S, max_comp, cfg.indexer_dim, generator=g).bfloat16().cuda()
    B = rows // n_tok
    slots = torch.randint(0, S, (B,), generator=g, dtype=torch.int32).cuda()
    pos = torch.randint(0, max_comp * cfg.indexer_ratio - n_tok, (B,), generator=g, dtype=torch.int32).cuda()
    pos[0] = 10  # one row below the budget (not sparse)
    return iq, comp, slots, pos


def _call(f, cfg, iq, comp, slots, pos, n_tok):
    rows = iq.shape[0]
    nblk = min(cfg.indexer_blocks, comp.shape[1])
    sel = torch.full((rows, nblk), -7, dtype=torch.int32, device="cuda")
    sparse = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    rc = f(iq.data_ptr(), comp.data_ptr(), 1, slots.data_ptr(), pos.data_ptr(), sel.data_ptr(), sparse.data_ptr(),
           rows, cfg.indexer_heads, cfg.indexer_dim, comp.shape[1], nblk, cfg.indexer_ratio, n_tok,
           torch.cuda.current_stream().cuda_stream)
    return rc, sel, sparse


def test_noalloc_matches_allocating_entry_point_twice():
    f, _ = _fn()
    cfg = fn_small_config(indexer_budget=64)
    for call, (rows, n_tok, max_comp) in enumerate([(12, 1, 300), (10, 5, 700)]):
        iq, comp, slots, pos = _inputs(cfg, rows, n_tok, max_comp, seed=call)
        rc, sel, sparse = _call(f, cfg, iq, comp, slots, pos, n_tok)
        torch.cuda.synchronize()
        assert rc == 0, rc
        sel_ref, sp_ref = fn_ops.qsa_select(iq, comp, slots, pos, cfg, n_tok)
        torch.cuda.synchronize()
        assert torch.equal(sparse.cpu(), sp_ref.cpu())
        assert int(sparse.cpu().sum()) > 0
        for r in range(rows):
            assert set(sel[r].cpu().tolist()) == set(sel_ref[r].cpu().tolist()), (call, r)


def test_noalloc_rejects_oversize_request():
    f, cap = _fn()
    cfg = fn_small_config(indexer_budget=64)
    max_comp = 1024
    rows = cap // max_comp + 1
    iq = torch.zeros(1, device="cuda")
    rc = f(iq.data_ptr(), iq.data_ptr(), 1, iq.data_ptr(), iq.data_ptr(), iq.data_ptr(), iq.data_ptr(), rows,
           cfg.indexer_heads, cfg.indexer_dim, max_comp, 16, cfg.indexer_ratio, 1,
           torch.cuda.current_stream().cuda_stream)
    assert rc == 2


def test_noalloc_rejects_misaligned_keys():
    """A key pointer that the 16-byte vector loads cannot read is refused before any launch."""
    f, _ = _fn()
    cfg = fn_small_config(indexer_budget=64)
    iq, comp, slots, pos = _inputs(cfg, 4, 1, 300, seed=5)
    sel = torch.zeros(4, 16, dtype=torch.int32, device="cuda")
    sparse = torch.zeros(4, dtype=torch.int32, device="cuda")
    rc = f(iq.data_ptr(), comp.data_ptr() + 2, 1, slots.data_ptr(), pos.data_ptr(), sel.data_ptr(),
           sparse.data_ptr(), 4, cfg.indexer_heads, cfg.indexer_dim, comp.shape[1], 16, cfg.indexer_ratio, 1,
           torch.cuda.current_stream().cuda_stream)
    assert rc == 1

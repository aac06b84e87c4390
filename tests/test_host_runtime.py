"""Native host runtime (C++ `_host`): allocator parity with the Python allocator, group quantization, the
deterministic multi-threaded quantized reducer, and the binary step log."""
import random

import numpy as np
import pytest
import torch

_host = pytest.importorskip("arcagi2_flashnext_dots3_b200._host")

from arcagi2_flashnext_dots3_b200.engine.block_manager import PyBlockAllocator  # noqa: E402
from arcagi2_flashnext_dots3_b200.utils import steplog  # noqa: E402


def test_allocator_matches_python():
    a, b = _host.BlockAllocator(50, 4), PyBlockAllocator(50, 4)
    rng = random.Random(0)
    for _ in range(300):
        op, s = rng.randrange(3), rng.randrange(4)
        if op == 0:
            n = rng.randrange(6)
            if n <= b.n_free():
                assert list(a.allocate(s, n)) == b.allocate(s, n)
            else:
                with pytest.raises(RuntimeError):
                    a.allocate(s, n)
        elif op == 1:
            assert a.release(s) == b.release(s)
        else:
            k = rng.randrange(5)
            assert a.truncate(s, k) == b.truncate(s, k)
        assert a.n_free() == b.n_free() and list(a.blocks_of(s)) == b.blocks_of(s)


@pytest.mark.parametrize("bits", [8, 6, 5])
def test_quantize_roundtrip(bits):
    x = torch.randn(1000) * 3
    codes, scales = _host.quantize_groups(x, bits)
    assert codes.numel() == (1000 if bits == 8 else (1000 * bits + 7) // 8)
    y = _host.dequantize_groups(codes, scales, 1000, bits)
    s = scales.repeat_interleave(128)[:1000]
    assert ((x - y).abs() <= s / 2 + 1e-6).all()


def test_reducer_is_exact_and_thread_invariant():
    W, n, bits = 4, 5000, 6
    xs = [torch.randn(n) for _ in range(W)]
    q = [_host.quantize_groups(x, bits) for x in xs]
    want = np.zeros(n, dtype=np.float32)
    for c, s in q:  # rank order, fp32
        want = want + _host.dequantize_groups(c, s, n, bits).numpy()
    outs = []
    for threads in (1, 8):
        oc, os_, total = _host.HostReducer(threads).reduce([c for c, _ in q], [s for _, s in q], n, bits, 8)
        outs.append(total)
        assert np.array_equal(total.numpy(), want)
    assert torch.equal(outs[0], outs[1])
    back = _host.dequantize_groups(oc, os_, n, 8)
    assert (back - outs[0]).abs().max() <= os_.max() / 2 + 1e-6


def test_steplog_roundtrip(tmp_path):
    p = str(tmp_path / "steps.bin")
    lg = steplog.StepLog(p)
    for i in range(5000):
        lg.append(t_us=i * 10, batch=64, tokens=64 + i % 3, accepted=i % 4)
    lg.close()
    r = steplog.read(p)
    assert len(r["t_us"]) == 5000 and r["tokens"][2] == 66 and r["accepted"][3] == 3

"""Start-up gates: exact-and-faster enabling, error bounds, failing candidates, contiguous size ranges (CPU with a
fake clock), and this framework's GPU gates on a B200."""
import json

import pytest
import torch

from arcagi2_flashnext_dots3_b200.engine.gates import Gates, engine_gates


def test_gates_enable_only_accurate_and_faster(tmp_path):
    cost = {}

    def timed(value, us):
        f = lambda: value
        cost[id(f)] = us
        return f
    gates = Gates(log_path=str(tmp_path / "g.jsonl"), timer=lambda fn: cost[id(fn)])
    state = {}
    x = torch.ones(4)
    gates.add("fast_exact", timed(x, 10.0), timed(x.clone(), 5.0), lambda on: state.__setitem__("a", on))
    gates.add("fast_wrong", timed(x, 10.0), timed(x * 1.1, 5.0), lambda on: state.__setitem__("b", on), tol=0.05)
    gates.add("slow", timed(x, 10.0), timed(x, 9.8), lambda on: state.__setitem__("c", on))

    def boom():
        raise RuntimeError("kernel missing")
    gates.add("broken", timed(x, 10.0), boom, lambda on: state.__setitem__("d", on))
    gates.run()
    assert state == {"a": True, "b": False, "c": False, "d": False}
    rows = [json.loads(l) for l in open(tmp_path / "g.jsonl")]
    assert [r["gate"] for r in rows] == ["fast_exact", "fast_wrong", "slow", "broken"] and rows[0]["speedup"] == 2.0


def test_sized_gate_picks_best_contiguous_range():
    # (baseline us, candidate us) per size: wins at 2 (gain 5) and at 8-16 (gain 12 + 30)
    times = {1: (10, 12), 2: (10, 5), 4: (10, 11), 8: (20, 8), 16: (40, 10), 32: (80, 90)}
    cur = {}

    def side(which):
        def f(size):
            cur.update(size=size, which=which)
            return torch.ones(3)
        return f
    got = {}
    gates = Gates(timer=lambda fn: (fn(), times[cur["size"]][cur["which"]])[1])
    gates.add_sized("ar", sorted(times), side(0), side(1), lambda rng: got.setdefault("rng", rng))
    res = gates.run()
    assert got["rng"] == (8, 16)
    assert [r.enabled for r in res] == [False, False, False, True, True, False]


@pytest.mark.gpu
def test_engine_gates_on_gpu():
    from arcagi2_flashnext_dots3_b200.models import fn as fn_model
    from arcagi2_flashnext_dots3_b200.ops import d3_ops
    saved = (fn_model.GEMV_MOE, d3_ops._MLA_CUDA_CORE)
    try:
        res = engine_gates("cuda", reps=5).run()
        by = {r.name: r for r in res}
        assert set(by) == {"moe_gemv_int8", "mla_tcgen05"}
        for r in res:
            assert r.err < 5e-2 and r.base_us > 0 and r.cand_us > 0, r
        assert by["mla_tcgen05"].enabled        # the tcgen05 latent attention is ~10x the CUDA-core kernel
    finally:
        fn_model.GEMV_MOE, d3_ops._MLA_CUDA_CORE = saved

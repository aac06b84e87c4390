"""D3 direct solver pieces on CPU: grid formats and answer parsing, the repetition monitor, the confidence gate
and the deadline-aware solver with forced conclusions over a scripted stream."""
import asyncio
import json
import math

import numpy as np

from arcagi2_flashnext_dots3_b200.agent import conf_gate, d3_solver, gridfmt, loop_detect

TASK = {"train": [{"input": [[1, 0], [0, 0]], "output": [[0, 1], [0, 0]]},
                  {"input": [[0, 2], [0, 0]], "output": [[2, 0], [0, 0]]}],
        "test": [{"input": [[3, 0], [0, 4]]}]}


def test_prompt_formats_and_answer_parsing():
    tpl = d3_solver.DEFAULT_TEMPLATE
    js = gridfmt.prompt_body(tpl, TASK, 0, "json")
    assert "[[1, 0], [0, 0]]" in js and gridfmt.FORMAT_NOTE not in js
    cp = gridfmt.prompt_body(tpl, TASK, 0, "compact")
    assert "INPUT (2x2):\n30\n04" in cp and gridfmt.WRITE_NOTE in cp and gridfmt.ANSWER_NOTE in cp
    assert gridfmt.WRITE_NOTE not in gridfmt.prompt_body(tpl, TASK, 0, "compact_noinstr")
    jl = d3_solver.json_grid
    assert gridfmt.parse_answer("so [[1, 2], [3, 4]] done", jl) == [[1, 2], [3, 4]]
    assert gridfmt.parse_answer('[["0012", "3450"]]', jl) == [[0, 0, 1, 2], [3, 4, 5, 0]]
    assert gridfmt.parse_answer("rows:\n0012\n3450\nend", jl) == [[0, 0, 1, 2], [3, 4, 5, 0]]
    assert gridfmt.parse_answer("no grid", jl) is None
    assert gridfmt.trace_grid("30\n04\nthen\n03\n40\n", (2, 2), [[3, 0], [0, 4]]) == [[0, 3], [4, 0]]


def test_repetition_monitor():
    loop = "7 " * 60000
    pos = loop_detect.first_fire(loop)
    assert pos is not None and pos >= 49152
    rng = np.random.default_rng(0)
    prose = " ".join("".join(chr(97 + c) for c in rng.integers(0, 26, 6)) for _ in range(20000))
    assert loop_detect.first_fire(prose) is None
    m = loop_detect.RepetitionMonitor()
    fired = False
    for i in range(0, len(prose[:40000]) + len(loop), 500):
        fired = m.update((prose[:40000] + loop)[i:i + 500]) or fired
    assert fired and 0 < m.cut_at < m.fired_at


def test_confidence_gate_features():
    assert conf_gate.parse_spec("100000:7.9, 2000:1") == [(2000, 1.0), (100000, 7.9)]
    rng = np.random.default_rng(1)
    tops = -rng.random((3000, 5)) * 3
    g = conf_gate.ConfidenceGate([(3000, -1e9)], feature="lowest_group", k=5, group=512, stride=128)
    for t in tops:
        g.add(float(t[0]), list(t))
    c = -tops.mean(1)
    want = min(c[n - 512:n].mean() for n in range(512, 3001, 128))
    assert math.isclose(g.feature_value(), want, rel_tol=1e-9)
    gate = conf_gate.ConfidenceGate([(100, 10.0)], feature="avg_conf", k=2)
    fired = [gate.add(-0.1, [-0.1, -0.2]) for _ in range(100)]
    assert fired[-1] and gate.fired_at == 100 and not any(fired[:-1])


def test_direct_solver_forces_conclusions_and_writes_attempts():
    tasks = {"a": TASK, "b": {"train": TASK["train"], "test": [{"input": [[5, 5], [0, 0]]}]}}
    stream = d3_solver.fake_stream_factory({"30\n04": (4, [[0, 3], [4, 0]]), "55\n00": (500, [[5, 5], [1, 1]])})
    cfg = d3_solver.SolverConfig(deadline_s=60, margin_s=1, cap1=2000, cap2=1000, min_cap=500, min_cap2=200,
                                 protect=0, force_tokens=64, concurrency=4)
    s = d3_solver.DirectSolver(tasks, stream, cfg)
    sub = asyncio.run(s.solve())
    assert sub["a"][0]["attempt_1"] == [[0, 3], [4, 0]]
    assert sub["b"][0]["attempt_1"] == [[5, 5], [1, 1]]        # cut at its cap, then forced to answer
    a_b = s.attempts[("b", 0, 1)]
    assert a_b.stopped == "cap" and a_b.forced
    assert not s.attempts[("a", 0, 1)].forced
    assert json.dumps(sub)

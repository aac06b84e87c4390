"""Agent harness on CPU: grid helpers and invariants, the sandbox limits, voting, the solver loop with a scripted
model, atomic submissions, and the session client against a live CPU server."""
import asyncio
import json
import os

import numpy as np
import pytest

from arcagi2_flashnext_dots3_b200.agent import arckit as ak
from arcagi2_flashnext_dots3_b200.agent.sandbox import feedback, run_code_sync
from arcagi2_flashnext_dots3_b200.agent.solver import Solver, ensure_submission, write_submission
from arcagi2_flashnext_dots3_b200.agent.vote import rank

TASK = {"train": [{"input": [[1, 0], [0, 0]], "output": [[0, 1], [0, 0]]},
                  {"input": [[0, 0, 2], [0, 3, 0]], "output": [[2, 0, 0], [0, 3, 0]]}],
        "test": [{"input": [[5, 0, 0], [0, 0, 7]]}]}
GOOD = "def transform(g):\n    return [row[::-1] for row in g]\n"


def test_arckit_basics():
    g = ak.grid([[0, 0, 0], [0, 4, 4], [0, 4, 0]])
    assert ak.bg(g) == 0 and ak.palette(g) == [0, 4]
    assert ak.bbox(g != 0) == (1, 1, 2, 2)                       # inclusive box
    assert ak.crop(g, ak.bbox(g != 0)).tolist() == [[4, 4], [4, 0]]
    assert ak.trim(g).tolist() == [[4, 4], [4, 0]]
    objs = ak.objects(g)
    assert len(objs) == 1 and objs[0].size == 3 and objs[0].colour == 4
    assert "fliplr" in ak.symmetries([[1, 2, 1], [3, 3, 3]])
    assert ak.period([[1, 2, 1, 2], [1, 2, 1, 2]]) == (1, 2)
    assert ak.gravity([[1, 0], [0, 0]]).tolist() == [[0, 0], [1, 0]]
    assert ak.find_sub([[1, 2, 3], [4, 5, 6]], [[5, 6]]) == [(1, 1)]
    assert ak.downscale(ak.scale([[1, 2]], 3), 3).tolist() == [[1, 2]]
    assert ak.enclosed([[1, 1, 1], [1, 0, 1], [1, 1, 1]], bgc=0)[1, 1]


def test_arckit_reference_contract():
    """Semantics model-written programs rely on: orderings, tie rules, conventions and the added helpers."""
    assert list(ak.counts([[1, 1, 0], [2, 2, 2]])) == [2, 1, 0]
    assert ak.bg([[1, 2], [2, 1]]) == 1 and ak.bg([[0, 3], [3, 0]]) == 0
    assert ak.task_bg([{"input": [[5, 5]], "output": [[5, 0]]}]) == 5
    assert ak.d8([[1, 2], [3, 4]], "rot90").tolist() == [[3, 1], [4, 2]]
    assert ak.d8([[1, 2], [3, 4]], "antitranspose").tolist() == [[4, 2], [3, 1]]
    assert list(ak.d8([[1]])) == list(ak.D8)
    assert ak.ray([[0, 0, 3, 0]], 0, 0, 0, 1, 5, stop=3).tolist() == [[0, 5, 3, 0]]
    assert ak.ray([[0, 2, 0]], 0, 0, 0, 1, 5, overwrite=False).tolist() == [[0, 2, 5]]
    g = [[0, 3, 0], [0, 0, 0]]
    assert ak.move(g, ak.objects(g)[0], 1, 1).tolist() == [[0, 0, 0], [0, 0, 3]]
    sg = [[0, 0, 8, 0, 0], [0, 1, 8, 0, 0], [8, 8, 8, 8, 8], [0, 0, 8, 0, 2], [0, 0, 8, 0, 0]]
    s = ak.split_grid(sg)
    assert s["colour"] == 8 and s["rows"] == [2] and s["cols"] == [2]
    assert s["boxes"] == [[(0, 0, 1, 1), (0, 3, 1, 4)], [(3, 0, 4, 1), (3, 3, 4, 4)]]
    assert s["cells"][1][1].tolist() == [[0, 2], [0, 0]]
    assert ak.period([[1, 2, 1, 2], [1, 2, 9, 2]], ignore=9) == (1, 2)
    assert ak.repair_period([[1, 2, 1, 2], [1, 2, 9, 2]], 9).tolist() == [[1, 2, 1, 2], [1, 2, 1, 2]]
    assert ak.symmetries([[1, 2, 9], [3, 4, 3]], ignore=9) == ["fliplr"]
    assert ak.complete_symmetry([[1, 2, 9], [3, 4, 3]], 9).tolist() == [[1, 2, 1], [3, 4, 3]]
    assert ak.downscale([[0, 0], [0, 3]], 2).tolist() == [[0]]
    assert ak.downscale([[0, 0], [0, 3]], 2, how="any").tolist() == [[3]]
    with pytest.raises(ValueError):
        ak.line([[0] * 4] * 4, 0, 0, 1, 3, 1)
    o = ak.objects([[0, 4, 4], [0, 4, 0]])[0]
    assert repr(o) == "Obj(colour=4 size=3 box=(0,1,1,2) 2x2 border)" and o.box == (0, 1, 1, 2)
    ring = ak.objects([[1, 1, 1], [1, 0, 1], [1, 1, 1]], bgc=0)[0]
    assert ring.holes == 1 and ring.size == 8 and not ring.rect
    ev = ak.obj_diff([[1, 0, 0], [0, 0, 0]], [[0, 0, 0], [0, 0, 1]])
    assert [e[0] for e in ev] == ["moved"] and ev[0][3] == (1, 2)
    ev = ak.obj_diff([[1, 1, 0], [0, 0, 0]], [[2, 2, 0], [0, 0, 0]])
    assert ev[0][0] == "recoloured" and ev[0][3] == (1, 2)
    assert str(ak.diff([[1, 2]], [[1, 3]])) == "same shape; 1/2 cells change in box (0, 1, 0, 1); 2->3:1"
    assert "output = input scaled x2x2" in str(ak.diff([[1, 2]], ak.scale([[1, 2]], 2)))
    assert ak.size_rule(TASK["train"]).kind == "same as input"
    assert ak.gravity([[1, 1, 0], [0, 0, 0], [0, 0, 0]], rigid=True).tolist() == [[0, 0, 0], [0, 0, 0], [1, 1, 0]]
    assert ak.gravity([[1, 0], [2, 0], [0, 0]], "down").tolist() == [[0, 0], [1, 0], [2, 0]]
    ns = {}
    exec(GOOD, ns)
    rep = ak.check(ns["transform"], TASK["train"], [TASK["test"][0]["input"]], verbose=False)
    assert rep["ok"] and rep["text"].startswith("check: 2/2 training pairs correct")
    assert rep["tests"][0]["out"].tolist() == [[0, 0, 5], [7, 0, 0]]
    bad = ak.check(lambda g: g, TASK["train"], verbose=False)
    assert not bad["ok"] and "cells wrong in box" in bad["pairs"][0]["why"]
    assert "2 train pairs; task background 0" in ak.describe(TASK["train"], [TASK["test"][0]["input"]])


def test_invariants_and_flag():
    inv = ak.invariants(TASK["train"])
    assert "output shape == input shape" in inv
    assert "output colours subset of input colours" in inv
    bad = ak.flag(TASK["train"], [TASK["test"][0]["input"]], [[[9, 9, 9], [9, 9, 9]]])
    assert "output colours subset of input colours" in bad


def test_sandbox_runs_and_scores():
    r = run_code_sync(GOOD, TASK)
    assert r["has_transform"] and all(p["ok"] for p in r["train"])
    assert r["tests"][0]["out"] == [[0, 0, 5], [7, 0, 0]]
    r = run_code_sync("def transform(g):\n    return g\n", TASK)
    assert not r["train"][0]["ok"]
    fb = feedback(r, TASK)
    assert "0/2 training pairs correct" in fb and "cells wrong in box" in fb
    r.pop("check_text")                      # without the helper report: the sandbox's own masked diffs
    assert "train 0: wrong cells" in feedback(r, TASK)


@pytest.mark.parametrize("code,needle", [
    ("while True:\n    pass\n", "timeout"),
    ("import socket\nsocket.create_connection(('127.0.0.1', 9))\n", "not allowed"),
    ("import subprocess\nsubprocess.run(['true'])\n", "not allowed"),
    ("open('/tmp/fw_sandbox_escape', 'w').write('x')\n", "outside the sandbox"),
    ("x = bytearray(3 << 30)\n", "MemoryError"),
])
def test_sandbox_limits(code, needle):
    r = run_code_sync(code + GOOD, TASK, timeout=4.0, cpu_s=3)
    assert needle in (r.get("error") or ""), r
    assert not os.path.exists("/tmp/fw_sandbox_escape")


def test_vote_ranking():
    g1, g2, g3 = [[1]], [[2]], [[3]]
    recs = [{"progs": [{"verified": True, "tests": [g1], "n_ok": 2, "n_train": 2}]},
            {"progs": [{"verified": True, "tests": [g2], "n_ok": 2, "n_train": 2}]},
            {"progs": [{"verified": True, "tests": [g2], "n_ok": 2, "n_train": 2}]},
            {"progs": [{"verified": False, "tests": [g3], "n_ok": 1, "n_train": 2}], "answer": [g3]}]
    r = rank(recs, 1)[0]
    assert r["attempts"] == [g2, g1] and r["votes"] == [2, 1]
    r = rank(recs[3:], 1)[0]
    assert r["attempts"] == [g3] and r["from"] == ["fb"]


def test_solver_with_scripted_model(tmp_path):
    tasks = {"a": TASK, "b": TASK}

    def factory(tid, idx):
        turns = ["```python\ndef transform(g):\n    return g\n```", "fixed:\n```python\n" + GOOD + "```"]

        async def complete(messages, max_tokens):
            return turns[min(len([m for m in messages if m["role"] == "assistant"]), 1)]
        return complete

    s = Solver(tasks, factory, samples_per_task=3, concurrency=4, deadline_s=60, endgame_s=5, settle_votes=2)
    ans = asyncio.run(s.run())
    assert ans["a"][0]["attempt_1"] == [[0, 0, 5], [7, 0, 0]]
    assert all(x.get("verified") for x in s.log)
    assert 2 <= sum(1 for x in s.log if x["tid"] == "a") <= 3
    p = str(tmp_path / "submission.json")
    write_submission(p, {"a": ans["a"]})
    sub = ensure_submission(p, tasks)
    assert sub["b"][0]["attempt_1"] == TASK["test"][0]["input"]
    assert json.load(open(p)) == sub


def test_session_client_against_cpu_server():
    import socket
    import threading
    import time

    import torch
    import uvicorn

    from arcagi2_flashnext_dots3_b200.agent.client import SessionClient
    from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config
    from arcagi2_flashnext_dots3_b200.engine.llm import LLM
    from arcagi2_flashnext_dots3_b200.models import fn_weights
    from arcagi2_flashnext_dots3_b200.server.app import create_app
    from arcagi2_flashnext_dots3_b200.server.engine_loop import EngineLoop
    from arcagi2_flashnext_dots3_b200.server.tokenizer import ByteTokenizer

    cfg = fn_small_config(num_layers=1, ple_layers=())
    W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=0, symmetric=False), cfg, "cpu")
    eng = EngineLoop(LLM(cfg, W, "cpu", EngineConfig(max_seqs=2, max_model_len=512, block_size=16,
                                                     graph_batch_sizes=(1, 2))), ByteTokenizer()).start()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    server = uvicorn.Server(uvicorn.Config(create_app(eng), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    while not server.started:
        time.sleep(0.05)

    async def go():
        c = SessionClient(f"http://127.0.0.1:{port}", ByteTokenizer(), "t1", 512, temperature=0.0, chunk=3)
        msgs = [{"role": "user", "content": "hi"}]
        a = await c(msgs, 7)
        msgs += [{"role": "assistant", "content": a}, {"role": "user", "content": "more"}]
        b = await c(msgs, 5)
        await c.close()
        return a, b, eng.stats
    try:
        a, b, st = asyncio.run(go())
        assert st["sessions"] == 1 and st["pushes"] >= 3 and st["generated"] >= 12
    finally:
        server.should_exit = True
        th.join(timeout=10)
        eng.stop()


def test_vote_partial_weights_and_verified_override():
    """Partial evidence weighs 0.5 x pass rate; a grid with any verified vote ranks only by its votes."""
    g1, g2, g3 = [[1]], [[2]], [[3]]
    part = lambda g, ok: {"verified": False, "tests": [g], "n_ok": ok, "n_train": 4}
    recs = [{"progs": [part(g1, 4)], "answer": [g2]},          # g2 answer 1.0, g1 partial 0.5
            {"progs": [part(g3, 2)], "answer": [g3]},          # g3 answer 1.0 + partial 0.25
            {"progs": [{"verified": True, "tests": [g1], "n_ok": 4, "n_train": 4}]}]
    r = rank(recs, 1)[0]
    assert r["attempts"] == [g1, g3] and r["from"] == ["ver", "fb"] and r["n_verified"] == 1
    r = rank(recs[:2], 1)[0]
    assert r["attempts"] == [g3, g2] and r["votes"] == [0, 0]


def test_rate_meter_and_sample_budget():
    from arcagi2_flashnext_dots3_b200.agent.solver import RateMeter
    t = [0.0]
    m = RateMeter(window=10.0, clock=lambda: t[0])
    assert m.rate() is None
    for k in range(12):
        t[0] = float(k)
        m.add(100)
    assert abs(m.rate() - 100.0) < 1e-6          # sliding window keeps a steady 100 tok/s
    s = Solver({"a": TASK, "b": TASK}, lambda tid, i: None, samples_per_task=2, deadline_s=100, endgame_s=0,
               max_turns=4, max_tokens=2048, rate=m, min_sample_tokens=64)
    now = s.cut - 10.0                           # 10 s x 100 tok/s = 1000 tokens for 4 samples to run
    assert s.sample_budget(now) == 250
    assert s.sample_budget(s.cut + 1) == 64      # past the cut only the floor is left
    m2 = RateMeter()
    s.rate = m2
    assert s.sample_budget(now) == 4 * 2048      # no rate yet: the turn-based cap


def test_server_room_and_tiers():
    from arcagi2_flashnext_dots3_b200.agent.solver import ServerRoom
    stats = {"kv_blocks_free": 10, "block_size": 64}
    room = ServerRoom(lambda: stats)
    assert room() == 640
    room.grow[("a", 0)] = 600
    assert room() == 40
    s = Solver({"a": TASK, "b": TASK}, lambda tid, i: None, samples_per_task=3, ctx_room=room,
               est_ctx=lambda task: 100)
    assert s.pick() is None                      # 40 tokens of room, 100 projected
    room.grow.clear()
    st = s.pick()
    assert st.tid == "a" and st.tier(2) == 0
    st.started = 1
    st.recs.append({"verified": True, "answer": [[[1]]], "progs": []})
    assert st.tier(2) == 2 and s.pick().tid == "b"   # never-started tasks first
    s.tasks["b"].started = 1
    s.tasks["b"].recs.append({"verified": False, "answer": [], "progs": []})
    assert s.pick().tid == "b"                   # unverified before verified-unsettled


def test_session_forced_conclusion_and_budget():
    from arcagi2_flashnext_dots3_b200.agent.session import FORCE, solve_sample
    seen = []

    async def complete(messages, n_tok):
        seen.append((messages[-1]["content"], n_tok))
        return "```python\ndef transform(g):\n    return g\n```"
    import time
    rec = asyncio.run(solve_sample(TASK, complete, max_turns=5, max_tokens=512, force_at=time.time() + 3600,
                                   token_budget=1200, force_tokens=128))
    # turn 1 and 2 regular (1200 - 2 x ~13 > 512), then budget stays > 512: no forcing by budget here
    assert rec["turns"] == 5 and not rec["forced"]
    seen.clear()
    rec = asyncio.run(solve_sample(TASK, complete, max_turns=5, max_tokens=512, force_at=0.0, force_tokens=128))
    assert rec["turns"] == 1 and rec["forced"] and seen[0][1] == 128
    assert rec["answer"] == [TASK["test"][0]["input"]]   # the forced program's test outputs are the answer
    seen.clear()
    rec = asyncio.run(solve_sample(TASK, complete, max_turns=5, max_tokens=512, token_budget=520,
                                   force_tokens=128))
    assert rec["turns"] == 2 and rec["forced"] and seen[1] == (FORCE, 128)

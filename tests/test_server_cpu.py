"""HTTP server on a CPU engine: completions equal the engine's greedy decode, sessions keep their cache across
pushes (a continuation equals an uninterrupted decode), context overflow is refused with 409."""
import json

import pytest
import torch

from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config
from arcagi2_flashnext_dots3_b200.engine.llm import LLM
from arcagi2_flashnext_dots3_b200.models import fn_weights

fastapi = pytest.importorskip("fastapi")
import requests  # noqa: E402
import socket  # noqa: E402
import threading  # noqa: E402
import time  # noqa: E402

import uvicorn  # noqa: E402

from arcagi2_flashnext_dots3_b200.server.app import create_app  # noqa: E402
from arcagi2_flashnext_dots3_b200.server.engine_loop import EngineLoop  # noqa: E402
from arcagi2_flashnext_dots3_b200.server.tokenizer import ByteTokenizer  # noqa: E402


@pytest.fixture(scope="module")
def setup():
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=0, symmetric=False), cfg, "cpu")
    ec = EngineConfig(max_seqs=3, max_model_len=48, block_size=16, graph_batch_sizes=(1, 2, 4))
    eng = EngineLoop(LLM(cfg, W, "cpu", ec), ByteTokenizer()).start()
    ref = LLM(cfg, W, "cpu", ec)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    server = uvicorn.Server(uvicorn.Config(create_app(eng), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.05)
    yield Client(f"http://127.0.0.1:{port}"), ref
    server.should_exit = True
    th.join(timeout=10)
    eng.stop()


class Client:
    def __init__(self, base):
        self.base = base

    def get(self, path):
        return requests.get(self.base + path, timeout=60)

    def post(self, path, json):
        return requests.post(self.base + path, json=json, timeout=60)

    def stream(self, method, path, json):
        return requests.request(method, self.base + path, json=json, stream=True, timeout=60)


def test_health_and_models(setup):
    c, _ = setup
    assert c.get("/health").status_code == 200
    assert c.get("/v1/models").json()["data"][0]["max_model_len"] == 48


def test_completion_greedy_matches_engine(setup):
    c, ref = setup
    prompt = [5, 9, 11, 40, 7]
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6, "temperature": 0, "logprobs": 1})
    assert r.status_code == 200, r.text
    body = r.json()
    want = ref.generate([prompt], max_new_tokens=6)[0]
    assert body["usage"]["completion_tokens"] == 6
    assert len(body["choices"][0]["logprobs"]["token_logprobs"]) == 6
    assert body["choices"][0]["finish_reason"] == "length"
    assert ByteTokenizer().decode(want) == body["choices"][0]["text"]


def _read_until(lines, key):
    evs = []
    for line in lines:
        if not line:
            continue
        ev = json.loads(line)
        evs.append(ev)
        if key in ev:
            return evs
    raise AssertionError(f"stream ended before {key}: {evs}")


def test_session_push_continues_the_same_sequence(setup):
    c, ref = setup
    prompt = [3, 8, 21, 13]
    want = ref.generate([prompt], max_new_tokens=7)[0]
    with c.stream("POST", "/arc/session", json={"rid": "s1", "prompt_ids": prompt, "max_tokens": 4, "keep": True,
                                                 "temperature": 0}) as r:
        lines = r.iter_lines(chunk_size=1)
        evs = _read_until(lines, "chunk_end")
        got = [t for e in evs for t in e.get("ids", [])]
        assert evs[-1]["chunk_end"] == "length" and got == want[:4]
        p = c.post("/arc/session/push", json={"rid": "s1", "prompt_ids": [got[-1]], "max_tokens": 3, "keep": True,
                                               "temperature": 0})
        assert p.status_code == 200, p.text
        evs = _read_until(lines, "chunk_end")
        got += [t for e in evs for t in e.get("ids", [])]
        assert got == want
        # a push that would overflow max_model_len is refused and ends the session
        p = c.post("/arc/session/push", json={"rid": "s1", "prompt_ids": list(range(3, 60)), "max_tokens": 2})
        assert p.status_code == 409 and p.json()["error"] == "ctx_full"
        evs = _read_until(lines, "end")
        assert evs[-1]["end"] == "ctx_full"
    st = c.get("/arc/session/stats").json()
    assert st["sessions"] >= 1 and st["pushes"] >= 1 and st["push_refused"] >= 1
    assert c.post("/arc/session/push", json={"rid": "s1", "prompt_ids": [1], "max_tokens": 1}).status_code == 404


def test_sampled_completion_is_reproducible(setup):
    c, _ = setup
    body = {"prompt": "abc", "max_tokens": 5, "temperature": 1.0, "top_p": 0.9, "seed": 7}
    a = c.post("/v1/completions", json=body).json()["choices"][0]["text"]
    b = c.post("/v1/completions", json=body).json()["choices"][0]["text"]
    assert a == b

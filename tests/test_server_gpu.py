"""Server on the GPU engine: a session with pushes reproduces an uninterrupted greedy decode."""
import json
import socket
import threading
import time

import pytest
import requests
import torch

pytestmark = pytest.mark.gpu


def test_gpu_session_roundtrip():
    import uvicorn
    from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config
    from arcagi2_flashnext_dots3_b200.engine.llm import LLM
    from arcagi2_flashnext_dots3_b200.models import fn_weights
    from arcagi2_flashnext_dots3_b200.server.app import create_app
    from arcagi2_flashnext_dots3_b200.server.engine_loop import EngineLoop
    from arcagi2_flashnext_dots3_b200.server.tokenizer import ByteTokenizer

    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=0, symmetric=False), cfg, "cuda")
    ec = EngineConfig(max_seqs=4, max_model_len=128, block_size=16, graph_batch_sizes=(1, 2, 4))
    ref = LLM(cfg, W, "cuda", ec)
    prompt = [3, 8, 21, 13, 99]
    want = ref.generate([prompt], max_new_tokens=9)[0]
    eng = EngineLoop(LLM(cfg, W, "cuda", ec), ByteTokenizer()).start()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    server = uvicorn.Server(uvicorn.Config(create_app(eng), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    while not server.started:
        time.sleep(0.05)
    base = f"http://127.0.0.1:{port}"
    try:
        r = requests.post(base + "/arc/session", json={"rid": "g", "prompt_ids": prompt, "max_tokens": 5, "keep": True,
                                                      "temperature": 0}, stream=True, timeout=120)
        lines = r.iter_lines(chunk_size=1)
        got = []
        for line in lines:
            ev = json.loads(line)
            got += ev.get("ids", [])
            if "chunk_end" in ev:
                break
        assert requests.post(base + "/arc/session/push", json={"rid": "g", "prompt_ids": [got[-1]], "max_tokens": 4,
                                                               "temperature": 0}, timeout=60).status_code == 200
        for line in lines:
            ev = json.loads(line)
            got += ev.get("ids", [])
            if "chunk_end" in ev:
                break
        assert got == want
        requests.post(base + "/arc/session/close", json={"rid": "g"}, timeout=60)
    finally:
        server.should_exit = True
        th.join(timeout=10)
        eng.stop()

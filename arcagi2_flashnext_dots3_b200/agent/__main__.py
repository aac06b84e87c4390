"""Solve a task file against a running server and write the submission:

    python -m arcagi2_flashnext_dots3_b200.agent --tasks test.json --server http://127.0.0.1:8000 --out submission.json

`--tasks` is the ARC challenge format ({task id: {"train": [...], "test": [{"input"}]}}). Each sample is one
multi-turn session on the server; the submission is written atomically at the end (and completed with the test
inputs for anything missing, so a partial run still leaves a valid file).
"""
from __future__ import annotations

import argparse
import asyncio
import json

from .client import SessionClient
from .solver import Solver, ServerRoom, ensure_submission, write_submission


def stats_poller(server: str, every_s: float = 1.0):
    """A cached synchronous read of the server's session stats (free KV blocks, block size)."""
    import time

    import requests
    last = {"t": 0.0, "v": None}

    def get():
        now = time.time()
        if now - last["t"] >= every_s:
            try:
                last["v"] = requests.get(f"{server}/arc/session/stats", timeout=2.0).json()
            except (requests.RequestException, ValueError):
                pass              # keep the last reading; no reading at all means no room limit
            last["t"] = now
        return last["v"] or {"kv_blocks_free": 1 << 40, "block_size": 1}
    return get


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tasks", required=True)
    ap.add_argument("--server", default="http://127.0.0.1:8000")
    ap.add_argument("--out", default="submission.json")
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--samples", type=int, default=4)
    ap.add_argument("--concurrency", type=int, default=32)
    ap.add_argument("--deadline-s", type=float, default=3600.0)
    ap.add_argument("--endgame-s", type=float, default=120.0)
    ap.add_argument("--max-turns", type=int, default=4)
    ap.add_argument("--max-tokens", type=int, default=4096)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--max-model-len", type=int, default=16384)
    a = ap.parse_args(argv)
    from ..server.tokenizer import load_tokenizer
    tok = load_tokenizer(a.tokenizer)
    tasks = json.load(open(a.tasks))
    ensure_submission(a.out, tasks)

    def factory(tid, idx):
        return SessionClient(a.server, tok, f"{tid}_{idx}", a.max_model_len, temperature=a.temperature,
                             seed=hash((tid, idx)) & 0x7FFFFFFF)
    def est_ctx(task):   # prompt (about 3.5 characters per token) plus every turn's generation
        return int(len(json.dumps(task)) / 3.5) + a.max_turns * (a.max_tokens + 256)
    s = Solver(tasks, factory, a.samples, a.concurrency, a.deadline_s, a.endgame_s, max_turns=a.max_turns,
               max_tokens=a.max_tokens, ctx_room=ServerRoom(stats_poller(a.server)), est_ctx=est_ctx)
    write_submission(a.out, asyncio.run(s.run()))
    ensure_submission(a.out, tasks)
    print(json.dumps({"tasks": len(tasks), "samples": len(s.log), "verified": sum(bool(x.get("verified")) for x in s.log)}))


if __name__ == "__main__":
    main()

"""Multi-turn program-synthesis loop for one ARC task sample.

Turn structure (the reference's repl_session.py / repl_prompt.py): the prompt shows the train pairs and test
inputs; the model answers with a ```python``` block defining ``transform``; the block runs in the sandbox; the
feedback (errors, masked diffs of failing train pairs, invariant warnings) is appended as the next user turn;
the loop ends when a program passes every train pair ("verified"), the turn budget runs out, or the deadline
passes. Every program's outcome is recorded for voting (:mod:`.vote`).

The model is any async callable ``complete(messages, max_tokens) -> str``; :class:`..agent.client.SessionClient`
provides one backed by the server's incremental ``/arc/session`` routes (only the new turn is prefilled).
"""
from __future__ import annotations

import re
import time

from .sandbox import feedback, run_code

SYSTEM = ("You solve ARC puzzles by writing Python. Reply with one ```python``` block that defines "
          "transform(grid) -> grid (grids are lists of lists of ints 0-9). numpy is available as np and grid "
          "helpers as ak.")


def grid_text(g) -> str:
    return "\n".join(" ".join(str(v) for v in row) for row in g)


def task_prompt(task: dict) -> str:
    parts = []
    for k, p in enumerate(task["train"]):
        parts.append(f"Train {k} input:\n{grid_text(p['input'])}\nTrain {k} output:\n{grid_text(p['output'])}")
    for k, t in enumerate(task["test"]):
        parts.append(f"Test {k} input:\n{grid_text(t['input'])}")
    return "\n\n".join(parts)


CODE_RE = re.compile(r"```(?:python)?\s*\n(.*?)```", re.S)


def extract_code(text: str):
    blocks = CODE_RE.findall(text)
    return blocks[-1] if blocks else None


async def solve_sample(task: dict, complete, max_turns: int = 4, max_tokens: int = 2048, deadline: float = None,
                       sandbox_timeout: float = 25.0) -> dict:
    """Returns {"progs": [...], "answer": [...], "turns": n, "verified": bool}."""
    messages = [{"role": "system", "content": SYSTEM}, {"role": "user", "content": task_prompt(task)}]
    rec = {"progs": [], "answer": [], "turns": 0, "verified": False}
    n_train = len(task["train"])
    for turn in range(max_turns):
        if deadline is not None and time.time() > deadline:
            rec["stopped"] = "deadline"
            break
        reply = await complete(messages, max_tokens)
        rec["turns"] += 1
        messages.append({"role": "assistant", "content": reply})
        code = extract_code(reply)
        if code is None:
            messages.append({"role": "user", "content": "Reply with one ```python``` block defining transform."})
            continue
        res = await run_code(code, task, timeout=sandbox_timeout)
        train = res.get("train") or []
        n_ok = sum(bool(p.get("ok")) for p in train)
        tests = [t.get("out") for t in res.get("tests") or []]
        verified = bool(train) and n_ok == n_train and all(t is not None for t in tests) and not res.get("flags")
        rec["progs"].append({"k": turn, "verified": verified, "n_ok": n_ok, "n_train": n_train, "tests": tests,
                             "flags": res.get("flags"), "code": code})
        if verified:
            rec["verified"] = True
            rec["answer"] = tests
            break
        messages.append({"role": "user", "content": feedback(res, task)})
    return rec

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


FORCE = ("Time is almost up. Reply now with your final ```python``` block defining transform(grid), the best "
         "program you have; no further feedback will follow.")


def estimate_tokens(text: str) -> int:
    """Rough token count of generated text (about 3.5 characters per token for code and grids)."""
    return max(1, int(len(text) / 3.5))


async def solve_sample(task: dict, complete, max_turns: int = 4, max_tokens: int = 2048, deadline: float = None,
                       sandbox_timeout: float = 25.0, token_budget: int = None, force_at: float = None,
                       force_tokens: int = 1024) -> dict:
    """Returns {"progs": [...], "answer": [...], "turns": n, "verified": bool, "used": tokens}.

    ``token_budget`` caps the sample's generated tokens; ``force_at`` (a time) or a budget too small for another
    regular turn turns the next turn into a forced final answer of at most ``force_tokens`` tokens (the
    reference's forced conclusions, repl_session.py / repl_solve.py endgame)."""
    messages = [{"role": "system", "content": SYSTEM}, {"role": "user", "content": task_prompt(task)}]
    rec = {"progs": [], "answer": [], "turns": 0, "verified": False, "used": 0, "forced": False}
    n_train = len(task["train"])
    for turn in range(max_turns):
        if deadline is not None and time.time() > deadline:
            rec["stopped"] = "deadline"
            break
        left = None if token_budget is None else token_budget - rec["used"]
        forced = (force_at is not None and time.time() >= force_at) or (left is not None and left < max_tokens)
        if forced and rec["forced"]:
            rec["stopped"] = "budget"
            break
        if forced and turn > 0:
            messages.append({"role": "user", "content": FORCE})
        n_tok = min(force_tokens if forced else max_tokens, max(1, left) if left is not None else 1 << 30)
        reply = await complete(messages, n_tok)
        rec["forced"] = rec["forced"] or forced
        rec["used"] += estimate_tokens(reply)
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
        if rec["forced"]:
            rec["answer"] = tests
            break
        messages.append({"role": "user", "content": feedback(res, task)})
    if not rec["answer"] and rec["progs"]:   # best partial program's test outputs as the sample's answer
        best = max(rec["progs"], key=lambda p: (p["n_ok"], p["k"]))
        if all(t is not None for t in best["tests"]):
            rec["answer"] = best["tests"]
    return rec

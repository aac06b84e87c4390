"""Degeneration check of sampled generations (the reference's dotsnote/training/eval/degen_test.py: sampled
completions of held-out prompts are flagged when their tail stops being prose).

* degenerate: the last 3000 characters hold fewer than 30 characters other than digits, commas, whitespace and
  brackets (a grid dump that never ends);
* runaway: the last 3000 characters are nothing but digits, commas and spaces.
"""
from __future__ import annotations

import re

TAIL = 3000


def degenerate(text: str) -> bool:
    tail = text[-TAIL:]
    return len(re.sub(r"[\d,\s\[\]]", "", tail)) < 30


def runaway(text: str) -> bool:
    tail = text[-TAIL:]
    return len(tail) == TAIL and re.fullmatch(r"[\d, ]*", tail) is not None


def summarize(texts: list) -> dict:
    """Counts and a one-character-per-sample map: 'R' runaway, 'X' degenerate, '.' fine."""
    d = [degenerate(t) for t in texts]
    r = [runaway(t) for t in texts]
    return {"n": len(texts), "degenerate": sum(d), "runaway": sum(r),
            "map": "".join("R" if y else "X" if x else "." for x, y in zip(d, r))}


def run(llm, prompts: list, decode, max_new_tokens: int = 12000, temperature: float = 0.7) -> dict:
    """Sample one completion per prompt through the engine (seed = prompt index) and summarize; `decode` maps
    token ids to text."""
    from ..ops.sampling import SamplingParams
    outs = []
    for i, p in enumerate(prompts):
        outs.append(llm.generate([p], max_new_tokens=max_new_tokens,
                                 sp=SamplingParams(temperature=temperature, seed=i))[0])
    res = summarize([decode(o) for o in outs])
    res["tokens"] = [len(o) for o in outs]
    return res

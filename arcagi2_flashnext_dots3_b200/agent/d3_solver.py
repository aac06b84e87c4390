"""Deadline-aware direct-answer solver (the D3 model's solver; capabilities of the reference's
dotsnote/kaggle/runtime_dataset/solve.py: elastic caps :265-322, attempts and forced conclusions :361-600).

Every test input gets up to two attempts: a prompt (``gridfmt.prompt_body``) whose completion reasons and ends in
an answer grid. The solver streams completions concurrently through ``stream`` (an async function of
(prompt, max_tokens, seed) yielding dicts {"text", "logprobs"} and ending with {"finish"}), and keeps them within
the time left:

* elastic caps: from the generation rate observed over the last ten minutes of its own streams, the token budget
  B = rate x (time to the deadline - margin) is split so that the first attempts still queued plus those running
  fit: the largest cap L (tried from ``cap1`` down in steps of 8000) whose expected remaining work
  sum E[min(N, L) - progress] fits B, with N drawn from the observed natural completion lengths (the defaults
  ``natural`` until some are seen); second attempts get only what is left, and start only when their full cap
  fits;
* a running attempt past its (possibly lowered) cap, one the repetition monitor flags, or one the confidence gate
  fails is stopped and forced to conclude: the prompt plus its text (cut before a detected loop) plus a short
  conclusion request, with ``force_tokens`` more tokens;
* the answer is ``gridfmt.parse_answer`` of the final text, else the last compact grid of the trace with the
  expected shape (the size rule of the train pairs).

``submission()`` returns {task: [{"attempt_1", "attempt_2"}]} with the test input as fallback.
"""
from __future__ import annotations

import asyncio
import json
import random
import time
import zlib
from dataclasses import dataclass

from . import arckit as ak
from . import gridfmt
from .conf_gate import ConfidenceGate
from .loop_detect import RepetitionMonitor

FORCE_TEXT = "\n\nI have to stop reasoning now and commit to an answer.\nFinal answer (JSON list of rows):\n"
DEFAULT_TEMPLATE = ("Find the common rule that maps an input grid to an output grid, given the examples below."
                    "\n\n--Training Examples--\n{training_examples}--End of Training Examples--\n\n"
                    "--Test Input--\n{test_input}\n--End of Test Input--\n\n"
                    "Your response should include the output grid as a JSON list of rows.")


def json_grid(text: str):
    """The last well-formed JSON list-of-lists in a text, or None."""
    end = len(text)
    while True:
        j = text.rfind("]]", 0, end)
        if j < 0:
            return None
        i = text.rfind("[[", 0, j)
        while i >= 0:
            try:
                return json.loads(text[i:j + 2])
            except ValueError:
                i = text.rfind("[[", 0, i)
        end = j


@dataclass
class Attempt:
    task: str
    ti: int
    n: int                       # 1 or 2
    tokens: int = 0
    text: str = ""
    grid: list = None
    stopped: str = ""            # "", "cap", "loop", "conf"
    forced: bool = False
    done: bool = False


@dataclass
class SolverConfig:
    deadline_s: float = 3600.0
    margin_s: float = 60.0
    cap1: int = 96000
    cap2: int = 48000
    min_cap: int = 16000
    min_cap2: int = 8000
    protect: int = 32000          # a first attempt below this many tokens is never cut below it
    force_tokens: int = 2048
    concurrency: int = 32
    fmt: str = "compact"
    seed: int = 0
    natural: tuple = (12000, 20000, 30000, 45000, 60000, 80000, 96000)


class DirectSolver:
    def __init__(self, tasks: dict, stream, cfg: SolverConfig = None, template: str = DEFAULT_TEMPLATE,
                 gate: ConfidenceGate = None, monitor_kw: dict = None):
        self.tasks, self.stream, self.cfg = tasks, stream, cfg or SolverConfig()
        self.template, self.gate, self.monitor_kw = template, gate, monitor_kw or {}
        self.t0 = time.time()
        self.deadline = self.t0 + self.cfg.deadline_s
        self.history = []                           # (time, total generated tokens)
        self.generated = 0
        self.natural = []                           # completion lengths of attempts that ended by themselves
        self.progress = {}                          # attempt key -> tokens so far (running)
        self.caps = {1: self.cfg.cap1, 2: self.cfg.cap2}
        self.admit2 = True
        self.attempts = {}
        self.queue = [(t, i, 1) for t, task in tasks.items() for i in range(len(task["test"]))]

    # ------------------------------------------------------------------------------------- budget
    def rate(self):
        """Generated tokens per second over the last ten minutes of streams (None until measurable)."""
        if len(self.history) < 2:
            return None
        t1, g1 = self.history[-1]
        t0, g0 = next(((t, g) for t, g in self.history if t >= t1 - 600), self.history[0])
        return (g1 - g0) / (t1 - t0) if t1 > t0 else None

    def expected_left(self, cap: float, done: float = 0.0) -> float:
        """Expected further tokens of an attempt at `done` tokens under `cap` (natural lengths min cap)."""
        if done >= cap:
            return 0.0
        lens = [min(n, cap) for n in (self.natural or self.cfg.natural) if n > done]
        return sum(lens) / len(lens) - done if lens else cap - done

    def _fit_cap(self, budget, n_queued, running, hi, lo, fixed=0.0):
        c = self.cfg
        L = hi
        while L >= lo:
            run = sum(self.expected_left(max(L, c.protect) if p < c.protect else L, p) for p in running)
            if fixed + n_queued * (self.expected_left(L) + c.force_tokens / 5) + run <= budget:
                return L
            L -= 8000
        return lo - 1

    def update_caps(self):
        r = self.rate()
        if r is None:
            return
        c = self.cfg
        B = r * max(0.0, self.deadline - time.time() - c.margin_s)
        q1 = sum(1 for *_, n in self.queue if n == 1)
        p1 = [p for (t, i, n), p in self.progress.items() if n == 1]
        p2 = [p for (t, i, n), p in self.progress.items() if n == 2]
        L1 = max(c.min_cap, self._fit_cap(B, q1, p1, c.cap1, c.min_cap)) if q1 else c.cap1
        need1 = q1 * self.expected_left(L1) + sum(
            self.expected_left(max(L1, c.protect) if p < c.protect else L1, p) for p in p1)
        L2 = self._fit_cap(B - need1, 0, p2, c.cap2, c.min_cap2)
        self.caps = {1: L1, 2: max(L2, c.min_cap2)}
        self.admit2 = L2 >= c.cap2 and B - need1 - sum(self.expected_left(c.cap2, p) for p in p2) >= \
            self.expected_left(c.cap2)

    def live_cap(self, n_attempt: int, tokens: int) -> int:
        if n_attempt == 1 and tokens < self.cfg.protect:
            return max(self.caps[1], self.cfg.protect)
        return self.caps[n_attempt]

    # ------------------------------------------------------------------------------------- attempts
    def _prompt(self, task, ti):
        return gridfmt.prompt_body(self.template, task, ti, self.cfg.fmt)

    def _expected_shape(self, task, ti):
        rule = ak.size_rule(task["train"])
        return rule.predict(task["test"][ti]["input"]) if rule else None

    async def _run_stream(self, prompt, max_tokens, seed, key, att: Attempt, watch: bool):
        monitor = RepetitionMonitor(**self.monitor_kw) if watch else None
        gate = self.gate.fresh() if (self.gate is not None and watch) else None
        n_attempt = key[2]
        async for ev in self.stream(prompt, max_tokens, seed):
            if "text" in ev:
                att.text += ev["text"]
                k = ev.get("n", 1)
                att.tokens += k
                self.generated += k
                self.history.append((time.time(), self.generated))
                if watch:
                    self.progress[key] = att.tokens
                    if monitor.update(ev["text"]):
                        att.stopped = "loop"
                        att.text = att.text[:monitor.cut_at] if monitor.cut_at else att.text
                        return
                    if gate is not None and ev.get("logprobs") and gate.add_openai(ev["logprobs"]):
                        att.stopped = "conf"
                        return
                    if att.tokens >= self.live_cap(n_attempt, att.tokens):
                        att.stopped = "cap"
                        return
            if ev.get("finish"):
                if watch and ev["finish"] == "stop":
                    self.natural.append(att.tokens)
                elif watch and ev["finish"] == "length":   # the server ended it at max_tokens: same as our cap
                    att.stopped = "cap"
                return

    async def run_attempt(self, task_id, ti, n):
        task = self.tasks[task_id]
        key = (task_id, ti, n)
        att = self.attempts[key] = Attempt(task_id, ti, n)
        prompt = self._prompt(task, ti)
        seed = self.cfg.seed * 1000003 + zlib.crc32(repr(key).encode()) % 1000003
        try:
            await self._run_stream(prompt, self.live_cap(n, 0), seed, key, att, True)
            if att.stopped:
                att.forced = True
                tail = Attempt(task_id, ti, n)
                await self._run_stream(prompt + att.text + FORCE_TEXT, self.cfg.force_tokens, seed, key, tail, False)
                att.text += FORCE_TEXT + tail.text
        finally:
            self.progress.pop(key, None)
        tin = task["test"][ti]["input"]
        answer_part = att.text.rsplit(FORCE_TEXT, 1)[-1] if att.forced else att.text
        att.grid = gridfmt.parse_answer(answer_part, json_grid)
        if att.grid is None:
            att.grid = gridfmt.trace_grid(att.text, self._expected_shape(task, ti), tin)
        att.done = True
        self.update_caps()
        if n == 1 and self.admit2 and time.time() < self.deadline - self.cfg.margin_s:
            self.queue.append((task_id, ti, 2))
        return att

    async def solve(self):
        sem = asyncio.Semaphore(self.cfg.concurrency)
        running = set()

        async def go(item):
            async with sem:
                await self.run_attempt(*item)

        while self.queue or running:
            while self.queue and len(running) < self.cfg.concurrency and time.time() < self.deadline:
                item = self.queue.pop(0)
                if item[2] == 2 and not self.admit2:
                    continue
                running.add(asyncio.ensure_future(go(item)))
            if not running:
                break
            done, _ = await asyncio.wait(running, return_when=asyncio.FIRST_COMPLETED)
            running -= done
            for d in done:
                d.result()
        return self.submission()

    def submission(self) -> dict:
        out = {}
        for t, task in self.tasks.items():
            rows = []
            for i, test in enumerate(task["test"]):
                a1 = self.attempts.get((t, i, 1))
                a2 = self.attempts.get((t, i, 2))
                g1 = a1.grid if a1 and a1.grid else test["input"]
                g2 = a2.grid if a2 and a2.grid else g1
                rows.append({"attempt_1": g1, "attempt_2": g2})
            out[t] = rows
        return out


def fake_stream_factory(answers: dict, tokens_per_chunk: int = 64, chunk_text: str = "thinking about rows. ",
                        rng_seed: int = 0):
    """A scripted stream for tests: each prompt's completion is some reasoning text followed by the answer grid
    registered for the first matching key substring (answers: {substring: (n_reasoning_chunks, grid)})."""
    rng = random.Random(rng_seed)

    async def stream(prompt, max_tokens, seed):
        for key, (n_chunks, grid) in answers.items():
            if key in prompt:
                break
        else:
            n_chunks, grid = 4, [[0]]
        if prompt.endswith(FORCE_TEXT):
            yield {"text": json.dumps(grid), "n": 8}
            yield {"finish": "stop"}
            return
        used = 0
        for _ in range(n_chunks):
            if used + tokens_per_chunk > max_tokens:
                yield {"finish": "length"}
                return
            used += tokens_per_chunk
            await asyncio.sleep(0)
            yield {"text": chunk_text, "n": tokens_per_chunk, "logprobs": None}
        yield {"text": "\nAnswer: " + json.dumps(grid), "n": 8}
        yield {"finish": "stop"}
        rng.random()
    return stream


def sse_stream(base_url: str, timeout: float = 7200.0):
    """A ``stream`` function over this framework's server: POST /v1/completions with stream=true and read the
    server-sent events (one event per decoded piece)."""
    import httpx

    async def stream(prompt, max_tokens, seed):
        body = {"prompt": prompt, "max_tokens": int(max_tokens), "temperature": 0.7, "top_p": 1.0, "seed": int(seed),
                "stream": True}
        async with httpx.AsyncClient(timeout=timeout) as c:
            async with c.stream("POST", f"{base_url}/v1/completions", json=body) as r:
                async for line in r.aiter_lines():
                    if not line.startswith("data: "):
                        continue
                    data = line[6:]
                    if data == "[DONE]":
                        return
                    ch = json.loads(data)["choices"][0]
                    if ch.get("text"):
                        yield {"text": ch["text"], "n": 1, "logprobs": ch.get("logprobs")}
                    if ch.get("finish_reason"):
                        yield {"finish": ch["finish_reason"]}
    return stream


def main(argv=None):
    import argparse
    import glob
    import os
    ap = argparse.ArgumentParser(description="Direct-answer ARC solver against a running server")
    ap.add_argument("--tasks", required=True, help="directory of task json files")
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--out", default="submission.json")
    ap.add_argument("--deadline-s", type=float, default=3600.0)
    ap.add_argument("--cap1", type=int, default=96000)
    ap.add_argument("--cap2", type=int, default=48000)
    ap.add_argument("--concurrency", type=int, default=32)
    ap.add_argument("--fmt", default="compact", choices=gridfmt.FORMATS)
    a = ap.parse_args(argv)
    tasks = {os.path.basename(f)[:-5]: json.load(open(f)) for f in sorted(glob.glob(os.path.join(a.tasks, "*.json")))}
    cfg = SolverConfig(deadline_s=a.deadline_s, cap1=a.cap1, cap2=a.cap2, concurrency=a.concurrency, fmt=a.fmt)
    solver = DirectSolver(tasks, sse_stream(a.url), cfg, gate=ConfidenceGate.from_env())
    sub = asyncio.run(solver.solve())
    tmp = a.out + ".tmp"
    with open(tmp, "w") as f:
        json.dump(sub, f)
    os.replace(tmp, a.out)
    return sub


if __name__ == "__main__":
    main()

"""Task-level orchestration: schedule samples of many tasks on one server under a deadline, vote, and write the
submission atomically.

Scheduling follows the reference's Solver (flashnext/kaggle/code_dataset/repl_solve.py:627-1344): at most
`concurrency` live samples; the next sample goes to the task with the fewest started samples that is not yet
settled (a task settles once `settle_votes` samples agree on verified outputs); a sample is admitted only while
its estimated context fits the server's KV room (``ctx_room``); after the cut time no new samples start
(``endgame``) and running ones stop at the deadline. ``write_submission`` writes to a temporary file and renames
it (``ensure_submission`` fills every missing test with the input grid so the file is always complete), as the
reference does at repl_solve.py:1259 and run_l4.py:537.

Budget control (the reference's guard / time-cap / context projection, repl_solve.py:870-960, in a form of our
own): a :class:`RateMeter` measures the server's generated tokens per second over a sliding window; each new sample
gets a token cap equal to its share of what the server can still generate before the cut
(rate x time left / samples still to run), clamped to [``min_sample_tokens``, max_turns x max_tokens]; samples
running when the cut passes have their next turn forced into a final answer (``force_at``). :class:`ServerRoom`
turns the server's ``/v1/stats`` (free KV blocks x block size) minus the projected growth of the live samples into
the ``ctx_room`` the picker checks. Picking goes by tiers: never-started tasks, then tasks without a verified
program, then verified-but-unsettled ones; settled tasks get no new samples.
"""
from __future__ import annotations

import asyncio
import json
import os
import time
from dataclasses import dataclass, field

from .session import solve_sample
from .vote import rank


class RateMeter:
    """Generated tokens per second over the last ``window`` seconds (None until two points are in)."""

    def __init__(self, window: float = 60.0, clock=time.time):
        self.window, self.clock = window, clock
        self.points = []          # (t, cumulative tokens)
        self.total = 0

    def add(self, n_tokens: int):
        self.total += int(n_tokens)
        t = self.clock()
        self.points.append((t, self.total))
        while len(self.points) > 2 and self.points[1][0] < t - self.window:
            self.points.pop(0)

    def rate(self):
        if len(self.points) < 2:
            return None
        (t0, c0), (t1, c1) = self.points[0], self.points[-1]
        return (c1 - c0) / (t1 - t0) if t1 > t0 else None


class ServerRoom:
    """KV room in tokens left for new samples: ``stats()`` (the server's stats dict with ``kv_blocks_free`` and
    ``block_size``) minus the growth still ahead of the live samples (``grow[sample] = projected final context -
    current context``, kept by the solver)."""

    def __init__(self, stats, reserve_tokens: int = 0):
        self.stats, self.reserve = stats, reserve_tokens
        self.grow = {}

    def __call__(self) -> int:
        st = self.stats() or {}
        free = int(st.get("kv_blocks_free", 0)) * int(st.get("block_size", 1))
        return free - sum(self.grow.values()) - self.reserve


@dataclass
class TaskState:
    tid: str
    task: dict
    recs: list = field(default_factory=list)
    started: int = 0
    running: int = 0
    samples_left: int = 0

    def settled(self, votes: int) -> bool:
        if not self.recs:
            return False
        r = rank(self.recs, len(self.task["test"]))
        return all(x["votes"] and x["votes"][0] >= votes for x in r)

    def tier(self, votes: int) -> int:
        """0 never started, 1 no verified program yet, 2 verified but not settled, 3 settled."""
        if self.started == 0:
            return 0
        if not any(r.get("verified") for r in self.recs):
            return 1
        return 3 if self.settled(votes) else 2


class Solver:
    def __init__(self, tasks: dict, complete_factory, samples_per_task: int = 4, concurrency: int = 8,
                 deadline_s: float = 3600.0, endgame_s: float = 60.0, settle_votes: int = 2, max_turns: int = 4,
                 max_tokens: int = 2048, ctx_room=None, est_ctx=None, rate: RateMeter = None,
                 min_sample_tokens: int = 1024, force_tokens: int = 1024):
        self.tasks = {tid: TaskState(tid, t, samples_left=samples_per_task) for tid, t in tasks.items()}
        self.complete_factory = complete_factory
        self.samples = samples_per_task
        self.concurrency = concurrency
        self.t0 = time.time()
        self.deadline = self.t0 + deadline_s
        self.cut = self.deadline - endgame_s
        self.settle_votes = settle_votes
        self.max_turns, self.max_tokens = max_turns, max_tokens
        self.ctx_room = ctx_room or (lambda: 1 << 62)
        self.est_ctx = est_ctx or (lambda task: 4096)
        self.rate = rate or RateMeter()
        self.min_sample_tokens, self.force_tokens = min_sample_tokens, force_tokens
        self.log = []

    def sample_budget(self, now: float = None) -> int:
        """Token cap of a sample started now: its share of what the server can generate before the cut."""
        cap = self.max_turns * self.max_tokens
        r = self.rate.rate()
        if r is None:
            return cap
        now = time.time() if now is None else now
        to_run = sum(max(0, st.samples_left) for st in self.tasks.values()) + \
            sum(st.running for st in self.tasks.values())
        share = r * max(0.0, self.cut - now) / max(1, to_run)
        return int(max(self.min_sample_tokens, min(cap, share)))

    def pick(self):
        """Next task to sample by tier (never started, unverified, verified-unsettled), then fewest started
        samples; settled tasks and tasks whose projected context does not fit the KV room are skipped."""
        cand = [s for s in self.tasks.values() if s.started < self.samples]
        if not cand:
            return None
        keyed = sorted(((s.tier(self.settle_votes), s.started, s.tid), s) for s in cand)
        room = self.ctx_room()
        for (tier, _, _), st in keyed:
            if tier == 3:
                return None
            if self.est_ctx(st.task) <= room:
                return st
        return None

    async def _sample(self, st: TaskState, idx: int):
        inner = self.complete_factory(st.tid, idx)
        key = (st.tid, idx)
        room = self.ctx_room if isinstance(self.ctx_room, ServerRoom) else None
        budget = self.sample_budget()
        if room is not None:
            room.grow[key] = self.est_ctx(st.task)

        async def complete(messages, n_tok):
            reply = await inner(messages, n_tok)
            n = max(1, int(len(reply) / 3.5))
            self.rate.add(n)
            if room is not None:
                room.grow[key] = max(0, room.grow.get(key, 0) - n)
            return reply

        try:
            rec = await solve_sample(st.task, complete, self.max_turns, self.max_tokens, deadline=self.deadline,
                                     token_budget=budget, force_at=self.cut, force_tokens=self.force_tokens)
            st.recs.append(rec)
            self.log.append({"tid": st.tid, "idx": idx, "verified": rec["verified"], "turns": rec["turns"],
                             "used": rec.get("used"), "budget": budget, "forced": rec.get("forced"),
                             "t": round(time.time() - self.t0, 2)})
        except Exception as e:  # one failing sample must not stop the run
            self.log.append({"tid": st.tid, "idx": idx, "error": repr(e)[:300]})
        finally:
            st.running -= 1
            if room is not None:
                room.grow.pop(key, None)
            closer = getattr(inner, "close", None)
            if closer is not None:
                await closer()

    async def run(self) -> dict:
        live = set()
        while True:
            now = time.time()
            if now < self.cut:
                while len(live) < self.concurrency:
                    st = self.pick()
                    if st is None:
                        break
                    st.started += 1
                    st.samples_left -= 1
                    st.running += 1
                    t = asyncio.create_task(self._sample(st, st.started - 1))
                    live.add(t)
            if not live:
                if now >= self.cut or self.pick() is None:
                    break
                await asyncio.sleep(0.05)
                continue
            timeout = max(0.01, self.deadline - time.time())
            done, live = await asyncio.wait(live, timeout=timeout, return_when=asyncio.FIRST_COMPLETED)
            if time.time() >= self.deadline:
                for t in live:
                    t.cancel()
                break
        return self.answers()

    def answers(self) -> dict:
        out = {}
        for tid, st in self.tasks.items():
            n = len(st.task["test"])
            r = rank(st.recs, n) if st.recs else [{"attempts": []} for _ in range(n)]
            out[tid] = []
            for k in range(n):
                att = r[k]["attempts"]
                inp = st.task["test"][k]["input"]
                a1 = att[0] if att else inp
                a2 = att[1] if len(att) > 1 else a1
                out[tid].append({"attempt_1": a1, "attempt_2": a2})
        return out


def write_submission(path: str, answers: dict):
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "w") as fh:
        json.dump(answers, fh)
        fh.flush()
        os.fsync(fh.fileno())
    os.replace(tmp, path)


def ensure_submission(path: str, tasks: dict):
    """Make sure every task and test input has both attempts (missing ones = the test input itself)."""
    try:
        with open(path) as fh:
            sub = json.load(fh)
    except (OSError, ValueError):
        sub = {}
    changed = False
    for tid, t in tasks.items():
        rows = sub.get(tid) or []
        for k, test in enumerate(t["test"]):
            if k >= len(rows):
                rows.append({"attempt_1": test["input"], "attempt_2": test["input"]})
                changed = True
            for a in ("attempt_1", "attempt_2"):
                if rows[k].get(a) is None:
                    rows[k][a] = test["input"]
                    changed = True
        sub[tid] = rows
    if changed or not os.path.exists(path):
        write_submission(path, sub)
    return sub

"""Engine thread: continuous batching of sessions and completions over one :class:`..engine.llm.LLM`.

All model work happens on this thread; HTTP handlers talk to it through a command queue and receive events on
per-request asyncio queues (``loop.call_soon_threadsafe``). Each loop iteration applies the pending commands
(start = submit, push = extend a kept session, close) and then runs one iteration of the
:class:`..engine.scheduler.Scheduler`: admission under the KV budget, a bounded amount of chunked prefill, one
CUDA-graph decode step for every running sequence; idle sessions keep their KV and are evicted, least recently
used first, when the cache deadlocks (their next push rebuilds them exactly).

Session semantics follow the reference's `/arc/session` routes (flashnext/kaggle/code_dataset/fnext/session/
session_ep.py:35-135): a session's KV stays resident between chunks; a chunk ends at its token budget
(``chunk_end: length``, the stream stays open for a push) or at a stop/eos token (``chunk_end: stop``; the stream
ends unless ``keep``); the newest sampled token of a finished chunk is not yet in the cache, so a continuation
pushes it back first; a push that would overflow ``max_model_len`` is refused (409) and ends the session with
``ctx_full``.
"""
from __future__ import annotations

import asyncio
import concurrent.futures as cf
import queue
import threading
import time
import traceback
from collections import Counter
from dataclasses import dataclass, field

from ..engine.llm import ContextFull
from ..ops.sampling import SamplingParams


@dataclass
class Session:
    rid: str
    events: asyncio.Queue
    loop: asyncio.AbstractEventLoop
    keep: bool = False
    oneshot: bool = False           # /v1/completions: end at the first chunk end
    want_lp: bool = False
    req: object = None              # engine.scheduler.Request
    n: int = 0
    sent: int = 0                   # tokens of seq.out already emitted
    closed: bool = False
    t_start: float = field(default_factory=time.time)

    @property
    def seq(self):
        return self.req.seq if self.req is not None else None


class EngineLoop:
    def __init__(self, llm, tokenizer, idle_wait: float = 0.02, prefill_budget: int = 4096, chunk: int = 2048):
        from ..engine.scheduler import Scheduler
        self.llm, self.tok = llm, tokenizer
        self.sched = Scheduler(llm, prefill_budget=prefill_budget, chunk=chunk)
        self.cmds: queue.Queue = queue.Queue()
        self.sessions: dict = {}
        self.by_req: dict = {}
        self.stats = Counter()
        self.idle_wait = idle_wait
        self._stop = threading.Event()
        self.thread = threading.Thread(target=self._run, name="engine", daemon=True)
        self.error = None

    def start(self):
        self.thread.start()
        return self

    def stop(self):
        self._stop.set()
        self.thread.join(timeout=30)

    @property
    def healthy(self) -> bool:
        return self.thread.is_alive() and self.error is None

    # ------------------------------------------------------------------------------------- handler side
    def submit(self, kind: str, **kw) -> cf.Future:
        fut = cf.Future()
        self.cmds.put((kind, kw, fut))
        return fut

    # ------------------------------------------------------------------------------------- engine side
    def _emit(self, s: Session, ev: dict):
        s.loop.call_soon_threadsafe(s.events.put_nowait, ev)

    def _emit_new_tokens(self, s: Session):
        out = s.seq.out
        if len(out) > s.sent:
            ids = out[s.sent:]
            ev = {"ids": ids, "text": self.tok.decode(ids)}
            if s.want_lp:
                ev["lp"] = s.seq.lps[s.sent:len(out)]
            s.n += len(ids)
            s.sent = len(out)
            self.stats["generated"] += len(ids)
            self._emit(s, ev)

    def _chunk_end(self, s: Session):
        seq = s.seq
        ev = {"chunk_end": seq.finish or "length", "n": s.n}
        if seq.ctx_full:
            ev["ctx_full"] = True
        self._emit(s, ev)
        if seq.ctx_full:
            self.stats["ctx_full"] += 1
            self._end(s, "ctx_full")
        elif s.oneshot or (seq.finish != "length" and not s.keep):
            self._end(s, "done")

    def _end(self, s: Session, why: str):
        if s.closed:
            return
        s.closed = True
        if s.req is not None:
            self.sched.close(s.req)
            self.by_req.pop(s.req.rid, None)
        self.sessions.pop(s.rid, None)
        self.stats["open"] -= 1
        self._emit(s, {"end": why, "n": s.n})

    def _start(self, kw, fut):
        s: Session = kw["session"]
        sp: SamplingParams = kw["sp"]
        if s.rid in self.sessions:
            fut.set_result((409, {"ok": False, "error": "session id in use"}))
            return
        try:
            req = self.sched.submit(kw["prompt_ids"], max_new_tokens=max(1, sp.max_tokens), sp=sp,
                                    keep_kv=not s.oneshot)
        except (ValueError, RuntimeError) as e:
            fut.set_result((400 if isinstance(e, ValueError) else 503, {"ok": False, "error": str(e)}))
            return
        s.req = req
        self.sessions[s.rid] = s
        self.by_req[req.rid] = s
        self.stats["sessions"] += 1
        self.stats["open"] += 1
        self.stats["start_tokens"] += len(kw["prompt_ids"])
        fut.set_result((200, {"ok": True}))

    def _push(self, kw, fut):
        s = self.sessions.get(kw["rid"])
        if s is None or s.closed:
            fut.set_result((404, {"ok": False, "error": "no such session"}))
            return
        req = s.req
        if not req.done:
            fut.set_result((409, {"ok": False, "error": "session is generating"}))
            return
        sp: SamplingParams = kw.get("sp")
        if sp is not None:
            sp.seed = req.seq.sp.seed if kw.get("seed") is None else sp.seed
        s.keep = bool(kw.get("keep", s.keep))
        try:
            self.sched.extend(req, kw["prompt_ids"], max(1, int(kw["max_tokens"])), sp=sp)
        except ContextFull:
            self.stats["push_refused"] += 1
            fut.set_result((409, {"ok": False, "error": "ctx_full", "held": len(req.history),
                                  "max_model_len": self.llm.ec.max_model_len}))
            self._end(s, "ctx_full")
            return
        self.stats["pushes"] += 1
        self.stats["pushed_tokens"] += len(kw["prompt_ids"])
        fut.set_result((200, {"ok": True}))

    def _close(self, kw, fut):
        s = self.sessions.get(kw["rid"])
        if s is not None:
            self._end(s, "closed")
        fut.set_result((200, {"ok": s is not None}))

    def _run(self):
        handlers = {"start": self._start, "push": self._push, "close": self._close}
        try:
            while not self._stop.is_set():
                busy = self.sched.has_work()
                try:
                    item = self.cmds.get_nowait() if busy else self.cmds.get(timeout=self.idle_wait)
                except queue.Empty:
                    item = None
                while item is not None:
                    kind, kw, fut = item
                    try:
                        handlers[kind](kw, fut)
                    except Exception as e:  # a bad request must not kill the engine thread
                        if not fut.done():
                            fut.set_result((500, {"ok": False, "error": repr(e)}))
                    try:
                        item = self.cmds.get_nowait()
                    except queue.Empty:
                        item = None
                if not self.sched.has_work():
                    continue
                produced = self.sched.step()
                self.stats["steps"] += 1
                for rid in produced:
                    s = self.by_req.get(rid)
                    if s is None or s.closed:
                        continue
                    self._emit_new_tokens(s)
                for rid in produced:
                    s = self.by_req.get(rid)
                    if s is not None and not s.closed and s.req.done:
                        self._chunk_end(s)
        except Exception:  # pragma: no cover - reported through /health
            self.error = traceback.format_exc()
            for s in list(self.sessions.values()):
                self._emit(s, {"end": "error", "n": s.n, "error": self.error[-500:]})

"""Continuous-batching scheduler over :class:`.llm.LLM`: requests are admitted while KV blocks and sequence slots
allow, prompts (and session pushes) are prefilled in chunks interleaved with the decode steps of the running
sequences, KV blocks grow as sequences generate, and when blocks run out the most recently admitted sequence is
preempted and later resumed by recomputation; idle sessions that keep their KV between turns are evicted, least
recently used first, when nothing else can make room.

The reference leaves this to vLLM's scheduler (chunked prefill, recompute preemption) plus its own session layer
(flashnext/kaggle/code_dataset/fnext/session/session_ep.py:145, idle-session eviction when the KV cache deadlocks;
resume_fix.py, exact resume). One iteration of :meth:`Scheduler.step`:

1. admission: waiting requests, first come first served; each needs a sequence slot (unless it still holds one)
   and KV blocks for everything it must prefill, while ``watermark`` blocks stay free for the decode growth of
   the running sequences; when the head of the queue does not fit and nothing is running or prefilling, idle
   sessions are evicted (then the external ``evict_idle`` callback is asked) before giving up;
2. prefill: up to ``prefill_budget`` tokens, in chunks of at most ``chunk`` tokens, oldest admission first; a
   request whose prefill completes samples its next token (unless it was preempted mid-decode, see below) and
   joins the running set;
3. decode: every running sequence first gets the block covering the position it feeds next (on exhaustion the
   newest running sequence is preempted), then one CUDA-graph decode step for all of them.

Every request keeps the exact list of tokens fed to its cache (``history``: prompt, then each decoded token as it
is fed, then pushed tokens, in order). A preempted or evicted request is rebuilt by prefilling its history: a
preempted one keeps its pending newest token and continues decoding from it (no token is sampled twice); an
evicted idle session prefills history + the pushed tokens when it is pushed again. Sampling randomness depends
only on (seed, position), so rebuilt sequences sample what they would have sampled.
"""
from __future__ import annotations

import collections
import itertools
import time
from dataclasses import dataclass, field

import torch

from ..ops.sampling import SamplingParams
from .llm import ContextFull, Sequence


@dataclass
class Request:
    rid: int
    prompt: list
    max_new: int
    sp: SamplingParams
    keep_kv: bool = False      # a session: its KV stays resident after a chunk ends, until closed or evicted
    seq: Sequence = None
    fed: list = None           # tokens to prefill, placed from position `base`
    base: int = 0
    cursor: int = 0            # prefill progress within `fed`
    history: list = field(default_factory=list)   # every token fed to the cache, in order
    resumed: bool = False      # rebuilt after preemption: its newest token is pending, nothing to sample
    holds_slot: bool = False   # slot and blocks still allocated (a kept session being pushed)
    evicted: bool = False      # an idle session whose KV was dropped
    offloaded: bool = False    # an idle session whose KV waits in the host tier
    closed: bool = False
    done: bool = False
    t_submit: float = 0.0
    t_first: float = 0.0
    t_idle: float = 0.0
    t_done: float = 0.0
    preemptions: int = 0

    @property
    def out(self) -> list:
        return self.seq.out[: self.max_new] if self.seq is not None else []


@dataclass
class SchedulerStats:
    admitted: int = 0
    preempted: int = 0
    evicted_sessions: int = 0
    offloaded_sessions: int = 0
    restored_sessions: int = 0
    prefill_tokens: int = 0
    decode_steps: int = 0
    generated: int = 0
    finished: int = 0
    blocked_admissions: int = 0


class Scheduler:
    def __init__(self, llm, prefill_budget: int = 4096, chunk: int = 2048, watermark: int = None,
                 evict_idle=None, host_tier=None):
        """``host_tier``: an :class:`.kv_tier.HostKVTier`; idle sessions are offloaded there before being dropped."""
        self.llm = llm
        self.host_tier = host_tier
        self.prefill_budget, self.chunk = prefill_budget, chunk
        self.bs = llm.ec.block_size
        # free blocks kept for the running sequences' next decode blocks
        self.watermark = watermark if watermark is not None else max(1, llm.ec.max_seqs // 2)
        self.evict_idle = evict_idle
        self.waiting = collections.deque()
        self.prefilling = []
        self.running = []          # admission order
        self.idle = []             # finished session chunks holding KV, least recently used first
        self.stats = SchedulerStats()
        self._ids = itertools.count()
        self._done_now = []

    def _blocks(self, n_tokens: int) -> int:
        return (n_tokens + self.bs - 1) // self.bs

    def has_work(self) -> bool:
        return bool(self.waiting or self.prefilling or self.running)

    # ------------------------------------------------------------------------------------------ requests
    def submit(self, prompt, max_new_tokens: int = 64, sp: SamplingParams = None, keep_kv: bool = False) -> Request:
        prompt = list(map(int, prompt))
        if not prompt:
            raise ValueError("empty prompt")
        need = len(prompt) + max_new_tokens
        if need > self.llm.ec.max_model_len:
            raise ValueError(f"request needs {need} tokens > max_model_len {self.llm.ec.max_model_len}")
        if self._blocks(len(prompt) + 1) > self.llm.caches.n_blocks - 1:
            raise ValueError("prompt larger than the whole KV cache")
        r = Request(next(self._ids), prompt, max_new_tokens, sp or SamplingParams(), keep_kv=keep_kv,
                    fed=list(prompt), t_submit=time.perf_counter())
        self.waiting.append(r)
        return r

    def extend(self, r: Request, tokens: list, max_new_tokens: int, sp: SamplingParams = None):
        """Push tokens to a finished session chunk and generate up to max_new_tokens more. The session's pending
        sampled token is dropped in favour of the pushed tokens (a continuation pushes it back first)."""
        if not r.done or r.closed:
            raise ValueError("extend needs a finished, open session chunk")
        tokens = list(map(int, tokens))
        if not tokens:
            raise ValueError("extend needs at least one token")
        held = len(r.history)
        if held + len(tokens) > self.llm.ec.max_model_len - 1:
            raise ContextFull(f"{held} held + {len(tokens)} pushed > max_model_len {self.llm.ec.max_model_len} - 1")
        seq = r.seq
        if sp is not None:
            seq.sp = sp
        seq.prompt += tokens
        seq.max_new = len(seq.out) + max_new_tokens
        r.max_new = seq.max_new
        seq.done, seq.finish, seq.ctx_full = False, "", False
        r.done, r.resumed = False, False
        if r in self.idle:
            self.idle.remove(r)
        if r.offloaded:
            r.fed, r.base, r.holds_slot = tokens, held, False
        elif r.evicted:
            r.fed, r.base, r.holds_slot = r.history + tokens, 0, False
        else:
            r.fed, r.base, r.holds_slot = tokens, held, True
        r.cursor = 0
        self.waiting.append(r)

    def close(self, r: Request):
        """Release a request's slot and KV (sessions: end of the session)."""
        if r.closed:
            return
        r.closed = True
        if r in self.idle:
            self.idle.remove(r)
        for q in (self.prefilling, self.running):
            if r in q:
                q.remove(r)
        if r in self.waiting:
            self.waiting.remove(r)
        if r.seq is not None and r.holds_slot:
            self._release(r)
        if r.offloaded and self.host_tier is not None:
            self.host_tier.drop(r.rid)
            r.offloaded = False

    def _release(self, r: Request):
        llm = self.llm
        llm.running.pop(r.seq.slot, None)
        llm.alloc.release(r.seq.slot)
        llm.model.reset_slot(r.seq.slot)
        llm.free_slots.append(r.seq.slot)
        r.holds_slot = False

    def _evict_one_idle(self) -> bool:
        if not self.idle:
            return False
        r = self.idle.pop(0)
        if self.host_tier is not None and self.host_tier.offload(r.rid, r.seq.slot):
            llm = self.llm                   # blocks went to the host tier; the slot is free for others
            llm.running.pop(r.seq.slot, None)
            llm.model.reset_slot(r.seq.slot)
            llm.free_slots.append(r.seq.slot)
            r.holds_slot = False
            r.offloaded = True
            self.stats.offloaded_sessions += 1
            return True
        self._release(r)
        r.evicted = True
        self.stats.evicted_sessions += 1
        return True

    # ------------------------------------------------------------------------------------------ admission
    def _admit(self):
        llm = self.llm
        while self.waiting:
            r = self.waiting[0]
            start = r.base if r.holds_slot else 0
            need = self._blocks(start + len(r.fed) + 1)
            extra = need - (llm.alloc.n_blocks_of(r.seq.slot) if r.holds_slot else 0)
            reserve = self.watermark if self.running else 0
            fits = (r.holds_slot or llm.free_slots) and llm.alloc.n_free() - extra >= reserve
            deadlock = not fits and not self.running and not self.prefilling
            if deadlock and self._evict_one_idle():
                continue
            if deadlock and self.evict_idle is not None and self.evict_idle():
                self.stats.evicted_sessions += 1
                continue
            if not fits:
                self.stats.blocked_admissions += 1
                return
            self.waiting.popleft()
            if not r.holds_slot:
                slot = llm.free_slots.pop()
                llm.model.reset_slot(slot)
                if r.seq is None:
                    r.seq = Sequence(slot, list(r.prompt), r.max_new, sp=r.sp)
                else:
                    r.seq.slot = slot
                if r.offloaded:              # KV and state come back from the host tier; prefill only the push
                    self.host_tier.restore(r.rid, slot)
                    r.offloaded = False
                    self.stats.restored_sessions += 1
                else:
                    r.base = 0
                r.holds_slot = True
                r.evicted = False
            llm.model.assign_blocks(r.seq.slot, r.base + len(r.fed) + 1, llm.alloc)
            r.seq.pos = r.base
            r.cursor = 0
            self.prefilling.append(r)
            self.stats.admitted += 1

    # ------------------------------------------------------------------------------------------ prefill
    def _prefill(self):
        llm, dev = self.llm, self.llm.device
        budget = self.prefill_budget
        for r in list(self.prefilling):
            if budget <= 0:
                break
            seq = r.seq
            x = None
            while r.cursor < len(r.fed) and budget > 0:
                n = min(self.chunk, budget, len(r.fed) - r.cursor)
                ids = torch.tensor(r.fed[r.cursor:r.cursor + n], dtype=torch.int32, device=dev)
                x = llm.model.step(ids, torch.tensor([seq.slot], dtype=torch.int32, device=dev),
                                   torch.tensor([r.base + r.cursor], dtype=torch.int32, device=dev), n_tok=n)
                r.cursor += n
                budget -= n
                self.stats.prefill_tokens += n
            if r.cursor < len(r.fed):
                continue
            seq.pos = r.base + len(r.fed)
            r.history = r.history[:r.base] + r.fed
            if not r.resumed:
                llm._append_sample(seq, x[-1:])
                if not r.t_first:
                    r.t_first = time.perf_counter()
            r.resumed = False
            self.prefilling.remove(r)
            if llm._finished(seq):
                self._chunk_done(r)
                self._done_now.append(r)
            else:
                llm.running[seq.slot] = seq
                self.running.append(r)

    # ------------------------------------------------------------------------------------------ decode
    def _preempt(self, r: Request):
        self.running.remove(r)
        self._release(r)
        r.fed, r.base = list(r.history), 0      # rebuild from everything fed; the newest token stays pending
        r.resumed = True
        r.preemptions += 1
        self.waiting.appendleft(r)
        self.stats.preempted += 1

    def _grow(self):
        """Blocks covering the position each running sequence feeds next; idle sessions are evicted first, then
        the newest running sequence is preempted."""
        llm = self.llm
        i = 0
        while i < len(self.running):
            r = self.running[i]
            need = self._blocks(r.seq.pos + 1)
            have = llm.alloc.n_blocks_of(r.seq.slot)
            if need <= have:
                i += 1
            elif llm.alloc.n_free() >= need - have:
                llm.model.assign_blocks(r.seq.slot, r.seq.pos + 1, llm.alloc)
                i += 1
            elif not self._evict_one_idle():
                self._preempt(self.running[-1])

    def _chunk_done(self, r: Request):
        r.done = True
        r.t_done = time.perf_counter()
        self.stats.finished += 1
        if r.keep_kv and not r.closed:
            r.t_idle = time.perf_counter()
            self.llm.running.pop(r.seq.slot, None)
            self.idle.append(r)
        else:
            self._release(r)

    def step(self) -> dict:
        """One scheduler iteration; returns {request id: [tokens produced this iteration]}."""
        self._admit()
        self._done_now = []
        before = {r.rid: len(r.seq.out) for r in self.prefilling + self.running}
        self._prefill()
        self._grow()
        if self.running:
            pending = {r.rid: r.seq.out[-1] for r in self.running}
            self.llm.step()
            self.stats.decode_steps += 1
            for r in self.running:
                r.history.append(pending[r.rid])       # the pending token was fed by this step
        res = {}
        for r in list(self.running) + self._done_now:
            new = r.seq.out[before.get(r.rid, len(r.seq.out)):]
            if new:
                res[r.rid] = new
                self.stats.generated += len(new)
            if r in self.running and r.seq.done:
                self.running.remove(r)
                self._chunk_done(r)
        return res

    def run(self, requests=None):
        """Iterate until the given requests (default: all work) are done."""
        while self.has_work():
            if requests is not None and all(r.done for r in requests):
                break
            self.step()

    def generate(self, prompts, max_new_tokens: int = 64, sp: SamplingParams = None) -> list:
        reqs = [self.submit(p, max_new_tokens, sp) for p in prompts]
        self.run(reqs)
        return [r.out for r in reqs]

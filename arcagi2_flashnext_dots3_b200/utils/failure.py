"""Failure detection for multi-process runs: host heartbeats, step-boundary checks, bounded device waits, and a
restart supervisor.

The reference detects failures with device waits that give up after a time limit and record an error code
(dotsnote/engine/arcstats_pkg/arcstats/host_ar.py:47-58, `_wait` :126-143), a monitor thread that reports the code
and optionally exits the process (`_monitor` :1224-1235), and a launcher that restarts the server up to three
times (flashnext/kaggle/code_dataset/kaggle_fn.sh:46-56). Here:

* device side: every spin-wait in this repository's kernels is bounded and writes a code to the per-device error
  word (:func:`..ops.native.check_error` raises :class:`..ops.native.DeviceWaitTimeout`); the context stays usable;
* :class:`Heartbeat`: each rank stamps a key in the process-group store every `period` seconds; a watcher thread
  marks peers whose stamp is older than `limit`; :meth:`Heartbeat.check` (called between steps, before any
  collective or peer kernel is launched) raises :class:`PeerFailure` so surviving ranks stop before they would
  wait on a dead peer;
* :class:`Supervisor`: runs a command, restarting it after a non-zero exit up to `max_restarts` times.

A rank leaves only between steps, with none of its kernels or collectives in flight.
"""
from __future__ import annotations

import os
import subprocess
import threading
import time


class PeerFailure(RuntimeError):
    """A peer rank stopped heartbeating."""


class Heartbeat:
    def __init__(self, store, rank: int, world: int, period: float = 0.2, limit: float = 2.0, prefix: str = "hb"):
        self.store, self.rank, self.world = store, rank, world
        self.period, self.limit, self.prefix = period, limit, prefix
        self.failed = set()
        self._stop = threading.Event()
        self._beat = threading.Thread(target=self._beat_loop, daemon=True)
        self._watch = threading.Thread(target=self._watch_loop, daemon=True)
        self.t_start = time.time()

    def start(self):
        self._stamp()
        self._beat.start()
        self._watch.start()
        return self

    def stop(self):
        """Stop heartbeating (a clean leave still looks like a failure to peers: they stop at their next step)."""
        self._stop.set()
        self._beat.join(timeout=5)
        self._watch.join(timeout=5)

    def _stamp(self):
        self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def _beat_loop(self):
        while not self._stop.wait(self.period):
            try:
                self._stamp()
            except Exception:  # the store host itself went away: peers will notice our silence
                return

    def _watch_loop(self):
        while not self._stop.wait(self.period):
            now = time.time()
            for r in range(self.world):
                if r == self.rank or r in self.failed:
                    continue
                try:
                    t = float(self.store.get(f"{self.prefix}/{r}").decode())
                except Exception:
                    t = self.t_start
                if now - t > self.limit:
                    self.failed.add(r)

    def check(self):
        """Call between steps: raises PeerFailure if any peer stopped heartbeating."""
        if self.failed:
            raise PeerFailure(f"rank(s) {sorted(self.failed)} stopped heartbeating (limit {self.limit:.1f}s)")


class StepGuard:
    """Step-boundary guard: peer heartbeat check before the step, device error word after it."""

    def __init__(self, heartbeat: Heartbeat | None = None, device=None):
        self.hb, self.device = heartbeat, device

    def __enter__(self):
        if self.hb is not None:
            self.hb.check()
        return self

    def __exit__(self, et, ev, tb):
        if et is None and self.device is not None:
            from ..ops import native
            import torch
            torch.cuda.synchronize(self.device)
            native.check_error(self.device)
        return False


class Supervisor:
    """Run `cmd`; restart after a non-zero exit (at most `max_restarts` times, `backoff` seconds apart)."""

    def __init__(self, cmd, max_restarts: int = 3, backoff: float = 1.0, env=None, log=print):
        self.cmd, self.max_restarts, self.backoff, self.env, self.log = cmd, max_restarts, backoff, env, log
        self.restarts = 0
        self.exit_codes = []

    def run(self) -> int:
        while True:
            rc = subprocess.call(self.cmd, env=self.env or dict(os.environ))
            self.exit_codes.append(rc)
            if rc == 0:
                return 0
            if self.restarts >= self.max_restarts:
                self.log(f"supervisor: giving up after {self.restarts} restarts (exit {rc})")
                return rc
            self.restarts += 1
            self.log(f"supervisor: exit {rc}, restart {self.restarts}/{self.max_restarts}")
            time.sleep(self.backoff)

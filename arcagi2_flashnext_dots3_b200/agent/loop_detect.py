"""Runaway-repetition monitor for streamed reasoning traces (the capability of the reference's
dotsnote/kaggle/runtime_dataset/loop_detect.py; detection rule and default parameters kept, code independent).

Rule: measure how well the most recent ``window`` characters compress (zlib level 6, compressed / raw bytes) at
every multiple of ``stride`` characters once ``max(window, min_chars)`` characters have streamed. Ordinary ARC
reasoning compresses to roughly 0.2-0.45; a loop (one sentence or token repeated) to a few percent. The trace is
flagged when every measurement over the last ``persist`` characters was below ``thr``. ``cut_at`` then points
one window before the low run began, where a caller truncates before forcing a conclusion.
"""
from __future__ import annotations

import zlib

__all__ = ["RepetitionMonitor", "first_fire", "compress_ratio"]


def compress_ratio(text: str) -> float:
    raw = text.encode("utf-8", "replace")
    return len(zlib.compress(raw, 6)) / max(1, len(raw))


class RepetitionMonitor:
    def __init__(self, window: int = 8192, stride: int = 1024, thr: float = 0.10, persist: int = 49152,
                 min_chars: int = 8192):
        self.cfg = (window, stride, thr, persist)
        self._text = []                # recent chunks, trimmed to the window
        self._len = 0
        self.total = 0
        self._mark = max(window, min_chars)
        self._low_run = None           # character count at the first low measurement of the current run
        self.fired_at = None
        self.cut_at = None
        self.ratios = []               # (characters seen, ratio) of every measurement

    def _recent(self) -> str:
        s = "".join(self._text)
        window = self.cfg[0]
        if len(s) > window:
            s = s[-window:]
        self._text, self._len = [s], len(s)
        return s

    def update(self, chunk: str) -> bool:
        """Feed newly streamed text; returns True from the moment the trace is judged a runaway loop."""
        if self.fired_at is not None:
            return True
        window, stride, thr, persist = self.cfg
        self._text.append(chunk)
        self._len += len(chunk)
        self.total += len(chunk)
        while self.total >= self._mark:
            r = compress_ratio(self._recent())
            self.ratios.append((self._mark, r))
            self._mark += stride
            if r >= thr:
                self._low_run = None
            elif self._low_run is None:
                self._low_run = self.total
            if self._low_run is not None and self.total - self._low_run >= persist:
                self.fired_at = self.total
                self.cut_at = max(0, self._low_run - window)
                return True
        return False


def first_fire(text: str, chunk: int = 256, **kw):
    """Where (in characters) the monitor flags a complete trace replayed in streaming-sized chunks, or None."""
    mon = RepetitionMonitor(**kw)
    for i in range(0, len(text), chunk):
        if mon.update(text[i:i + chunk]):
            return mon.fired_at
    return None

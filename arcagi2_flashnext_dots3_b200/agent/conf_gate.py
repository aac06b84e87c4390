"""Confidence gate for reasoning traces: stop attempts whose token confidence says they are doomed (the
capability of the reference's dotsnote/kaggle/runtime_dataset/conf_gate.py, a DeepConf-style signal,
arXiv 2508.15260; the feature definitions and the configuration string are kept, the code is independent).

Per generated token i: confidence c_i = -(mean of its top-k log-probabilities) and its sampled log-probability.
Group confidence at token n = mean of c over tokens n-group+1..n, taken at every n that is a multiple of
``stride`` once n >= group. Features of a trace so far:

* ``lowest_group``: the smallest group confidence;   ``bottom10_group``: mean of the lowest 10% of them;
* ``avg_conf``: mean c;   ``tail_conf``: mean c of the last ``group`` tokens;   ``neg_nll``: mean sampled log-prob.

(With no full group yet, the group features use the mean c of all tokens so far.) Checkpoints are token counts
with thresholds; when a trace reaches a checkpoint and its feature is below the threshold, the gate fires.
Configuration "<tokens>:<threshold>[,...]" (``ARC_CONF_KILL``), with ``ARC_CONF_FEATURE``, ``ARC_CONF_K`` and
``ARC_CONF_GROUP``; off when unset.
"""
from __future__ import annotations

import math
import os

import numpy as np

FEATURES = ("lowest_group", "bottom10_group", "avg_conf", "tail_conf", "neg_nll")


def parse_spec(spec) -> list:
    """'tokens:threshold,...' -> [(tokens, threshold)] sorted by tokens ('' or None -> [])."""
    pairs = [p.strip().split(":") for p in (spec or "").split(",") if p.strip()]
    return sorted((int(float(x)), float(t)) for x, t in pairs)


class ConfidenceGate:
    def __init__(self, checkpoints, feature: str = "lowest_group", k: int = 5, group: int = 2048,
                 stride: int = 256):
        if feature not in FEATURES:
            raise ValueError(f"unknown feature {feature}")
        self.checkpoints = sorted(checkpoints)
        self.feature, self.k, self.group, self.stride = feature, k, group, stride
        self._conf = []
        self._lp = []
        self._pending = list(self.checkpoints)
        self.fired_at = None
        self.evaluations = []          # (tokens, feature value, threshold)

    @classmethod
    def from_env(cls, env=None):
        env = os.environ if env is None else env
        cps = parse_spec(env.get("ARC_CONF_KILL", ""))
        return cls(cps, env.get("ARC_CONF_FEATURE", "lowest_group"), int(env.get("ARC_CONF_K", "5")),
                   int(env.get("ARC_CONF_GROUP", "2048"))) if cps else None

    def fresh(self):
        """A gate with the same settings and no tokens (one per attempt)."""
        return ConfidenceGate(self.checkpoints, self.feature, self.k, self.group, self.stride)

    @property
    def tokens(self) -> int:
        return len(self._conf)

    def feature_value(self):
        n = len(self._conf)
        if n == 0:
            return None
        c = np.asarray(self._conf, dtype=np.float64)
        if self.feature == "avg_conf":
            return float(c.mean())
        if self.feature == "neg_nll":
            return float(np.mean(self._lp))
        if self.feature == "tail_conf":
            return float(c[-self.group:].mean())
        csum = np.concatenate([[0.0], np.cumsum(c)])
        ends = np.arange(self.stride, n + 1, self.stride)
        ends = ends[ends >= self.group]
        groups = (csum[ends] - csum[ends - self.group]) / self.group if ends.size else np.array([c[-self.group:].mean()])
        if self.feature == "lowest_group":
            return float(groups.min())
        low = np.sort(groups)[: max(1, groups.size // 10)]
        return float(low.mean())

    def add(self, sampled_logprob, top_logprobs) -> bool:
        """Record one generated token; True when this token's count reaches a checkpoint the trace fails."""
        tops = sorted((float(v) for v in top_logprobs), reverse=True)[: self.k]
        self._conf.append(-sum(tops) / len(tops) if tops else 0.0)
        if sampled_logprob is None or (isinstance(sampled_logprob, float) and math.isnan(sampled_logprob)):
            sampled_logprob = tops[0] if tops else 0.0
        self._lp.append(float(sampled_logprob))
        if self.fired_at is not None or not self._pending or len(self._conf) < self._pending[0][0]:
            return False
        _, thr = self._pending.pop(0)
        v = self.feature_value()
        self.evaluations.append((len(self._conf), v, thr))
        if v is not None and v < thr:
            self.fired_at = len(self._conf)
            return True
        return False

    def add_openai(self, logprobs) -> bool:
        """Feed the ``logprobs`` object of one streamed completion chunk; True if the gate fired within it."""
        toks = (logprobs or {}).get("tokens") or []
        lps = logprobs.get("token_logprobs") or [None] * len(toks) if toks else []
        tops = logprobs.get("top_logprobs") or [None] * len(toks) if toks else []
        fired = False
        for lp, top in zip(lps, tops):
            fired = self.add(lp, (top or {}).values()) or fired
        return fired

    @property
    def exhausted(self) -> bool:
        """No checkpoint left to evaluate."""
        return not self._pending

"""Per-step binary log (spec-decode / serving step records) and its reader.

File format (the reference's steplog, dotsnote/engine/arcstats_pkg/arcstats/steplog.py: fixed-width int64
records): a 16-byte header (magic, number of fields) followed by records of `n_fields` int64 values. Writing
goes through the native buffered writer (`_host.StepLog`) when the host extension is built.
"""
from __future__ import annotations

import numpy as np

MAGIC = 0x474F4C50455453
FIELDS = ("t_us", "batch", "tokens", "drafted", "accepted", "prefill_tokens", "kv_blocks_free")


class StepLog:
    def __init__(self, path: str, fields=FIELDS):
        self.fields = tuple(fields)
        try:
            from .. import _host
            self._w = _host.StepLog(path, len(self.fields))
            self._py = None
        except ImportError:
            self._w = None
            self._py = open(path, "ab")
            if self._py.tell() == 0:
                self._py.write(np.array([MAGIC, len(self.fields)], dtype=np.int64).tobytes())

    def append(self, **kw):
        rec = [int(kw.get(f, 0)) for f in self.fields]
        if self._w is not None:
            self._w.append(rec)
        else:
            self._py.write(np.array(rec, dtype=np.int64).tobytes())

    def close(self):
        if self._w is not None:
            self._w.close()
        else:
            self._py.close()


def read(path: str, fields=FIELDS) -> dict:
    a = np.fromfile(path, dtype=np.int64)
    if a.size < 2 or a[0] != MAGIC:
        raise ValueError(f"{path}: not a step log")
    n = int(a[1])
    recs = a[2:].reshape(-1, n)
    return {f: recs[:, i] for i, f in enumerate(fields[:n])}

"""Loader for the in-tree sm_100a extension and the device error word.

On a machine with a CUDA device the extension is mandatory: :func:`C` raises if it is missing or was built for
another architecture, so no GPU path silently falls back to eager PyTorch. CPU tensors use the torch reference
implementations in :mod:`.ref` instead.

Kernels with bounded waits write a nonzero code into a per-device int32 error word when a wait gives up
(code = 1000 * role + step, see csrc/ptx.cuh). :func:`check_error` reads and clears it; :func:`ErrorMonitor`
polls it from a host thread, like the reference's AR timeout monitor
(dotsnote/engine/arcstats_pkg/arcstats/host_ar.py:1214-1235).
"""
from __future__ import annotations

import importlib
import os
import threading
import time

import torch

_C = None
_err = {}
DEFAULT_TIMEOUT_NS = int(float(os.environ.get("FW_WAIT_TIMEOUT_MS", "500")) * 1e6)


class NativeMissing(RuntimeError):
    pass


def C():
    """The compiled `_C` module (raises :class:`NativeMissing` if it is not built)."""
    global _C
    if _C is None:
        try:
            _C = importlib.import_module("arcagi2_flashnext_dots3_b200._C")
        except ImportError as e:  # pragma: no cover - exercised on GPU boxes without a build
            raise NativeMissing(
                "arcagi2_flashnext_dots3_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"(or __graft_entry__.build()). Import error: {e}") from e
    return _C


def available() -> bool:
    try:
        C()
        return True
    except NativeMissing:
        return False


def err_word(device=None) -> torch.Tensor:
    dev = torch.device(device or "cuda")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    w = _err.get(dev)
    if w is None:
        w = torch.zeros(4, dtype=torch.int32, device=dev)
        _err[dev] = w
    return w


class DeviceWaitTimeout(RuntimeError):
    pass


def check_error(device=None, clear=True):
    """Raise :class:`DeviceWaitTimeout` if a kernel on this device recorded a wait timeout."""
    w = err_word(device)
    code = int(w[0].item())
    if code:
        if clear:
            w.zero_()
        raise DeviceWaitTimeout(f"device wait timed out (code {code})")
    return 0


class ErrorMonitor:
    """Host thread that polls the error words of the given devices every `period` seconds and calls
    `on_error(device, code)` (default: log and remember). Reading a device word synchronizes nothing but a
    4-byte copy on a side stream."""

    def __init__(self, devices, period=1.0, on_error=None):
        self.devices = list(devices)
        self.period = period
        self.on_error = on_error or (lambda d, c: None)
        self.errors = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def start(self):
        self._t.start()
        return self

    def stop(self):
        self._stop.set()
        self._t.join(timeout=5)

    def _run(self):
        streams = {d: torch.cuda.Stream(device=d) for d in self.devices}
        while not self._stop.is_set():
            for d in self.devices:
                with torch.cuda.stream(streams[d]):
                    code = int(err_word(d)[0].item())
                if code:
                    self.errors.append((d, code))
                    self.on_error(d, code)
            time.sleep(self.period)

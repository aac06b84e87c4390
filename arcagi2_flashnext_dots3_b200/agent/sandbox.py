"""Sandboxed execution of model-written programs.

Each program runs in a fresh ``python -I`` child process in its own temporary directory, with the reference's
limits (flashnext/kaggle/code_dataset/repl_sandbox.py:60-70 and docs: 2 GiB address space, CPU seconds, 16 MiB
files, no core dumps, a wall-clock timeout that kills the whole process group) and an audit hook installed before
the program is compiled that refuses network access, subprocess creation and file writes outside the working
directory. The program must define ``transform(grid)``; the runner applies it to every train input (scored
against the train output) and every test input, and returns a JSON result.
"""
from __future__ import annotations

import asyncio
import json
import os
import resource
import shutil
import signal
import subprocess
import sys
import tempfile

RUNNER = r'''
import sys, json, io, os, contextlib, traceback, copy
_cwd = os.getcwd()
def _audit(event, args):
    if event in ("socket.connect", "socket.bind", "socket.getaddrinfo", "subprocess.Popen", "os.system",
                 "os.exec", "os.posix_spawn", "os.fork", "os.forkpty", "pty.spawn", "ctypes.dlopen"):
        raise PermissionError(f"{event} is not allowed in the sandbox")
    if event == "open" and len(args) > 1 and isinstance(args[0], str) and args[1] and any(c in str(args[1]) for c in "wax+"):
        p = os.path.abspath(args[0])
        if not p.startswith(_cwd):
            raise PermissionError(f"write outside the sandbox: {p}")
sys.path.insert(0, ".")
import numpy as np
import arckit as ak
sys.addaudithook(_audit)
D = json.load(open("task.json"))
train, test_inputs = D["train"], D["test_inputs"]
ns = {"np": np, "numpy": np, "ak": ak, "arckit": ak, "train": copy.deepcopy(train),
      "test_inputs": copy.deepcopy(test_inputs), "__name__": "__main__"}
buf = io.StringIO()
err = None
try:
    with contextlib.redirect_stdout(buf), contextlib.redirect_stderr(buf):
        exec(compile(open("code.py").read(), "<tool>", "exec"), ns)
except BaseException:
    err = "".join(traceback.format_exc().splitlines(True)[-6:])

def to_grid(x):
    g = np.asarray(x)
    if g.ndim != 2 or g.size == 0:
        raise ValueError(f"transform returned shape {g.shape}, expected a non-empty 2-D grid")
    out = [[int(v) for v in row] for row in g.tolist()]
    if len(out) > 30 or len(out[0]) > 30 or any(v < 0 or v > 9 for r in out for v in r):
        raise ValueError("transform returned an invalid ARC grid (values 0-9, at most 30x30)")
    return out

def call(f, g):
    with contextlib.redirect_stdout(io.StringIO()), contextlib.redirect_stderr(io.StringIO()):
        try:
            return to_grid(f(copy.deepcopy(g)))
        except ValueError:
            raise
        except Exception:
            return to_grid(f(np.array(g)))

res = {"stdout": buf.getvalue()[:2500], "error": err, "has_transform": callable(ns.get("transform"))}
if res["has_transform"]:
    f = ns["transform"]
    res["train"] = []
    for p in train:
        r = {}
        try:
            out = call(f, p["input"])
            r["out"], r["ok"] = out, out == p["output"]
        except BaseException as e:
            r["ok"], r["exc"] = False, (type(e).__name__ + ": " + str(e))[:300]
        res["train"].append(r)
    res["tests"] = []
    for g in test_inputs:
        try:
            res["tests"].append({"out": call(f, g)})
        except BaseException as e:
            res["tests"].append({"out": None, "exc": (type(e).__name__ + ": " + str(e))[:300]})
    if all(p.get("ok") for p in res["train"]) and all(t["out"] is not None for t in res["tests"]):
        try:
            res["flags"] = ak.flag(train, test_inputs, [t["out"] for t in res["tests"]])
        except Exception as e:
            res["flags_err"] = repr(e)[:200]
    try:   # the helper library's full report: masked diffs, leave-one-out, size / invariant / equivariance notes
        with contextlib.redirect_stdout(io.StringIO()), contextlib.redirect_stderr(io.StringIO()):
            res["check_text"] = ak.check(f, train, test_inputs, verbose=False)["text"][:4000]
    except BaseException as e:
        res["check_err"] = repr(e)[:200]
with open("result.json", "w") as fh:
    json.dump(res, fh)
'''

ARCKIT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "arckit.py")


def _limits(cpu_s: int, mem_bytes: int):
    def f():
        os.setsid()
        resource.setrlimit(resource.RLIMIT_AS, (mem_bytes, mem_bytes))
        resource.setrlimit(resource.RLIMIT_CPU, (cpu_s, cpu_s + 1))
        resource.setrlimit(resource.RLIMIT_FSIZE, (16 << 20, 16 << 20))
        resource.setrlimit(resource.RLIMIT_CORE, (0, 0))
    return f


def run_code_sync(code: str, task: dict, timeout: float = 25.0, cpu_s: int = 21, mem_bytes: int = 2 << 30) -> dict:
    d = tempfile.mkdtemp(prefix="fwsb_")
    try:
        with open(os.path.join(d, "task.json"), "w") as fh:
            json.dump({"train": task["train"], "test_inputs": [t["input"] for t in task["test"]]}, fh)
        with open(os.path.join(d, "code.py"), "w") as fh:
            fh.write(code)
        with open(os.path.join(d, "runner.py"), "w") as fh:
            fh.write(RUNNER)
        shutil.copyfile(ARCKIT, os.path.join(d, "arckit.py"))
        env = {"PATH": "/usr/bin:/bin", "OMP_NUM_THREADS": "1", "OPENBLAS_NUM_THREADS": "1", "HOME": d}
        p = subprocess.Popen([sys.executable, "-I", "runner.py"], cwd=d, env=env, stdout=subprocess.PIPE,
                             stderr=subprocess.PIPE, preexec_fn=_limits(cpu_s, mem_bytes))
        try:
            _, err = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            os.killpg(p.pid, signal.SIGKILL)
            p.communicate()
            return {"error": f"timeout after {timeout:.0f}s", "timeout": True, "has_transform": False}
        rp = os.path.join(d, "result.json")
        if p.returncode in (-signal.SIGXCPU, -signal.SIGKILL) and not os.path.exists(rp):
            return {"error": f"timeout (CPU limit {cpu_s}s)", "timeout": True, "has_transform": False}
        if not os.path.exists(rp):
            return {"error": (err.decode(errors="replace")[-800:] or f"sandbox exited with {p.returncode}"),
                    "has_transform": False, "rc": p.returncode}
        with open(rp) as fh:
            return json.load(fh)
    finally:
        shutil.rmtree(d, ignore_errors=True)


async def run_code(code: str, task: dict, timeout: float = 25.0, **kw) -> dict:
    return await asyncio.to_thread(run_code_sync, code, task, timeout, **kw)


def feedback(res: dict, task: dict, max_cells: int = 400) -> str:
    """Text fed back to the model: errors, and for each failing train pair the expected grid with matching cells
    masked ('.') against the program's output."""
    if res.get("timeout"):
        return "Your program timed out."
    if res.get("check_text") and res.get("has_transform"):
        parts = ["Error:\n" + res["error"]] if res.get("error") else []
        parts.append(res["check_text"])
        if res.get("stdout"):
            parts.append("Printed output:\n" + res["stdout"][:1500])
        return "\n".join(parts)
    parts = []
    if res.get("error"):
        parts.append("Error:\n" + res["error"])
    if not res.get("has_transform"):
        parts.append("Define a function transform(grid) that returns the output grid.")
        return "\n".join(parts)
    for k, (p, r) in enumerate(zip(task["train"], res.get("train", []))):
        if r.get("ok"):
            parts.append(f"train {k}: correct")
            continue
        if "exc" in r:
            parts.append(f"train {k}: exception {r['exc']}")
            continue
        exp, got = p["output"], r.get("out")
        if got is None or len(got) != len(exp) or len(got[0]) != len(exp[0]):
            shape = None if got is None else (len(got), len(got[0]))
            parts.append(f"train {k}: wrong shape {shape}, expected {(len(exp), len(exp[0]))}")
            continue
        if len(exp) * len(exp[0]) <= max_cells:
            masked = "\n".join("".join("." if e == g else str(g) for e, g in zip(er, gr)) for er, gr in zip(exp, got))
            parts.append(f"train {k}: wrong cells (dots match):\n{masked}")
        else:
            parts.append(f"train {k}: wrong")
    if res.get("flags"):
        parts.append("Warning: test outputs break train invariants: " + "; ".join(res["flags"]))
    if res.get("stdout"):
        parts.append("stdout:\n" + res["stdout"][:1000])
    return "\n".join(parts)

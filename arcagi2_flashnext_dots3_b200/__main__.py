"""Command-line entry point: ``python -m arcagi2_flashnext_dots3_b200 <command> [args]``.

Commands (each forwards its arguments to the module named):

  serve          HTTP server (server)                       solve         REPL solver against a server (agent)
  solve-direct   direct-answer solver (agent.d3_solver)     train-rl      RL repair training (training.train_rl)
  train-kd       distillation (training.kd)                 preflight     build/runtime checks (launch.preflight)
  package        offline bundle (launch.package)            gates         start-up gates on this GPU
  bench          headline decode benchmark (bench.py)       serve-bench   prefill + generation (launch.serve_bench)
  spec-bench     speculative decoding (launch.spec_bench)   d3-bench      D3 decode (launch.d3_bench)
  kbench         kernel microbenchmarks (launch.kbench)     ref-kernels   reference kernels vs ours
  compare        build comparison (evaluation.compare)      paired        paired bootstrap (evaluation.paired)
"""
from __future__ import annotations

import importlib
import json
import runpy
import sys
from pathlib import Path

COMMANDS = {
    "serve": "server.__main__", "solve": "agent.__main__", "solve-direct": "agent.d3_solver",
    "train-rl": "training.train_rl", "train-kd": "training.kd", "preflight": "launch.preflight",
    "package": "launch.package", "serve-bench": "launch.serve_bench", "spec-bench": "launch.spec_bench",
    "d3-bench": "launch.d3_bench", "kbench": "launch.kbench", "ref-kernels": "launch.ref_kernels",
    "compare": "evaluation.compare", "paired": "evaluation.paired",
}


def _gates(argv):
    import argparse
    ap = argparse.ArgumentParser(prog="gates")
    ap.add_argument("--log", default=None)
    ap.add_argument("--reps", type=int, default=10)
    a = ap.parse_args(argv)
    from .engine.gates import engine_gates
    for r in engine_gates("cuda", a.log, a.reps).run():
        print(json.dumps({"gate": r.name, "enabled": r.enabled, "err": r.err, "base_us": round(r.base_us, 1),
                          "cand_us": round(r.cand_us, 1)}))


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(__doc__)
        return 0
    cmd, rest = argv[0], argv[1:]
    if cmd == "gates":
        return _gates(rest)
    if cmd == "bench":
        sys.argv = ["bench.py"] + rest
        runpy.run_path(str(Path(__file__).resolve().parents[1] / "bench.py"), run_name="__main__")
        return 0
    if cmd not in COMMANDS:
        raise SystemExit(f"unknown command {cmd!r}; one of: gates, bench, {', '.join(COMMANDS)}")
    mod = importlib.import_module(f"{__package__}.{COMMANDS[cmd]}")
    sys.argv = [cmd] + rest
    fn = getattr(mod, "main")
    import inspect
    return fn(rest) if inspect.signature(fn).parameters else fn()   # some mains read sys.argv themselves


if __name__ == "__main__":
    main()

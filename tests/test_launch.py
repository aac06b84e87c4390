"""Launch layer on CPU: pre-flight checks of a build with deltas, offline bundles with an md5 manifest, the
command-line entry point."""
import json
import subprocess
import sys

import torch

from arcagi2_flashnext_dots3_b200.config import fn_small_config
from arcagi2_flashnext_dots3_b200.formats import deltas
from arcagi2_flashnext_dots3_b200.launch import package, preflight
from arcagi2_flashnext_dots3_b200.models import fn_loader, fn_weights


def _build(tmp_path):
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.random_dense(cfg, seed=0, symmetric=False)
    return fn_loader.save_build(W, cfg, tmp_path / "base")


def test_preflight_accepts_good_build_and_flags_corrupt_delta(tmp_path):
    base = _build(tmp_path)
    res = preflight.check_build(base)
    assert res and all(ok for _, ok, _ in res), res
    d = tmp_path / "delta"
    d.mkdir()
    torch.save({"weight": torch.zeros(3, 4)}, d / "router-L00.pt")     # wrong row count
    deltas.write_manifest(d)
    res = dict((n, ok) for n, ok, _ in preflight.check_build(base, [d]))
    assert res["manifest delta"] and not res["layer 0"]
    with open(d / "router-L00.pt", "ab") as f:
        f.write(b"x")
    assert not dict((n, ok) for n, ok, _ in preflight.check_build(base, [d]))["manifest delta"]


def test_bundle_manifest_roundtrip(tmp_path):
    base = _build(tmp_path)
    info = package.make_bundle(tmp_path / "bundle", base, copy_build=True)
    assert info["build_copied"] and (tmp_path / "bundle" / "run.sh").exists()
    assert package.verify_bundle(tmp_path / "bundle") == []
    victim = next((tmp_path / "bundle" / "code").rglob("config.py"))
    victim.write_text(victim.read_text() + "\n# edited\n")
    assert package.verify_bundle(tmp_path / "bundle") == [str(victim.relative_to(tmp_path / "bundle"))]


def test_cli_dispatch_help_and_unknown():
    r = subprocess.run([sys.executable, "-m", "arcagi2_flashnext_dots3_b200"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "serve-bench" in r.stdout
    r = subprocess.run([sys.executable, "-m", "arcagi2_flashnext_dots3_b200", "nope"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode != 0 and "unknown command" in r.stderr

"""Failure detection without any GPU fault: host-side rank failures on gloo ranks, a restart supervisor, and
(GPU) a bounded device wait that times out on a flag nothing sets and leaves the context usable."""
import os
import subprocess
import sys

import pytest
import torch

from arcagi2_flashnext_dots3_b200.utils.failure import Supervisor

HERE = os.path.dirname(os.path.abspath(__file__))


def _launch(mode, port):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "fail_worker.py"), mode]
    return subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=120)


def test_rank_leave_detected_by_heartbeat():
    r = _launch("leave", 29661)
    assert "RANK0_DETECTED_PEER_FAILURE" in r.stdout, (r.stdout[-2000:], r.stderr[-2000:])


def test_rank_exception_ends_peer_collective():
    r = _launch("raise", 29663)
    assert "RANK0_COLLECTIVE_ERROR" in r.stdout or "RANK0_DETECTED_PEER_FAILURE" in r.stdout, \
        (r.stdout[-2000:], r.stderr[-2000:])


def test_supervisor_restarts(tmp_path):
    flag = tmp_path / "n"
    code = ("import pathlib,sys; p=pathlib.Path(%r); n=int(p.read_text()) if p.exists() else 0; "
            "p.write_text(str(n+1)); sys.exit(0 if n >= 2 else 3)") % str(flag)
    sup = Supervisor([sys.executable, "-c", code], max_restarts=3, backoff=0.0, log=lambda m: None)
    assert sup.run() == 0 and sup.restarts == 2 and sup.exit_codes == [3, 3, 0]
    sup = Supervisor([sys.executable, "-c", "import sys; sys.exit(5)"], max_restarts=1, backoff=0.0,
                     log=lambda m: None)
    assert sup.run() == 5 and sup.restarts == 1


@pytest.mark.gpu
def test_device_wait_times_out_and_context_survives():
    from arcagi2_flashnext_dots3_b200.ops import native
    dev = torch.device("cuda")
    done = torch.zeros(2, dtype=torch.int64, device=dev)      # nothing ever sets these flags
    epoch = torch.ones(1, dtype=torch.int64, device=dev)
    err = native.err_word(dev)
    err.zero_()
    native.C().ep_wait_done(done, 2, epoch, err, int(0.2e9))  # 200 ms limit
    torch.cuda.synchronize()
    with pytest.raises(native.DeviceWaitTimeout):
        native.check_error(dev)
    a = torch.randn(256, 256, device=dev)
    assert torch.isfinite(a @ a).all()                        # the context is still usable
    native.check_error(dev)                                   # and the error word was cleared

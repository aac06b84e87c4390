"""Expert-parallel MoE: host-side plan/exchange on CPU gloo ranks, fused NVLink path on 2 GPUs."""
import os
import subprocess
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(nproc, comm, port, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "ep_worker.py"), comm]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "EP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])


def test_ep_exchange_cpu_two_ranks():
    _run(2, "nccl", 29631)


@pytest.mark.gpu
def test_ep_fused_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run(2, "fused", 29633, {"NCCL_NVLS_ENABLE": "0"})


@pytest.mark.gpu
def test_ep_nccl_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run(2, "nccl", 29635, {"NCCL_NVLS_ENABLE": "0", "EP_DEVICE": "cuda"})

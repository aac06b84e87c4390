"""Tensor-parallel D3 (heads + experts split, row-parallel o-projection and MoE partial sums all-reduced): gloo
ranks on CPU, fused NVLink all-reduce and NCCL on 2 GPUs."""
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
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "tp_worker.py"), comm]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "TP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])


def test_tp_cpu_two_ranks():
    _run(2, "nccl", 29681, {"CUDA_VISIBLE_DEVICES": ""})


@pytest.mark.gpu
@pytest.mark.parametrize("comm", ["fused", "nccl"])
def test_tp_two_gpus(comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run(2, comm, 29683 if comm == "fused" else 29685, {"NCCL_NVLS_ENABLE": "0", "TP_DEVICE": "cuda"})

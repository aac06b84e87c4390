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


def test_tp_cpu_two_ranks_sharded_index():
    """DSA index keys sharded by position mod 2: local select, all-gather, merge equals the replicated indexer."""
    _run(2, "nccl", 29695, {"CUDA_VISIBLE_DEVICES": "", "TP_SHARD_INDEX": "1"})


def test_tp_cpu_two_ranks_quantized_allreduce():
    """int8 two-shot all-reduce semantics on gloo ranks (the torch statement the GPU kernel is checked against)."""
    _run(2, "q8", 29687, {"CUDA_VISIBLE_DEVICES": "", "TP_DEVICE": "cpu"})


@pytest.mark.gpu
@pytest.mark.parametrize("comm", ["fused", "nccl", "q8"])
def test_tp_two_gpus(comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run(2, comm, {"fused": 29683, "nccl": 29685, "q8": 29689}[comm],
         {"NCCL_NVLS_ENABLE": "0", "TP_DEVICE": "cuda", "TP_SHARD_INDEX": "1" if comm == "fused" else "0"})


@pytest.mark.gpu
def test_tp_reduce_wait_times_out_with_error_code():
    """A source that never signals: the bounded wait of tp_reduce gives up, records 6401 + source and leaves the
    context usable (no peer needed: both source slots live on this GPU)."""
    from arcagi2_flashnext_dots3_b200.ops import native
    dev = torch.device("cuda")
    W, slot = 2, 4 * 256
    buf = torch.zeros(2, W, slot, device=dev)
    flags = torch.zeros(2, W, dtype=torch.int64, device=dev)
    epoch = torch.ones(1, dtype=torch.int64, device=dev)
    flags[1, 0] = 1          # source 0 signalled epoch 1 (parity 1); source 1 never does
    h = torch.ones(4, 256, device=dev)
    native.err_word(dev).zero_()
    native.C().tp_reduce(buf, flags, W, 4 * 256, slot, epoch, h, True, native.err_word(dev), 50_000_000)
    torch.cuda.synchronize()
    with pytest.raises(native.DeviceWaitTimeout, match="6402"):
        native.check_error(dev)
    assert bool((h == 1).all())                    # nothing was added
    assert float(torch.ones(3, device=dev).sum()) == 3.0   # the context still works


@pytest.mark.gpu
def test_quantized_allreduce_wait_times_out_with_error_code():
    """One launch of the int8 all-reduce as rank 0 of two, both ranks' areas on this GPU, rank 1 never running:
    its reduce-scatter wait gives up, records 6410 + 1 and leaves the context usable."""
    from arcagi2_flashnext_dots3_b200.ops import native
    dev = torch.device("cuda")
    W, n, G = 2, 4 * 256, 4
    nbytes = native.C().tp_qar_bytes(n, W, G)
    areas = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(W)]
    bases = torch.tensor([a.data_ptr() for a in areas], dtype=torch.int64, device=dev)
    epoch = torch.ones(1, dtype=torch.int64, device=dev)
    x = torch.randn(n, device=dev)
    h = torch.ones(n, device=dev)
    native.err_word(dev).zero_()
    native.C().tp_qar(x, h, n, bases, 0, n, G, epoch, native.err_word(dev), 50_000_000, 8, False, None)
    torch.cuda.synchronize()
    with pytest.raises(native.DeviceWaitTimeout, match="6411"):
        native.check_error(dev)
    assert bool((h == 1).all())
    assert float(torch.ones(3, device=dev).sum()) == 3.0


@pytest.mark.parametrize("nproc", [2, 3])
def test_vocab_sharded_pick_cpu(nproc):
    """Greedy and Gumbel-max temperature sampling over a vocabulary split across ranks equal the unsharded
    sampler exactly (ties resolved to the lowest index)."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={29690 + nproc}", os.path.join(HERE, "vocab_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "VOCAB_OK" in r.stdout, (r.stdout[-2000:], r.stderr[-3000:])


def test_fake_tp_rank_shapes_and_step():
    """One process emulating rank 0 of TP-2: weights at the shard's shapes (half the heads, half the experts,
    half the vocabulary), caches with the rank's heads, a decode step runs and picks ids inside the rank's slice."""
    from arcagi2_flashnext_dots3_b200.config import d3_small_config
    from arcagi2_flashnext_dots3_b200.models import d3_weights
    from arcagi2_flashnext_dots3_b200.parallel.fake_tp import fake_rank_model
    cfg = d3_small_config(num_layers=3, swa_n_heads=4, qk_nope_dim=64)
    m, W, c, grp = fake_rank_model(cfg, 2, "cpu", n_slots=2, max_len=32, block_size=8, shard_vocab=True)
    full = d3_weights.random_engine(cfg, "cpu", seed=0)
    assert m.cfg.n_heads == cfg.n_heads // 2 and grp.buf.shape == (2, 2, 64 * cfg.hidden_size)
    assert W["lm_head"].rows == full["lm_head"].rows // 2
    l_moe = next(l for l in range(cfg.num_layers) if cfg.is_moe(l))
    assert W["layers"][l_moe]["moe"]["gu"].n_experts == full["layers"][l_moe]["moe"]["gu"].n_experts // 2
    from arcagi2_flashnext_dots3_b200.engine.block_manager import BlockAllocator
    alloc = BlockAllocator(c.n_blocks, 2)
    m.assign_blocks(0, 8, alloc)
    x = m.step(torch.tensor([3, 4, 5], dtype=torch.int32), torch.tensor([0], dtype=torch.int32),
               torch.tensor([0], dtype=torch.int32), 3)
    ids = m.pick(x)
    assert ids.shape == (3,) and int(ids.max()) < W["vocab_range"][1]

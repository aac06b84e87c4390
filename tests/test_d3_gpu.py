"""Dots3-shaped model on the GPU: kernels (latent attention, DSA select, prep, routing) through the engine
against the CPU engine path (itself checked against the dense oracle), and greedy decode through the LLM API."""
import pytest
import torch

from arcagi2_flashnext_dots3_b200.config import EngineConfig, d3_small_config
from arcagi2_flashnext_dots3_b200.engine.block_manager import BlockAllocator
from arcagi2_flashnext_dots3_b200.engine.llm import LLM
from arcagi2_flashnext_dots3_b200.models import d3_reference as R
from arcagi2_flashnext_dots3_b200.models.d3 import D3Model, allocate_caches
from arcagi2_flashnext_dots3_b200.models.d3_weights import random_dense, to_engine
from arcagi2_flashnext_dots3_b200.ops import native

pytestmark = pytest.mark.gpu


def _run(dev, cfg, W, ids_list):
    c = allocate_caches(cfg, dev, len(ids_list), 64, block_size=16)
    m = D3Model(cfg, to_engine(W, cfg, dev), c, dev)
    alloc = BlockAllocator(c.n_blocks, len(ids_list))
    outs = []
    for s, ids in enumerate(ids_list):
        m.assign_blocks(s, 60, alloc)
        sl = torch.tensor([s], dtype=torch.int32, device=dev)
        x1 = m.step(ids[:19].to(dev), sl, torch.tensor([0], dtype=torch.int32, device=dev), 19)
        xs = [x1]
        for t in range(19, len(ids)):
            xs.append(m.step(ids[t:t + 1].to(dev), sl, torch.tensor([t], dtype=torch.int32, device=dev), 1))
        outs.append(m.logits(torch.cat(xs)).float().cpu())
    if dev != "cpu":
        torch.cuda.synchronize()
        native.check_error(torch.device(dev))
    return outs


def test_d3_engine_gpu_vs_cpu():
    cfg = d3_small_config()
    W = random_dense(cfg, seed=0)
    g = torch.Generator().manual_seed(4)
    ids = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (27, 33)]
    a = _run("cpu", cfg, W, ids)
    b = _run("cuda", cfg, W, ids)
    for x, y in zip(a, b):
        err = (x - y).abs().max() / x.abs().max()
        assert err < 5e-2, err   # the GPU's dense GEMMs quantize activations to e4m3 per 128-column group


def test_d3_llm_greedy_matches_oracle_prefix():
    cfg = d3_small_config()
    W = random_dense(cfg, seed=1)
    llm = LLM(cfg, to_engine(W, cfg, "cuda"), "cuda",
              EngineConfig(max_seqs=2, max_model_len=96, block_size=16, graph_batch_sizes=(2,)), model_cls=D3Model)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (20, 25)]
    outs = llm.generate(prompts, max_new_tokens=4)
    for p, o in zip(prompts, outs):
        ref = R.greedy(W, cfg, torch.tensor(p), 4)
        assert o[0] == ref[0]


def test_d3_index_share_gpu_vs_cpu():
    """Index sharing on the GPU (the shared layer's prep skips the index key; its attention reads the previous
    layer's top-k) agrees with the CPU engine path under the same pattern."""
    import dataclasses
    cfg = dataclasses.replace(d3_small_config(), index_share=True, dsa_pattern="FS")
    W = random_dense(cfg, seed=2)
    g = torch.Generator().manual_seed(5)
    ids = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (30,)]
    a = _run("cpu", cfg, W, ids)
    b = _run("cuda", cfg, W, ids)
    err = (a[0] - b[0]).abs().max() / a[0].abs().max()
    assert err < 5e-2, err   # e4m3 activations in the GPU's dense GEMMs (the CPU path keeps fp32)

"""Worker for the expert-parallel tests (launched once per rank). Compares the expert-parallel MoE layer of
every rank against the same layer with all experts local, on that rank's own tokens."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from arcagi2_flashnext_dots3_b200.config import fn_small_config  # noqa: E402
from arcagi2_flashnext_dots3_b200.models import fn_weights  # noqa: E402
from arcagi2_flashnext_dots3_b200.models.fn import FNModel, allocate_caches  # noqa: E402
from arcagi2_flashnext_dots3_b200.ops import fn_ops as ops  # noqa: E402
from arcagi2_flashnext_dots3_b200.ops import native  # noqa: E402
from arcagi2_flashnext_dots3_b200.parallel import ep as epm  # noqa: E402


def main():
    comm = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    cuda = comm == "fused" or os.environ.get("EP_DEVICE") == "cuda"
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    import datetime
    dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=120))
    cfg = fn_small_config(ple_layers=(), num_layers=2, n_experts=8, top_k=2)
    W = fn_weights.random_dense(cfg, seed=5, symmetric=False)
    full = fn_weights.to_engine(W, cfg, dev)
    local = fn_weights.to_engine(W, cfg, dev)
    epm.shard_model_experts(local, rank, world)
    c = allocate_caches(cfg, dev, 2, 64, block_size=16)
    ref_model = FNModel(cfg, full, c, dev)
    group = epm.EPGroup(cfg, rank, world, dev, max_tokens=32, comm=comm)
    ep_model = FNModel(cfg, local, c, dev, ep=group)
    g = torch.Generator().manual_seed(100 + rank)
    for it in range(3):  # several layers in a row: epochs advance, buffers are reused
        T = 5 + 3 * rank + it
        x = torch.randn(T, cfg.hidden_size, generator=g).to(dev, ops.act_dtype(dev))
        h0 = torch.randn(T, cfg.hc_count * cfg.hidden_size, generator=g).to(dev)
        inj = torch.rand(T, cfg.hc_count, generator=g).to(dev)
        p_ref = full["layers"][it % 2]["moe"]
        p_ep = local["layers"][it % 2]["moe"]
        h_ref = h0.clone()
        ref_model._moe(x, p_ref, h_ref, inj)
        h_ep = h0.clone()
        ep_model._moe(x, p_ep, h_ep, inj)
        if cuda:
            torch.cuda.synchronize()
            native.check_error(dev)
        err = (h_ep - h_ref).abs().max().item()
        scale = h_ref.abs().max().item()
        assert err <= 1e-3 * scale + 1e-4, (rank, it, err, scale)
    dist.barrier()
    if rank == 0:
        print("EP_OK", comm, world)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Worker for the tensor-parallel D3 tests: every rank runs its head/expert shard; logits of a prefill chunk and
decode steps must equal the single-process model on the same weights."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from arcagi2_flashnext_dots3_b200.config import d3_small_config  # noqa: E402
from arcagi2_flashnext_dots3_b200.engine.block_manager import BlockAllocator  # noqa: E402
from arcagi2_flashnext_dots3_b200.models.d3 import D3Model, allocate_caches  # noqa: E402
from arcagi2_flashnext_dots3_b200.models.d3_weights import random_dense, to_engine  # noqa: E402
from arcagi2_flashnext_dots3_b200.ops import native  # noqa: E402
from arcagi2_flashnext_dots3_b200.parallel.tp import TPGroup, shard_d3_weights, tp_config  # noqa: E402


def run(model, ids, dev, hidden=False):
    c = model.c
    alloc = BlockAllocator(c.n_blocks, 2)
    model.assign_blocks(0, 48, alloc)
    s0 = torch.tensor([0], dtype=torch.int32, device=dev)
    xs = [model.step(ids[:14].to(dev), s0, torch.tensor([0], dtype=torch.int32, device=dev), 14)]
    for t in range(14, ids.shape[0]):
        xs.append(model.step(ids[t:t + 1].to(dev), s0, torch.tensor([t], dtype=torch.int32, device=dev), 1))
    x = torch.cat(xs)
    return x if hidden else model.logits(x).float().cpu()


def main():
    comm = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    cuda = comm in ("fused", "q8") and os.environ.get("TP_DEVICE") != "cpu" or os.environ.get("TP_DEVICE") == "cuda"
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    import datetime
    dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=120))
    cfg = d3_small_config(num_layers=3, swa_n_heads=4, qk_nope_dim=64)
    W = random_dense(cfg, seed=4)
    ids = torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(5))
    ref = run(D3Model(cfg, to_engine(W, cfg, dev), allocate_caches(cfg, dev, 2, 64, block_size=16), dev), ids, dev)
    lc = tp_config(cfg, world)
    tp = TPGroup(rank, world, dev, max_tokens=32, hidden=cfg.hidden_size, comm=comm)
    m = D3Model(lc, to_engine(shard_d3_weights(W, cfg, rank, world), lc, dev),
                allocate_caches(lc, dev, 2, 64, block_size=16), dev, tp=tp)
    got = run(m, ids, dev)
    if cuda:
        torch.cuda.synchronize()
        native.check_error(dev)
    err = (got - ref).abs().max() / ref.abs().max()
    tol = 2e-2 if (cuda or comm == "q8") else 1e-4
    if comm == "nccl":
        # sequence parallel: residual rows split over the ranks, reduce-scatter / all-gather around the layers
        tps = TPGroup(rank, world, dev, max_tokens=32, hidden=cfg.hidden_size, comm="nccl", sequence_parallel=True)
        ms = D3Model(lc, to_engine(shard_d3_weights(W, cfg, rank, world), lc, dev),
                     allocate_caches(lc, dev, 2, 64, block_size=16), dev, tp=tps)
        got_sp = run(ms, ids, dev)
        if cuda:
            torch.cuda.synchronize()
        err_sp = float((got_sp - ref).abs().max() / ref.abs().max())
        assert err_sp < tol, (rank, "sp", err_sp)
    if comm == "q8":
        # the kernel's quantized all-reduce equals its torch statement on the gathered partials
        from arcagi2_flashnext_dots3_b200.parallel.tp import qar_reference
        g = torch.Generator().manual_seed(100 + rank)
        part = (torch.randn(13, cfg.hidden_size, generator=g) * (1 + rank)).to(dev)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        h = torch.full_like(part, 0.5)
        tp.allreduce_add(h, part)
        if cuda:
            torch.cuda.synchronize()
            native.check_error(dev)
        want = qar_reference([p.cpu() for p in parts]) + 0.5
        qerr = float((h.cpu() - want).abs().max() / want.abs().max())
        exact_sum = sum(p.cpu() for p in parts) + 0.5
        assert qerr < 1e-6, (rank, qerr)
        assert float((h.cpu() - exact_sum).abs().max() / exact_sum.abs().max()) < 2e-2
        # 4-bit payloads over a chain of all-reduces into one residual (one forward pass): with Hadamard rotation
        # and error feedback the residual keeps only about the last all-reduce's error
        errs = {}
        for name, kw in (("q4_ef", dict(comm="q4")),
                         ("q4_noef", dict(comm="q8", q_bits=4, hadamard=True, error_feedback=False))):
            tq = TPGroup(rank, world, dev, max_tokens=32, hidden=cfg.hidden_size, **kw)
            tq.begin_forward()
            hh = torch.zeros(13, cfg.hidden_size, device=dev)
            exact = torch.zeros(13, cfg.hidden_size)
            for l in range(6):
                gl = torch.Generator().manual_seed(1000 * l + 7)
                allp = [torch.randn(13, cfg.hidden_size, generator=gl) * (1 + r) for r in range(world)]
                tq.allreduce_add(hh, allp[rank].to(dev))
                exact += sum(allp)
            if cuda:
                torch.cuda.synchronize()
                native.check_error(dev)
            errs[name] = float((hh.cpu() - exact).abs().pow(2).mean().sqrt() / exact.abs().pow(2).mean().sqrt())
        assert errs["q4_ef"] < 0.6 * errs["q4_noef"] and errs["q4_ef"] < 0.08, (rank, errs)
    assert err < tol, (rank, float(err))
    if os.environ.get("TP_SHARD_INDEX") == "1":
        # index keys sharded by position mod world: same selection, same logits as the unsharded TP model
        import dataclasses
        lcs = dataclasses.replace(lc, shard_index=True)
        m3 = D3Model(lcs, to_engine(shard_d3_weights(W, cfg, rank, world), lcs, dev),
                     allocate_caches(lcs, dev, 2, 64, block_size=16, index_shards=world), dev, tp=tp)
        got3 = run(m3, ids, dev)
        if cuda:
            torch.cuda.synchronize()
            native.check_error(dev)
        err3 = float((got3 - got).abs().max() / got.abs().max())
        assert err3 < (2e-2 if cuda else 1e-5), (rank, err3)
    if not cuda:
        # LM head split across the ranks too: the sharded greedy pick equals the argmax of the full logits
        m2 = D3Model(lc, to_engine(shard_d3_weights(W, cfg, rank, world, shard_vocab=True), lc, dev),
                     allocate_caches(lc, dev, 2, 64, block_size=16), dev, tp=tp)
        picks = m2.pick(run(m2, ids, dev, hidden=True))
        assert picks.tolist() == ref.argmax(-1).tolist(), rank
    dist.barrier()
    if rank == 0:
        print("TP_OK", comm, world, float(err))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Smoke run of the flagship model on cuda:0: one tiny repair-training forward+backward of the FN-shaped
student (expert GEMMs on the tcgen05 kernel, scale gradients from the packed codes) and one engine decode step
(CUDA graph) of the same weights. Raises on any non-finite value or device error."""
from __future__ import annotations

import torch


def run_smoke(device: str = "cuda:0") -> dict:
    from ..config import EngineConfig, fn_small_config
    from ..engine.llm import LLM
    from ..models import fn_weights
    from ..ops import native
    from ..training.rl import seq_pg
    from ..training.student import FNStudent

    dev = torch.device(device)
    torch.cuda.set_device(dev)
    cfg = fn_small_config(num_layers=2, ple_layers=())
    W = fn_weights.random_dense(cfg, seed=0, symmetric=False)
    st = FNStudent(cfg, W, dev)
    ids = torch.randint(0, cfg.vocab_size, (48,), generator=torch.Generator().manual_seed(0))
    tot, stats = seq_pg(st, ids, torch.arange(24, 48), 1.0, chunk=16, grad=True)
    (-tot / 24).backward()
    torch.cuda.synchronize(dev)
    native.check_error(dev)
    gn = sum(float(p.grad.float().pow(2).sum()) for p in st.parameters() if p.grad is not None) ** 0.5
    if not (torch.isfinite(tot).item() and gn == gn and gn > 0):
        raise RuntimeError(f"smoke backward produced loss {float(tot)} grad norm {gn}")
    llm = LLM(cfg, fn_weights.to_engine(W, cfg, dev), dev,
              EngineConfig(max_seqs=2, max_model_len=128, block_size=16, graph_batch_sizes=(2,)))
    outs = llm.generate([[5, 6, 7, 8], [9, 10, 11]], max_new_tokens=3)
    torch.cuda.synchronize(dev)
    native.check_error(dev)
    return {"loss_lp_per_token": stats["lp"] / stats["n"], "grad_norm": gn, "decoded": outs}


if __name__ == "__main__":
    print(run_smoke())

"""Serve a model over HTTP: ``python -m arcagi2_flashnext_dots3_b200.server --model fn --build DIR``.

``--build`` loads a low-bit build directory (dense.pt + lowbit/router files); without it the model is random-init
of the named config (``fn``, ``fn-small``, ``tiny``, ``d3``, ``d3-small``), useful for load tests.
"""
from __future__ import annotations

import argparse

import torch


def build_llm(model: str, build: str | None, device: str, max_seqs: int, max_model_len: int, seed: int = 0):
    from ..config import EngineConfig, d3_config, d3_small_config, fn_config, fn_small_config, tiny_config
    from ..engine.llm import LLM
    graphs = tuple(b for b in (1, 2, 4, 8, 16, 32, 64, 128, 256) if b <= max_seqs) or (max_seqs,)
    ec = EngineConfig(max_seqs=max_seqs, max_model_len=max_model_len, block_size=64, graph_batch_sizes=graphs)
    if model.startswith("d3"):
        from ..models import d3_weights
        from ..models.d3 import D3Model
        cfg = {"d3": d3_config, "d3-small": d3_small_config}[model]()
        W = d3_weights.to_engine(d3_weights.random_dense(cfg, seed=seed), cfg, device)
        return cfg, LLM(cfg, W, device, ec, model_cls=D3Model)
    from ..models import fn_weights
    if build:
        from ..models.fn_loader import load_dense_build
        cfg, Wd = load_dense_build(build)
        return cfg, LLM(cfg, fn_weights.to_engine(Wd, cfg, device), device, ec)
    cfg = {"fn": fn_config, "fn-small": fn_small_config, "tiny": tiny_config}[model](ple_layers=())
    if model == "fn":
        W = fn_weights.random_engine(cfg, device, seed=seed)
    else:
        W = fn_weights.to_engine(fn_weights.random_dense(cfg, seed=seed), cfg, device)
    return cfg, LLM(cfg, W, device, ec)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="fn-small")
    ap.add_argument("--build", default=None)
    ap.add_argument("--tokenizer", default=None, help="local Hugging Face tokenizer directory (default: bytes)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-seqs", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=16384)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    import uvicorn
    from .app import create_app
    from .engine_loop import EngineLoop
    from .tokenizer import load_tokenizer
    cfg, llm = build_llm(a.model, a.build, a.device, a.max_seqs, a.max_model_len)
    eng = EngineLoop(llm, load_tokenizer(a.tokenizer)).start()
    uvicorn.run(create_app(eng, model_name=a.model), host=a.host, port=a.port, log_level="warning")


if __name__ == "__main__":
    main()

"""Repair-training driver (one process per GPU; `torchrun` for data parallel).

    python -m arcagi2_flashnext_dots3_b200.training.train_rl --data DIR --build BUILD --out OUT [--steps N]

`--data` holds rollout records (`*.npz` with `ids` int32 [L], `pos` int32 [n] generated-token positions, `adv`
float = leave-one-out advantage), as written by :func:`write_records`; `--build` is a low-bit build directory
(`lowbit-LNN.pt`, `router-LNN.pt`, plus the dense weights in `dense.pt`) or ``random:<config>`` for a
random-initialized model of a named config. Each optimizer step takes `--per-step` records over all replicas,
runs forward/backward per record (gradient checkpointing per layer), reduces the gradients with the overlapped
reduce-scatter of :class:`..parallel.zero.ShardedAdam`, updates, and appends one JSON line to `log.jsonl`.
`--resume` continues from OUT's checkpoint; the final trainables are exported as an FN delta in OUT/delta.
Options follow the reference's train_rl.py:45-72.
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

from ..config import fn_config, fn_small_config, tiny_config
from ..models import fn_weights
from ..parallel.zero import ShardedAdam
from . import checkpoint as ckpt
from .rl import lr_factor, seq_pg
from .student import FNStudent

CONFIGS = {"fn": fn_config, "fn-small": fn_small_config, "tiny": tiny_config}


def write_records(out_dir, seqs):
    """seqs: iterable of (ids, pos, adv). Writes rec-00000.npz ..."""
    os.makedirs(out_dir, exist_ok=True)
    for i, (ids, pos, adv) in enumerate(seqs):
        np.savez(os.path.join(out_dir, f"rec-{i:05d}.npz"), ids=np.asarray(ids, np.int32),
                 pos=np.asarray(pos, np.int32), adv=np.float32(adv))


def load_model_weights(build: str, layers: int | None):
    if build.startswith("random:"):
        name = build.split(":", 1)[1]
        kw = {"ple_layers": ()}
        if layers:
            kw["num_layers"] = layers
        cfg = CONFIGS[name](**kw)
        return cfg, fn_weights.random_dense(cfg, seed=0, symmetric=False)
    from ..models.fn_loader import load_dense_build
    return load_dense_build(build, layers)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--data", required=True)
    ap.add_argument("--build", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--steps", type=int, default=0, help="0 = one pass over the data (--epochs)")
    ap.add_argument("--epochs", type=float, default=1.0)
    ap.add_argument("--per-step", type=int, default=48)
    ap.add_argument("--tok-norm", type=float, default=16384.0)
    ap.add_argument("--trainable", default="scales,router")
    ap.add_argument("--lr-scales", type=float, default=3e-4)
    ap.add_argument("--lr-router", type=float, default=1.5e-5)
    ap.add_argument("--lr-norms", type=float, default=1e-5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--clip-adv", type=float, default=2.0)
    ap.add_argument("--ppo-clip", type=float, default=0.0)
    ap.add_argument("--chunk", type=int, default=1024)
    ap.add_argument("--resume", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--save-every", type=int, default=0)
    ap.add_argument("--dry", action="store_true", help="forward/backward only, no optimizer step")
    ap.add_argument("--write-synthetic", type=int, nargs=2, metavar=("N", "L"), default=None,
                    help="write N random rollout records of L tokens (second half generated) into --data and exit")
    ap.add_argument("--no-overlap", action="store_true",
                    help="reduce the gradients after the whole backward instead of from the backward's hooks")
    a = ap.parse_args(argv)

    if a.write_synthetic:
        n, L = a.write_synthetic
        cfg, _ = load_model_weights(a.build, 1) if not a.build.startswith("random:") else (
            CONFIGS[a.build.split(":", 1)[1]](), None)
        rng = np.random.default_rng(a.seed)
        write_records(a.data, [(rng.integers(0, cfg.vocab_size, L), np.arange(L // 2, L), float(rng.normal()))
                               for _ in range(n)])
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dev = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(minutes=30))
    out = Path(a.out)
    if rank == 0:
        out.mkdir(parents=True, exist_ok=True)
        json.dump(vars(a), open(out / "args.json", "w"), indent=1)
    cfg, W = load_model_weights(a.build, a.layers)
    model = FNStudent(cfg, W, dev, train_norms="norms" in a.trainable)
    for m in model.moe:
        m.t_gu.requires_grad_("scales" in a.trainable)
        m.t_d.requires_grad_("scales" in a.trainable)
        m.router.requires_grad_("router" in a.trainable)
    groups = [g for g in model.param_groups(a.lr_scales, a.lr_router, a.lr_norms)
              if all(p.requires_grad for p in g["params"])]
    opt = ShardedAdam(groups, overlap=not a.no_overlap)
    files = sorted(glob.glob(os.path.join(a.data, "*.npz")))
    if not files:
        raise SystemExit(f"no records in {a.data}")
    total = a.steps or max(1, int(len(files) * a.epochs) // a.per_step)
    step = ckpt.load(out, model, opt, rank) if a.resume and (out / "trained.pt").exists() else 0
    rng = np.random.default_rng(a.seed)
    order = []
    while len(order) < total * a.per_step:
        order.extend(rng.permutation(len(files)).tolist())
    logf = open(out / "log.jsonl", "a") if rank == 0 else None
    while step < total:
        t0 = time.time()
        if cuda:                             # device time of the step (backward + reduction + update), max over ranks
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            ev0.record()
        batch = order[step * a.per_step:(step + 1) * a.per_step][rank::world]
        opt.zero_grad()
        st = {"lp": 0.0, "ent": 0.0, "n": 0, "clipped": 0}
        for i, fi in enumerate(batch):
            z = np.load(files[fi])
            A = float(np.clip(float(z["adv"]), -a.clip_adv, a.clip_adv))
            tot, s = seq_pg(model, z["ids"], z["pos"], A, a.chunk, grad=True)
            loss = -tot / (a.per_step * a.tok_norm)
            opt.last_backward = i == len(batch) - 1
            loss.backward()
            for k in st:
                st[k] += s[k]
        if not batch:  # a rank without records still takes part in the collectives
            opt.last_backward = True
        gnorm = None
        if not a.dry:
            opt.finish_reduction()
            gnorm = opt.grad_norm()
            opt.step(lr_factor(step, total, a.warmup))
        step += 1
        dev_ms = None
        if cuda:
            ev1.record()
            torch.cuda.synchronize()
            t = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dev_ms = round(float(t), 2)
        if logf:
            logf.write(json.dumps({"step": step, "loss_lp": st["lp"] / max(1, st["n"]), "ent": st["ent"] / max(1, st["n"]),
                                   "tokens": st["n"], "grad_norm": gnorm, "lr_factor": lr_factor(step - 1, total, a.warmup),
                                   "s": round(time.time() - t0, 3), "step_ms_device_max_ranks": dev_ms,
                                   "overlap": not a.no_overlap, "world": world}) + "\n")
            logf.flush()
        if a.save_every and step % a.save_every == 0:
            ckpt.save(out, step, model, opt, rank)
    ckpt.save(out, step, model, opt, rank)
    if rank == 0 and not a.build.startswith("random:"):
        from ..models.fn_loader import expert_layers
        ckpt.export_delta(model, expert_layers(a.build, a.layers), out / "delta",
                          keep_json=os.path.join(a.build, "keep.json"))
    if world > 1:
        dist.barrier()
    return step


if __name__ == "__main__":
    main()

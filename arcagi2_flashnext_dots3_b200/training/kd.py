"""Knowledge distillation of the FN student against a teacher's top-K next-token distributions.

The recipe is the reference's (flashnext/training/kd/train_kd.py `kl21`, `load`, `tool_weights`; teacher dumps
from kd/dump.py): over the generated positions of recorded sequences, KL(teacher || student) on 21 bins, the
teacher's top-20 tokens plus one tail bin holding the remaining mass of each distribution; positions inside
tool-call spans may be weighted differently. Only the student's trainables (expert scales, router rows,
optionally norms) learn.

Record format (``*.npz``): ``ids`` int32 [L], ``plen`` int (prompt length), ``gen`` int [n, 2] half-open ranges of
generated positions, ``top_ids`` int32 [n_gen, K] / ``top_lp`` fp32 [n_gen, K] teacher top-K per generated
position in order (id -1 pads unused slots).

The student's log-probabilities at the teacher's K tokens come from :class:`VocabTopK`, which keeps only the
hidden rows and recomputes each row chunk's [rows, vocab] projection in backward.

    python -m arcagi2_flashnext_dots3_b200.training.kd --data DIR --build BUILD --out OUT [--steps N]
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

TOOL_OPEN, TOOL_CLOSE = 248058, 248059   # FN chat template's tool-call delimiters


class VocabTopK(torch.autograd.Function):
    """log softmax(h W^T) at K token ids per row: [rows, K]. Backward: d z = scatter(g) - softmax(z) * sum(g),
    recomputed chunk by chunk."""

    @staticmethod
    def forward(ctx, h, W, ids, rows: int):
        Wf = W.float()
        out = torch.empty(ids.shape, dtype=torch.float32, device=h.device)
        lse = torch.empty(h.shape[0], dtype=torch.float32, device=h.device)
        for s in range(0, h.shape[0], rows):
            z = h[s:s + rows].float() @ Wf.t()
            lse[s:s + rows] = torch.logsumexp(z, -1)
            out[s:s + rows] = z.gather(1, ids[s:s + rows]) - lse[s:s + rows, None]
        ctx.save_for_backward(h, W, ids, lse)
        ctx.rows = rows
        return out

    @staticmethod
    def backward(ctx, g):
        h, W, ids, lse = ctx.saved_tensors
        Wf = W.float()
        dh = torch.empty_like(h) if ctx.needs_input_grad[0] else None
        dW = torch.zeros_like(Wf) if ctx.needs_input_grad[1] else None
        for s in range(0, h.shape[0], ctx.rows):
            hs = h[s:s + ctx.rows].float()
            gs = g[s:s + ctx.rows].float()
            d = (hs @ Wf.t()).sub_(lse[s:s + ctx.rows, None]).exp_().mul_(-gs.sum(1, keepdim=True))
            d.scatter_add_(1, ids[s:s + ctx.rows], gs)
            if dh is not None:
                dh[s:s + ctx.rows] = (d @ Wf).to(dh.dtype)
            if dW is not None:
                dW.addmm_(d.t(), hs)
        return dh, (dW.to(W.dtype) if dW is not None else None), None, None


def kl21(student_lp_k: torch.Tensor, t_ids: torch.Tensor, t_lp: torch.Tensor):
    """Per-row KL(teacher || student) over the teacher's top-K bins plus a tail bin. student_lp_k [n, K] are the
    student's log-probs at t_ids (padding ids < 0 masked out)."""
    valid = t_ids >= 0
    lt = torch.where(valid, t_lp.float(), torch.full_like(t_lp.float(), -1e4))
    pt = lt.exp()
    ps = torch.where(valid, student_lp_k.exp(), torch.zeros_like(student_lp_k))
    tail_t = (1 - pt.sum(1)).clamp_min(1e-8)
    tail_s = (1 - ps.sum(1)).clamp_min(1e-8)
    top = (pt * (lt - student_lp_k)).masked_fill(~valid, 0).sum(1)
    return top + tail_t * (tail_t.log() - tail_s.log())


def load_record(path, max_len: int = 0):
    """(ids, positions scored, teacher ids, teacher log-probs) of one record; position p is scored from the
    hidden state at p - 1, so the first position and prompt positions are never scored."""
    z = np.load(path)
    ids = z["ids"][:max_len] if max_len else z["ids"]
    plen = int(z["plen"])
    mask = np.zeros(len(ids), bool)
    for a, b in z["gen"]:
        mask[a:min(b, len(ids))] = True
    mask[:max(plen, 1)] = False
    pos = np.nonzero(mask)[0]
    return ids, pos, z["top_ids"][pos - plen], z["top_lp"][pos - plen]


def tool_weights(ids, pos, w_tool: float):
    """Per scored position: w_tool inside tool-call spans (delimiters included), 1 elsewhere."""
    w = np.ones(len(pos), np.float32)
    if w_tool == 1.0:
        return w
    inside = np.zeros(len(ids), bool)
    start = None
    for i, t in enumerate(ids):
        if t == TOOL_OPEN:
            start = i
        elif t == TOOL_CLOSE and start is not None:
            inside[start:i + 1] = True
            start = None
    w[inside[pos]] = w_tool
    return w


def seq_kd(model, path, chunk: int = 1024, grad: bool = True, w_tool: float = 1.0, max_len: int = 0):
    """(weighted KL sum tensor, stats) of one record, or None when it has no scored position."""
    ids, pos, tid, tlp = load_record(path, max_len)
    if len(pos) == 0:
        return None
    dev = model.device
    ctx = torch.enable_grad() if grad else torch.no_grad()
    with ctx:
        h = model.hidden(torch.as_tensor(ids, dtype=torch.long, device=dev), ckpt=grad)
        at = torch.as_tensor(pos, device=dev)
        tid_t = torch.as_tensor(tid, dtype=torch.long, device=dev)
        rows = h.index_select(0, at - 1)
        lp_k = VocabTopK.apply(rows, model.lm_head, tid_t.clamp_min(0), max(1, chunk))
        kl = kl21(lp_k, tid_t, torch.as_tensor(tlp, device=dev))
        w = torch.as_tensor(tool_weights(ids, pos, w_tool), device=dev)
        loss = (kl * w).sum()
    agree = float((lp_k.detach().argmax(1) == 0).float().sum())   # student's best of the K is the teacher's top-1
    return loss, {"kl": float(kl.detach().sum()), "n": len(pos), "agree": agree}


def write_kd_records(out_dir, seqs):
    """seqs: iterable of (ids, plen, gen ranges, top_ids, top_lp). Writes kd-00000.npz ..."""
    os.makedirs(out_dir, exist_ok=True)
    for i, (ids, plen, gen, tid, tlp) in enumerate(seqs):
        np.savez(os.path.join(out_dir, f"kd-{i:05d}.npz"), ids=np.asarray(ids, np.int32), plen=np.int64(plen),
                 gen=np.asarray(gen, np.int64).reshape(-1, 2), top_ids=np.asarray(tid, np.int32),
                 top_lp=np.asarray(tlp, np.float32))


def main(argv=None):
    from ..parallel.zero import ShardedAdam
    from . import checkpoint as ckpt
    from .rl import lr_factor
    from .student import FNStudent
    from .train_rl import load_model_weights
    ap = argparse.ArgumentParser()
    ap.add_argument("--data", required=True)
    ap.add_argument("--build", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--steps", type=int, default=0)
    ap.add_argument("--per-step", type=int, default=16)
    ap.add_argument("--trainable", default="scales,router")
    ap.add_argument("--lr-scales", type=float, default=1e-4)
    ap.add_argument("--lr-router", type=float, default=1e-5)
    ap.add_argument("--lr-norms", type=float, default=1e-5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tool-weight", type=float, default=1.0)
    ap.add_argument("--max-len", type=int, default=0)
    ap.add_argument("--chunk", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--resume", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
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
    cfg, W = load_model_weights(a.build, a.layers)
    model = FNStudent(cfg, W, dev, train_norms="norms" in a.trainable)
    for m in model.moe:
        m.t_gu.requires_grad_("scales" in a.trainable)
        m.t_d.requires_grad_("scales" in a.trainable)
        m.router.requires_grad_("router" in a.trainable)
    opt = ShardedAdam([g for g in model.param_groups(a.lr_scales, a.lr_router, a.lr_norms)
                       if all(p.requires_grad for p in g["params"])])
    files = sorted(glob.glob(os.path.join(a.data, "*.npz")))
    if not files:
        raise SystemExit(f"no records in {a.data}")
    total = a.steps or max(1, len(files) // a.per_step)
    step = ckpt.load(out, model, opt, rank) if a.resume and (out / "trained.pt").exists() else 0
    rng = np.random.default_rng(a.seed)
    order = []
    while len(order) < total * a.per_step:
        order.extend(rng.permutation(len(files)).tolist())
    log = open(out / "log.jsonl", "a") if rank == 0 else None
    while step < total:
        t0 = time.time()
        batch = order[step * a.per_step:(step + 1) * a.per_step][rank::world]
        opt.zero_grad()
        st = {"kl": 0.0, "n": 0, "agree": 0.0}
        n_tok = sum(len(load_record(files[i], a.max_len)[1]) for i in batch)
        for i, fi in enumerate(batch):
            r = seq_kd(model, files[fi], a.chunk, True, a.tool_weight, a.max_len)
            opt.last_backward = i == len(batch) - 1
            if r is None:
                continue
            loss, s = r
            (loss / max(1, n_tok)).backward()
            for k in st:
                st[k] += s[k]
        opt.last_backward = True
        opt.finish_reduction()
        opt.step(lr_factor(step, total, a.warmup))
        step += 1
        if log:
            log.write(json.dumps({"step": step, "kl": st["kl"] / max(1, st["n"]), "agree": st["agree"] / max(1, st["n"]),
                                  "tokens": st["n"], "s": round(time.time() - t0, 3)}) + "\n")
            log.flush()
    ckpt.save(out, step, model, opt, rank)
    if world > 1:
        dist.barrier()
    return step


if __name__ == "__main__":
    main()

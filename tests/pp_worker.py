"""Worker for the pipeline-parallel test: two stages of the FN student over gloo; per-stage trainable gradients
and the losses must equal a single-process student's on the same micro-batches."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from arcagi2_flashnext_dots3_b200.config import fn_small_config  # noqa: E402
from arcagi2_flashnext_dots3_b200.models import fn_weights  # noqa: E402
from arcagi2_flashnext_dots3_b200.parallel.pipeline import PipelineStage  # noqa: E402
from arcagi2_flashnext_dots3_b200.training import rl  # noqa: E402
from arcagi2_flashnext_dots3_b200.training.student import FNStudent  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo")
    cfg = fn_small_config(num_layers=3, ple_layers=())
    W = fn_weights.random_dense(cfg, seed=0, symmetric=False)
    mbs = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n)) for n in (20, 27, 16)]

    def objective(model, h, m):
        ids = mbs[m]
        pos = torch.arange(8, len(ids))
        lp = rl.VocabLogProb.apply(h[pos - 1], model.lm_head, ids[pos].long(), 8)
        return -(0.5 + m) * lp.sum() / 100.0
    stage = PipelineStage(cfg, W, "cpu", rank, world)
    losses = stage.step(mbs, objective)
    ref = FNStudent(cfg, W, "cpu")
    ref_losses = []
    for m, ids in enumerate(mbs):
        loss = objective(ref, ref.hidden(ids, ckpt=True), m)
        loss.backward()
        ref_losses.append(float(loss))
    if stage.last:
        assert all(abs(a - b) < 1e-5 * max(1.0, abs(b)) for a, b in zip(losses, ref_losses)), (losses, ref_losses)
    for j, l in enumerate(range(stage.a, stage.b)):
        g, gr = stage.student.moe[j].t_gu.grad, ref.moe[l].t_gu.grad
        assert g is not None and torch.allclose(g, gr, rtol=1e-4, atol=1e-7), (rank, l, float((g - gr).abs().max()))
    dist.barrier()
    if rank == 0:
        print("PP_OK", world)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Worker for the vocabulary-sharded pick test: every rank holds a slice of the same logits; the sharded greedy
and Gumbel-max picks must equal the unsharded sampler's."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from arcagi2_flashnext_dots3_b200.ops import sampling  # noqa: E402
from arcagi2_flashnext_dots3_b200.parallel.tp import sharded_pick, vocab_range  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo")
    V, T = 1003, 6
    logits = torch.randn(T, V, generator=torch.Generator().manual_seed(1)) * 3
    logits[2, 10] = logits[2, 900] = logits[2].max() + 1     # a tie across ranks: the lower index wins
    v0, v1 = vocab_range(V, rank, world)
    got = sharded_pick(logits[:, v0:v1], v0)
    assert got.tolist() == logits.argmax(-1).tolist(), (got.tolist(), logits.argmax(-1).tolist())
    for seed, step, temp in [(3, 0, 1.0), (77, 12, 0.7)]:
        got = sharded_pick(logits[:, v0:v1], v0, temperature=temp, seed=seed, step=step)
        want = [sampling._sample_row(logits[r], temp, 0, 1.0, seed, step) for r in range(T)]
        assert got.tolist() == want, (got.tolist(), want)
    # top-k / top-p over the split head: the unsharded CPU sampler's tokens
    from arcagi2_flashnext_dots3_b200.parallel.tp import sharded_sample
    lgk = logits.clone()
    lgk[4, 5] = lgk[4, 995] = lgk[4].max() + 0.5      # a tie inside the top k across ranks
    for seed, step, temp, k, p in [(5, 1, 1.0, 20, 1.0), (6, 3, 0.8, 0, 0.9), (7, 8, 1.3, 50, 0.5),
                                   (8, 0, 0.6, 3, 0.95), (9, 2, 1.0, 2000, 0.99)]:
        got = sharded_sample(lgk[:, v0:v1], v0, V, temperature=temp, top_k=k, top_p=p, seed=seed, step=step)
        want = [sampling._sample_row(lgk[r], temp, k, p, seed, step) for r in range(T)]
        assert got.tolist() == want, (seed, got.tolist(), want)
    # speculative verification over the split head: same accepted counts and next tokens as unsharded
    from arcagi2_flashnext_dots3_b200.parallel.tp import sharded_speculative_accept
    B, k = 5, 3
    lg = torch.randn(B, k + 1, V, generator=torch.Generator().manual_seed(2)) * 2
    drafts = lg[:, :k].argmax(-1)
    drafts[1, 1] = (drafts[1, 1] + 7) % V            # a greedy row rejected at position 1
    drafts[3, 0] = 900                               # a draft owned by the last rank
    temps, seeds, steps = [0.0, 0.0, 0.9, 1.2, 0.5], [1, 2, 3, 4, 5], [0, 4, 9, 2, 30]
    want = sampling.speculative_accept(lg, drafts, temps, seeds, steps)
    got = sharded_speculative_accept(lg[..., v0:v1].contiguous(), v0, drafts, temps, seeds, steps)
    assert got == want, (got, want)
    acc, nxt = want
    assert acc[0] == k and nxt[0] == int(lg[0, k].argmax())        # greedy row, every draft accepted + bonus
    assert acc[1] == 1 and nxt[1] == int(lg[1, 1].argmax())        # greedy row, rejected at position 1
    dist.barrier()
    if rank == 0:
        print("VOCAB_OK", world)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

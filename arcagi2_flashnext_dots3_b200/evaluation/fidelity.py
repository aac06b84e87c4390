"""Teacher-forced fidelity of a candidate model against a reference model (the reference's
dotsnote/training/eval/fidelity.py measures a served build's top-20 prompt log-probabilities against an FP8 base on
recorded traces, KL by context band).

Both models run in lockstep over the same token sequences, chunk by chunk through their engine step (paged caches,
the kernels that serve), and each chunk's statistics are reduced at once, so no [length, vocab] tensor is kept.
Per position: full-vocabulary KL(P_ref || P_cand), the top-K KL (reference's top-K tokens, both distributions
renormalized over them, the reference tool's measure), and whether the argmaxes agree; means per context band.
"""
from __future__ import annotations

import torch

BANDS = ((0, 4096), (4096, 16384), (16384, 1 << 30))


def _slot(llm):
    if not llm.free_slots:
        raise RuntimeError("no free sequence slot")
    return llm.free_slots.pop()


def fidelity(ref_llm, cand_llm, sequences, k: int = 20, chunk: int = 512, bands=BANDS) -> dict:
    """Statistics of cand against ref over the given token sequences (lists of ids). Returns {"bands": [{"lo",
    "hi", "n", "kl", "kl_topk", "agree"}], "n", "kl", "kl_topk", "agree"}."""
    nb = len(bands)
    acc = torch.zeros(nb, 4, dtype=torch.float64)   # n, kl, kl_topk, agree
    for ids in sequences:
        sa, sb = _slot(ref_llm), _slot(cand_llm)
        try:
            L = len(ids)
            for llm, s in ((ref_llm, sa), (cand_llm, sb)):
                llm.model.reset_slot(s)
                llm.model.assign_blocks(s, L, llm.alloc)
            dev_a, dev_b = ref_llm.device, cand_llm.device
            t_all = torch.tensor(ids, dtype=torch.int32)
            for p0 in range(0, L - 1, chunk):
                n = min(chunk, L - 1 - p0)   # the last token has no successor to score
                xa = ref_llm.model.step(t_all[p0:p0 + n].to(dev_a), torch.tensor([sa], dtype=torch.int32, device=dev_a),
                                        torch.tensor([p0], dtype=torch.int32, device=dev_a), n)
                xb = cand_llm.model.step(t_all[p0:p0 + n].to(dev_b), torch.tensor([sb], dtype=torch.int32,
                                                                                  device=dev_b),
                                         torch.tensor([p0], dtype=torch.int32, device=dev_b), n)
                la = torch.log_softmax(ref_llm.model.logits(xa).float(), -1)
                lb = torch.log_softmax(cand_llm.model.logits(xb).float().to(la.device), -1)
                kl = (la.exp() * (la - lb)).sum(-1)
                top = la.topk(k, -1).indices
                ta = torch.log_softmax(la.gather(1, top), -1)
                tb = torch.log_softmax(lb.gather(1, top), -1)
                klk = (ta.exp() * (ta - tb)).sum(-1)
                agree = (la.argmax(-1) == lb.argmax(-1)).double()
                pos = torch.arange(p0, p0 + n, device=la.device)
                for bi, (lo, hi) in enumerate(bands):
                    m = (pos >= lo) & (pos < hi)
                    if bool(m.any()):
                        acc[bi] += torch.stack([m.sum().double(), kl[m].double().sum(), klk[m].double().sum(),
                                                agree[m].sum()]).cpu()
        finally:
            for llm, s in ((ref_llm, sa), (cand_llm, sb)):
                llm.alloc.release(s)
                llm.model.reset_slot(s)
                llm.free_slots.append(s)
    rows = []
    for (lo, hi), a in zip(bands, acc):
        n = max(1.0, float(a[0]))
        rows.append({"lo": lo, "hi": hi, "n": int(a[0]), "kl": float(a[1]) / n, "kl_topk": float(a[2]) / n,
                     "agree": float(a[3]) / n})
    tot = acc.sum(0)
    n = max(1.0, float(tot[0]))
    return {"bands": rows, "n": int(tot[0]), "kl": float(tot[1]) / n, "kl_topk": float(tot[2]) / n,
            "agree": float(tot[3]) / n}

"""Speculative decoding: drafters propose k tokens per sequence, one main-model step verifies all k + 1 positions.

Step (greedy sequences; the reference's MTP-3 verify loop, fnext/mtp/fnmtp.py, with the recurrent-state
rollback of its RecoverSSM / lazy-fold patches, fnext/kv/0001-...recoverssm.patch and fnext/base/gdn_lazy.py):

1. tokens [pending, d_1 .. d_k] of every sequence run through the main model in one step (``verify=True``): the
   attention caches are written at their positions, recurrent states are not committed;
2. targets y_j = argmax of the logits at each position; accepted a = length of the prefix with d_j == y_j;
3. ``commit`` advances the recurrent states by a + 1 tokens and replays the PLE token history;
4. the sequence gains d_1 .. d_a and y_{a+1} (pending); output equals plain greedy decoding exactly.

Drafters:
* :class:`MTPDrafter` — the model's MTP head (:mod:`..models.fn_mtp`): run over the verified rows (filling its KV
  cache), then chained k - 1 single-token steps;
* :class:`NgramDrafter` — prompt lookup: the continuation of the most recent earlier occurrence of the last n
  tokens (n = max_n .. 1) in the sequence's own history (no model, host only);
* :class:`OracleDrafter` — replays known continuations (tests of the verify/commit path at full acceptance).
"""
from __future__ import annotations

import torch

from ..ops import fn_ops as ops
from .block_manager import BlockAllocator
from .llm import greedy_ids


class NgramDrafter:
    def __init__(self, max_n: int = 3):
        self.max_n = max_n

    def propose(self, llm, seqs, k):
        out = []
        for s in seqs:
            ctx = s.prompt + s.out
            d = []
            for n in range(min(self.max_n, len(ctx) - 1), 0, -1):
                key = ctx[-n:]
                for i in range(len(ctx) - n - 1, -1, -1):
                    if ctx[i:i + n] == key:
                        d = ctx[i + n:i + n + k]
                        break
                if d:
                    break
            out.append((d + [ctx[-1]] * k)[:k])
        return out

    def observe(self, llm, seqs, x, ids, accepted, k):
        pass


class OracleDrafter:
    def __init__(self, continuations: dict):
        self.cont = continuations  # tuple(prompt) -> full expected output list

    def propose(self, llm, seqs, k):
        out = []
        for s in seqs:
            full = self.cont[tuple(s.prompt)]
            n = len(s.out)
            out.append((full[n:n + k] + [0] * k)[:k])
        return out

    def observe(self, llm, seqs, x, ids, accepted, k):
        pass


class MTPDrafter:
    """Keeps, per slot, the MTP hidden state and next drafts produced after the last verify."""

    def __init__(self, head):
        self.head = head
        self.alloc = BlockAllocator(head.caches.n_blocks, head.caches.block_table.shape[0])
        self.next = {}

    def prefill(self, llm, seq, x_rows: torch.Tensor, k: int):
        """MTP over the prompt: position q reads (x_q, t_{q+1}); the last row uses the first sampled token."""
        dev = llm.device
        toks = seq.prompt[1:] + [seq.out[0]]
        self.head.reset_slot(seq.slot)
        self.alloc.release(seq.slot)
        self.head.assign_blocks(seq.slot, len(seq.prompt) + seq.max_new + k + 8, self.alloc)
        sl = torch.tensor([seq.slot], dtype=torch.int32, device=dev)
        xm = self.head.step(x_rows, torch.tensor(toks, dtype=torch.int32, device=dev), sl,
                            torch.tensor([0], dtype=torch.int32, device=dev), len(toks))
        self._chain(llm, [seq], xm[-1:], torch.tensor([len(toks) - 1], device=dev), k)

    def _chain(self, llm, seqs, xm, q_last, k):
        """From MTP hidden rows xm [B, H] at positions q_last: draft 1 = argmax, then k - 1 chained steps."""
        dev = llm.device
        sl = torch.tensor([s.slot for s in seqs], dtype=torch.int32, device=dev)
        d = self.head.draft_ids(xm)
        drafts = [d]
        for i in range(1, k):
            xm = self.head.step(xm, d, sl, (q_last + i).to(torch.int32), 1)
            d = self.head.draft_ids(xm)
            drafts.append(d)
        dd = torch.stack(drafts, 1).tolist()
        for s, row in zip(seqs, dd):
            self.next[s.slot] = row

    def propose(self, llm, seqs, k):
        return [self.next.get(s.slot, [s.out[-1]] * k)[:k] for s in seqs]

    def observe(self, llm, seqs, x, ids, accepted, k):
        """x [B*(k+1), H] verify hidden rows; ids [B, k+1] verify tokens; accepted [B] (host list)."""
        dev = llm.device
        B, k1 = len(seqs), k + 1
        toks = []
        for b, s in enumerate(seqs):
            a = accepted[b]
            row = ids[b][1:a + 1] + [s.out[-1]]          # next tokens of rows 0..a
            toks.append((row + [s.out[-1]] * k1)[:k1])
        sl = torch.tensor([s.slot for s in seqs], dtype=torch.int32, device=dev)
        pos0 = torch.tensor([s.pos - accepted[b] - 1 for b, s in enumerate(seqs)], dtype=torch.int32, device=dev)
        for s in seqs:
            self.head.assign_blocks(s.slot, s.pos + 2 * k1 + 8, self.alloc)
        xm = self.head.step(x, torch.tensor(toks, dtype=torch.int32, device=dev).view(-1), sl, pos0, k1)
        idx = torch.tensor([b * k1 + accepted[b] for b in range(B)], device=dev)
        self._chain(llm, seqs, xm[idx], pos0.long() + torch.tensor(accepted, device=dev), k)


class SpecGraph:
    """One speculative step for a fixed batch bucket, captured as a CUDA graph: verify the k + 1 tokens of every
    row, count accepted drafts on the device (leading matches of drafts and verify argmaxes), commit the recurrent
    states with those counts and, with an MTP head, run the head over the accepted rows and chain its next k
    drafts, all without a host round trip. The accepted rows' next tokens are exactly the verify argmaxes
    y[0..a], which is what the head reads. Padding rows use the engine's scratch slot."""

    def __init__(self, llm, head, batch: int, k: int):
        dev = llm.device
        self.llm, self.head, self.B, self.k = llm, head, batch, k
        k1 = k + 1
        self.ids = torch.zeros(batch, k1, dtype=torch.int32, device=dev)
        self.slots = torch.full((batch,), llm.scratch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.y = torch.zeros(batch, k1, dtype=torch.int32, device=dev)
        self.acc = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.nd = torch.zeros(batch, k, dtype=torch.int32, device=dev)
        self.graph = None

    def _body(self):
        m, B, k, k1 = self.llm.model, self.B, self.k, self.k + 1
        x = m.step(self.ids.view(-1), self.slots, self.pos, k1, verify=True)
        y = greedy_ids(m, x).view(B, k1)
        match = (self.ids[:, 1:] == y[:, :k]).to(torch.int32)
        acc = torch.cumprod(match, 1).sum(1).to(torch.int32)
        m.commit(acc + 1)
        self.y.copy_(y)
        self.acc.copy_(acc)
        if self.head is not None:
            h = self.head
            xm = h.step(x, y.reshape(-1), self.slots, self.pos, k1)
            rows = torch.arange(B, device=x.device) * k1 + acc.long()
            xa = xm[rows]
            q = self.pos + acc
            d = h.draft_ids(xa)
            drafts = [d]
            for i in range(1, k):
                xa = h.step(xa, d, self.slots, (q + i).to(torch.int32), 1)
                d = h.draft_ids(xa)
                drafts.append(d)
            self.nd.copy_(torch.stack(drafts, 1))

    def capture(self):
        """Warm up on the scratch slot only (a verify step commits recurrent state), then capture."""
        self.slots.fill_(self.llm.scratch)
        self.pos.zero_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        torch.cuda.synchronize()

    def run(self):
        self.graph.replay()


class SpecDecoder:
    def __init__(self, llm, drafter, k: int = 3, use_graph: bool = True):
        self.llm, self.drafter, self.k = llm, drafter, k
        self.stats = {"steps": 0, "drafted": 0, "accepted": 0, "emitted": 0}
        self.use_graph = use_graph and llm.device.type == "cuda" and llm.ec.cuda_graphs
        self.graphs = {}
        if self.use_graph and isinstance(drafter, MTPDrafter) and \
                drafter.head.caches.block_table.shape[0] <= llm.scratch:
            raise ValueError("the MTP head needs a cache slot for the engine's scratch slot (n_slots > max_seqs)")

    def add(self, prompt, max_new_tokens: int = 64, sp=None):
        llm = self.llm
        if isinstance(self.drafter, MTPDrafter):
            llm._keep_prefill_rows = True
        seq = llm.add(prompt, max_new_tokens, sp=sp)
        if isinstance(self.drafter, MTPDrafter):
            self.drafter.prefill(llm, seq, llm._prefill_rows, self.k)
            llm._keep_prefill_rows = False
        return seq

    def _graph_step(self, seqs, drafts):
        """Verify + commit (+ MTP chain) as one graph replay; returns (y rows, accepted counts) as host lists."""
        llm, k = self.llm, self.k
        k1 = k + 1
        n = len(seqs)
        bucket = next((b for b in llm.ec.graph_batch_sizes if b >= n), n)
        g = self.graphs.get(bucket)
        head = self.drafter.head if isinstance(self.drafter, MTPDrafter) else None
        if g is None:
            if head is not None:
                head.assign_blocks(llm.scratch, 2 * k1 + 8, self.drafter.alloc)
            llm.model.assign_blocks(llm.scratch, k1 + 1, llm.alloc)
            g = self.graphs[bucket] = SpecGraph(llm, head, bucket, k)
            g.capture()
        for s in seqs:
            llm.model.assign_blocks(s.slot, s.pos + k1 + 1, llm.alloc)
            if head is not None:
                head.assign_blocks(s.slot, s.pos + 2 * k1 + 8, self.drafter.alloc)
        pad = bucket - n
        ids = [[s.out[-1]] + list(d) for s, d in zip(seqs, drafts)] + [[0] * k1] * pad
        g.ids.copy_(torch.tensor(ids, dtype=torch.int32))
        g.slots.copy_(torch.tensor([s.slot for s in seqs] + [llm.scratch] * pad, dtype=torch.int32))
        g.pos.copy_(torch.tensor([s.pos for s in seqs] + [0] * pad, dtype=torch.int32))
        g.run()
        out = torch.cat([g.y, g.acc[:, None], g.nd], 1).cpu()
        y = out[:n, :k1].tolist()
        accepted = out[:n, k1].tolist()
        if head is not None:
            for s, row in zip(seqs, out[:n, k1 + 1:].tolist()):
                self.drafter.next[s.slot] = row
        return y, accepted

    def step(self) -> dict:
        llm, k = self.llm, self.k
        k1 = k + 1
        seqs = [s for s in llm.running.values() if not s.done]
        if not seqs:
            return {}
        sampled = any(s.sp.temperature > 0 for s in seqs)
        if any(s.sp.top_k or s.sp.top_p < 1.0 for s in seqs if s.sp.temperature > 0):
            raise ValueError("speculative sampling supports full-vocabulary temperature sampling (no top-k / top-p)")
        dev = llm.device
        drafts = self.drafter.propose(llm, seqs, k)
        if self.use_graph and not sampled:
            y, accepted = self._graph_step(seqs, drafts)
            return self._advance(seqs, drafts, y, accepted)
        ids = [[s.out[-1]] + list(d) for s, d in zip(seqs, drafts)]
        for s in seqs:
            llm.model.assign_blocks(s.slot, s.pos + k1 + 1, llm.alloc)
        sl = torch.tensor([s.slot for s in seqs], dtype=torch.int32, device=dev)
        pos = torch.tensor([s.pos for s in seqs], dtype=torch.int32, device=dev)
        x = llm.model.step(torch.tensor(ids, dtype=torch.int32, device=dev).view(-1), sl, pos, k1, verify=True)
        if sampled:
            accepted, nxt = self._sample_verify(seqs, x, drafts)
            y = [list(d[:a]) + [t] + [0] * (k1 - a - 1) for d, a, t in zip(drafts, accepted, nxt)]
        else:
            y = greedy_ids(llm.model, x).view(len(seqs), k1).tolist()
            accepted = []
            for d, yy in zip(drafts, y):
                a = 0
                while a < k and d[a] == yy[a]:
                    a += 1
                accepted.append(a)
        llm.model.commit(torch.tensor([a + 1 for a in accepted], dtype=torch.int32, device=dev))
        res = self._advance(seqs, drafts, y, accepted)
        self.drafter.observe(llm, seqs, x, ids, accepted, k)
        return res

    def _sample_verify(self, seqs, x, drafts):
        """Rejection-sampling verification (ops.sampling.speculative_accept; the sharded form when the LM head is
        split over a TP group). Emitted tokens follow the model's sampling distribution; greedy rows in the batch
        verify by argmax as before."""
        from ..ops import sampling
        m, k1 = self.llm.model, self.k + 1
        dr = torch.tensor([list(d) for d in drafts], dtype=torch.long).view(len(seqs), self.k)
        temps = [s.sp.temperature for s in seqs]
        seeds = [s.sp.seed for s in seqs]
        steps = [len(s.out) for s in seqs]        # index of the first token this verify emits
        if getattr(m, "vocab_sharded", False):
            from ..parallel.tp import sharded_speculative_accept
            lg = m._mm(x, m.W["lm_head"], f8=False).float().view(len(seqs), k1, -1)
            return sharded_speculative_accept(lg, m.W["vocab_range"][0], dr, temps, seeds, steps, m.tp.group)
        lg = m.logits(x).float().view(len(seqs), k1, -1)
        return sampling.speculative_accept(lg, dr, temps, seeds, steps)

    def _advance(self, seqs, drafts, y, accepted) -> dict:
        llm, k = self.llm, self.k
        res = {}
        for s, d, yy, a in zip(seqs, drafts, y, accepted):
            s.pos += a + 1
            new = list(d[:a]) + [yy[a]]
            for t in new:
                s.out.append(t)
                s.lps.append(0.0)
                res.setdefault(s.slot, []).append(t)
                if llm._finished(s):
                    break
            self.stats["emitted"] += len(res[s.slot])
        self.stats["steps"] += 1
        self.stats["drafted"] += k * len(seqs)
        self.stats["accepted"] += sum(accepted)
        return res

    def generate(self, prompts, max_new_tokens: int = 64, sp=None) -> list:
        seqs = [self.add(p, max_new_tokens, sp=sp) for p in prompts]
        while any(not s.done for s in seqs):
            self.step()
        outs = [s.out[: s.max_new] for s in seqs]
        for s in seqs:
            self.llm.release(s)
        return outs

    @property
    def acceptance(self) -> float:
        """Mean tokens emitted per sequence-step (1 + accepted drafts)."""
        n = self.stats["drafted"] / max(1, self.k)
        return self.stats["emitted"] / max(1, n)

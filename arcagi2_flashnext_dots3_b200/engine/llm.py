"""Public serving API: :class:`LLM` owns the model, the caches, the block allocator and the decode graphs.

Replaces the reference's external vLLM engine (scheduler, KV manager, CUDA graphs; the reference runs vLLM
0.30/0.32 with FULL_DECODE_ONLY graphs for batch sizes up to 128, flashnext/kaggle/code_dataset/kaggle_fn.sh:45).

* ``add(prompt)`` claims a slot, allocates paged-KV blocks and prefills in chunks.
* ``step()`` decodes one token for every running sequence: the input ids are copied host->device from pinned
  memory, one CUDA graph (captured per batch bucket) runs the whole model + LM head + sampler, and the new tokens
  (and their log-probabilities) come back device->host. Finished sequences (eos / stop ids / max tokens) stop.
  Sampling parameters are per sequence (:class:`..ops.sampling.SamplingParams`; default greedy).
* ``generate(prompts, max_new_tokens)`` = add + step until done.
* ``synthesize_context(lengths)`` fills slots with random cache state of the given lengths (used by the bench
  to measure decode at 6k-12k contexts without spending minutes on prefill).
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field

import torch

from ..config import EngineConfig
from ..ops import fn_ops as ops
from ..ops import native
from ..ops import sampling
from ..ops.sampling import SamplingParams
from .block_manager import BlockAllocator


def greedy_ids(model, x: torch.Tensor) -> torch.Tensor:
    """Greedy next token per row (int32). A model whose LM head is split over a TP group (``vocab_sharded``)
    picks through its own cross-rank pick, since its local logits are indexed by its vocabulary slice."""
    if getattr(model, "vocab_sharded", False):
        return model.pick(x)
    return ops.argmax(model.logits(x))


class ContextFull(ValueError):
    """A push would exceed max_model_len."""


@dataclass
class Sequence:
    slot: int
    prompt: list
    max_new: int
    out: list = field(default_factory=list)
    pos: int = 0          # tokens already in the cache
    done: bool = False
    t_first: float = 0.0
    t_last: float = 0.0
    sp: SamplingParams = field(default_factory=SamplingParams)
    lps: list = field(default_factory=list)   # log-probabilities of the generated tokens
    finish: str = ""                          # "stop" / "length" once done
    ctx_full: bool = False                    # stopped because the context reached max_model_len


class DecodeGraph:
    """Static-shape decode step for `batch` rows (one CUDA graph): ids/slots/positions in, next ids out.
    ``advance=True`` also feeds the next ids back and bumps positions inside the graph (device-only loops)."""

    def __init__(self, model, batch: int, advance: bool, use_graph: bool = True, scratch_slot: int = None,
                 sample: bool = False):
        dev = model.device
        self.scratch_slot = scratch_slot
        self.model = model
        self.batch = batch
        self.advance = advance
        self.sample = sample
        self.ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.slots = torch.arange(batch, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_lp = torch.zeros(batch, dtype=torch.float32, device=dev)
        # sampler inputs (temperature, top_k, top_p, seed, step); zeros = greedy
        self.sp = [torch.zeros(batch, dtype=dt, device=dev)
                   for dt in (torch.float32, torch.int32, torch.float32, torch.int64, torch.int64)]
        self.sp[2].fill_(1.0)
        self.graph = None
        self.use_graph = use_graph and model.device.type == "cuda"

    def _body(self):
        m = self.model
        x = m.step(self.ids, self.slots, self.positions)
        if self.sample:
            nxt, lp = sampling.sample(m.logits(x), *self.sp)
            self.next_lp.copy_(lp)
        else:
            nxt = greedy_ids(m, x)
        self.next_ids.copy_(nxt)
        if self.advance:
            self.ids.copy_(nxt)
            self.positions.add_(1)

    def capture(self):
        """Run the step once eagerly (warm-up, allocations), then capture it. The warm-up is a real decode step:
        callers capture before positions are meaningful or account for it."""
        if not self.use_graph:
            return
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        pos0, ids0, slots0 = self.positions.clone(), self.ids.clone(), self.slots.clone()
        if self.scratch_slot is not None:  # warm up on the scratch slot so no live sequence state changes
            self.slots.fill_(self.scratch_slot)
            self.positions.zero_()
        with torch.cuda.stream(s):
            self._body()
        torch.cuda.current_stream().wait_stream(s)
        self.positions.copy_(pos0)
        self.ids.copy_(ids0)
        self.slots.copy_(slots0)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        self.positions.copy_(pos0)
        self.ids.copy_(ids0)

    def run(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self._body()


class LLM:
    def __init__(self, cfg, weights: dict, device="cuda", engine: EngineConfig = None, model_cls=None, ep=None):
        from ..models.fn import FNModel, allocate_caches
        self.cfg = cfg
        self.ec = engine or EngineConfig()
        self.device = torch.device(device)
        ec = self.ec
        # one extra slot: padding rows of a graph bucket decode into it (never shared with a live sequence)
        self.scratch = ec.max_seqs
        alloc = getattr(model_cls, "allocate", None) or allocate_caches
        self.caches = alloc(cfg, self.device, ec.max_seqs + 1, ec.max_model_len, ec.block_size,
                            n_blocks=ec.kv_blocks or None, kv_dtype=ec.kv_dtype, state_dtype=ec.state_dtype)
        self.model = (model_cls or FNModel)(cfg, weights, self.caches, self.device, ep=ep)
        self.alloc = BlockAllocator(self.caches.n_blocks, ec.max_seqs + 1)
        self.model.assign_blocks(self.scratch, 1, self.alloc)
        self.free_slots = list(range(ec.max_seqs - 1, -1, -1))
        self.running: dict = {}
        self.graphs: dict = {}
        pin = self.device.type == "cuda"
        nh = max([ec.max_seqs] + list(ec.graph_batch_sizes))
        self.h_ids = torch.zeros(nh, dtype=torch.int32, pin_memory=pin)
        self.h_pos = torch.zeros(nh, dtype=torch.int32, pin_memory=pin)
        self.h_slots = torch.zeros(nh, dtype=torch.int32, pin_memory=pin)
        self.h_out = torch.zeros(nh, dtype=torch.int32, pin_memory=pin)
        self.h_lp = torch.zeros(nh, dtype=torch.float32, pin_memory=pin)
        self.h_sp = [torch.zeros(nh, dtype=dt, pin_memory=pin)
                     for dt in (torch.float32, torch.int32, torch.float32, torch.int64, torch.int64)]
        self.eos = getattr(cfg, "eos_token_id", -1)
        self.steplog = None
        if os.environ.get("FW_STEPLOG"):  # binary per-step records (utils/steplog.py)
            from ..utils.steplog import StepLog
            self.steplog = StepLog(os.environ["FW_STEPLOG"])
        self.stats = {"steps": 0, "tokens": 0, "prefill_tokens": 0}
        if os.environ.get("FW_FLAG_LOG"):   # record which optional paths this engine runs with
            import json
            from ..utils.observe import flag_report
            with open(os.environ["FW_FLAG_LOG"], "a") as f:
                f.write(json.dumps({"engine": type(self.model).__name__, "flags": flag_report()}) + "\n")

    # ---------------------------------------------------------------------------------- admission
    def add(self, prompt, max_new_tokens: int = 64, prefill_chunk: int = 2048, sp: SamplingParams = None) -> Sequence:
        if not self.free_slots:
            raise RuntimeError("no free sequence slot")
        slot = self.free_slots.pop()
        self.model.reset_slot(slot)
        seq = Sequence(slot, list(map(int, prompt)), max_new_tokens, sp=sp or SamplingParams())
        need = len(seq.prompt) + max_new_tokens
        if need > self.ec.max_model_len:
            self.free_slots.append(slot)
            raise ValueError(f"sequence needs {need} tokens > max_model_len {self.ec.max_model_len}")
        self.model.assign_blocks(slot, need, self.alloc)
        self._prefill(seq, prefill_chunk)
        self.running[slot] = seq
        return seq

    def _prefill(self, seq: Sequence, chunk: int):
        dev = self.device
        ids = torch.tensor(seq.prompt, dtype=torch.int32)
        last = None
        keep = getattr(self, "_keep_prefill_rows", False)   # speculative drafters read every prompt row
        rows = []
        for a in range(0, len(seq.prompt), chunk):
            b = min(len(seq.prompt), a + chunk)
            x = self.model.step(ids[a:b].to(dev), torch.tensor([seq.slot], dtype=torch.int32, device=dev),
                                torch.tensor([a], dtype=torch.int32, device=dev), n_tok=b - a)
            last = x[-1:]
            if keep:
                rows.append(x)
        self._prefill_rows = torch.cat(rows) if keep else None
        seq.pos = len(seq.prompt)
        self._append_sample(seq, last)
        self._finished(seq)
        seq.t_first = time.perf_counter()
        self.stats["prefill_tokens"] += len(seq.prompt)

    def extend(self, seq: Sequence, tokens: list, max_new_tokens: int = None):
        """Append tokens to a live sequence (multi-turn sessions: the cache is kept, only new tokens prefill).
        The previously sampled token that was never fed is dropped in favour of the pushed tokens."""
        if max_new_tokens is not None:
            seq.max_new = len(seq.out) + max_new_tokens
        if not tokens:
            raise ValueError("extend needs at least one token (push back the pending sampled token to continue)")
        if seq.pos + len(tokens) > self.ec.max_model_len - 1:
            raise ContextFull(f"{seq.pos} held + {len(tokens)} pushed > max_model_len {self.ec.max_model_len} - 1")
        seq.ctx_full = False
        need = seq.pos + len(tokens) + (seq.max_new - len(seq.out)) + 1
        self.model.assign_blocks(seq.slot, need, self.alloc)
        dev = self.device
        ids = torch.tensor(tokens, dtype=torch.int32, device=dev)
        x = self.model.step(ids, torch.tensor([seq.slot], dtype=torch.int32, device=dev),
                            torch.tensor([seq.pos], dtype=torch.int32, device=dev), n_tok=len(tokens))
        seq.prompt += list(tokens)
        seq.pos += len(tokens)
        seq.done = False
        seq.finish = ""
        self._append_sample(seq, x[-1:])
        self._finished(seq)
        self.running[seq.slot] = seq

    def _append_sample(self, seq: Sequence, x_last):
        """Sample the next token of `seq` from the hidden state of its last fed token."""
        if getattr(self.model, "vocab_sharded", False):
            if seq.sp.temperature > 0:
                raise NotImplementedError("sampling over a vocabulary-sharded LM head: only greedy picks are sharded")
            seq.out.append(int(greedy_ids(self.model, x_last)[0]))
            seq.lps.append(0.0)
            return
        ts = sampling.params_tensors([seq.sp], [len(seq.out)], self.device)
        ids, lp = sampling.sample(self.model.logits(x_last).float(), *[t.to(self.device) for t in ts])
        seq.out.append(int(ids[0]))
        seq.lps.append(float(lp[0]))

    def release(self, seq: Sequence):
        self.running.pop(seq.slot, None)
        self.alloc.release(seq.slot)
        self.free_slots.append(seq.slot)

    # -------------------------------------------------------------------------------------- decode
    def _graph_for(self, n: int) -> DecodeGraph:
        bucket = next((b for b in self.ec.graph_batch_sizes if b >= n), n)
        g = self.graphs.get(bucket)
        if g is None:
            # a vocabulary-sharded head has greedy picks only (temperature > 0 is refused at add time)
            g = DecodeGraph(self.model, bucket, advance=False, use_graph=self.ec.cuda_graphs,
                            scratch_slot=self.scratch, sample=not getattr(self.model, "vocab_sharded", False))
            g.capture()
            self.graphs[bucket] = g
        return g

    def step(self) -> dict:
        """One decode step for all running sequences. Returns {slot: new token}."""
        seqs = [s for s in self.running.values() if not s.done]
        if not seqs and self.model.ep is None:
            return {}
        # expert parallel: every rank steps in lockstep, a rank without sequences runs padding rows only
        n = len(seqs)
        g = self._graph_for(max(n, 1))
        B = g.batch
        hs = self.h_sp
        pad = B - n
        # vectorized fills of the pinned staging buffers (numpy views), one async copy per input vector
        self.h_ids.numpy()[:B] = [s.out[-1] for s in seqs] + [0] * pad
        self.h_pos.numpy()[:B] = [s.pos for s in seqs] + [0] * pad
        self.h_slots.numpy()[:B] = [s.slot for s in seqs] + [self.scratch] * pad
        hs[0].numpy()[:B] = [s.sp.temperature for s in seqs] + [0.0] * pad
        hs[1].numpy()[:B] = [s.sp.top_k for s in seqs] + [0] * pad
        hs[2].numpy()[:B] = [s.sp.top_p for s in seqs] + [1.0] * pad
        hs[3].numpy()[:B] = [s.sp.seed for s in seqs] + [0] * pad
        hs[4].numpy()[:B] = [len(s.out) for s in seqs] + [0] * pad
        g.ids.copy_(self.h_ids[:B], non_blocking=True)
        g.positions.copy_(self.h_pos[:B], non_blocking=True)
        g.slots.copy_(self.h_slots[:B], non_blocking=True)
        for dst, src in zip(g.sp, hs):
            dst.copy_(src[:B], non_blocking=True)
        g.run()
        self.h_out[:B].copy_(g.next_ids, non_blocking=True)
        self.h_lp[:B].copy_(g.next_lp, non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        now = time.perf_counter()
        res = {}
        toks = self.h_out[:n].tolist()
        lps = self.h_lp[:n].tolist()
        for s, t, lp in zip(seqs, toks, lps):
            s.pos += 1
            s.t_last = now
            s.out.append(t)
            s.lps.append(lp)
            res[s.slot] = t
            self._finished(s)
        self.stats["steps"] += 1
        self.stats["tokens"] += len(res)
        if self.steplog is not None:
            self.steplog.append(t_us=int(now * 1e6), batch=n, tokens=len(res), kv_blocks_free=self.alloc.n_free())
        return res

    def _finished(self, s: Sequence) -> bool:
        """Mark `s` done if its newest token ends it (eos / stop id) or it reached its token budget. The newest
        token is then left unfed (``pos`` counts fed tokens): a session continues by pushing it back first."""
        last = s.out[-1]
        if last == self.eos or last in s.sp.stop_token_ids:
            s.done, s.finish = True, "stop"
        elif len(s.out) >= s.max_new:
            s.done, s.finish = True, "length"
        elif s.pos + 1 >= self.ec.max_model_len - 1:
            s.done, s.finish, s.ctx_full = True, "length", True
        return s.done

    def generate(self, prompts, max_new_tokens: int = 64, sp: SamplingParams = None) -> list:
        seqs = [self.add(p, max_new_tokens, sp=sp) for p in prompts]
        while any(not s.done for s in seqs):
            self.step()
        outs = [s.out[: s.max_new] for s in seqs]
        for s in seqs:
            self.release(s)
        return outs

    # ------------------------------------------------------------------------------------ synthetic
    def synthesize_context(self, lengths, max_new_tokens: int, seed: int = 0) -> list:
        """Claim len(lengths) slots whose caches hold random state for contexts of the given lengths."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        c = self.caches
        if hasattr(self.model, "randomize_caches"):
            self.model.randomize_caches(g)
        else:
            self._randomize_fn_caches(g)
        seqs = []
        for L in lengths:
            slot = self.free_slots.pop()
            seq = Sequence(slot, [], max_new_tokens)
            self.model.assign_blocks(slot, int(L) + max_new_tokens + 2, self.alloc)
            seq.pos = int(L)
            seq.out.append(int(torch.randint(0, self.cfg.vocab_size, (1,), generator=g, device=self.device)))
            self.running[slot] = seq
            seqs.append(seq)
        if self.device.type == "cuda":
            torch.cuda.synchronize()
            native.check_error(self.device)
        return seqs

    def _randomize_fn_caches(self, g):
        c = self.caches
        for t in c.k + c.v:
            t.copy_(torch.randn(t.shape, generator=g, device=self.device).to(t.dtype))
        for t in c.comp:
            t.copy_(torch.randn(t.shape, generator=g, device=self.device).to(t.dtype))
        for t in c.kr_ring + c.conv:
            t.copy_(torch.randn(t.shape, generator=g, device=self.device))
        for t in c.ssm:
            t.copy_((torch.randn(t.shape, generator=g, device=self.device) * 0.05).to(t.dtype))

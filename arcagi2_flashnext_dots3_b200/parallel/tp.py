"""Tensor parallelism for the Dots3-shaped model: attention heads split over the ranks, row-parallel output
projection fused with an NVLink all-reduce, experts split over the ranks with every rank computing the partial MoE
sum of its experts for all tokens (no dispatch: tokens are replicated under TP), same all-reduce.

The reference runs D3 with TP4 and replaces NCCL's all-reduce by a host-staged quantized one
(dotsnote/engine/arcstats_pkg/arcstats/host_ar.py; routed in arcstats/__init__.py:383-410). Here
``comm="fused"``: the o-projection GEMM stores its fp32 partial directly into every rank's symmetric buffer
(wgemm fan-out epilogue), then csrc/k_tp.cu signals and reduces (bounded waits, deterministic rank order, the
residual add fused into the reduce); the MoE partial is pushed the same way. ``comm="q8"``: one kernel
(csrc/k_tp.cu ``tp_qar``) quantizes the partial to int8 per 128 elements, reduce-scatters it over peer memory,
re-quantizes each owner's sum and all-gathers it into the residual (2 (W-1)/W bytes per element per rank instead
of 4 (W-1)). ``comm="nccl"``: all_reduce.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist

from ..ops import native


def tp_config(cfg, world: int):
    """The per-rank view of a D3 config: head counts divided by the TP world."""
    if cfg.n_heads % world or cfg.swa_n_heads % world or cfg.n_experts % world:
        raise ValueError(f"heads/experts of {cfg.name} do not split over {world} ranks")
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // world, swa_n_heads=cfg.swa_n_heads // world)


class TPGroup:
    def __init__(self, rank: int, world: int, device, max_tokens: int, hidden: int, group=None, comm: str = "fused",
                 timeout_ns: int = None, q_bits: int = 8, hadamard: bool = False, error_feedback: bool = False,
                 sequence_parallel: bool = False):
        """``comm="q8"`` options: ``q_bits`` 8 or 4 (codes -7..7), ``hadamard`` (128-point Walsh-Hadamard rotation
        of every scale group before quantizing), ``error_feedback`` (within one forward pass each rank adds the
        quantization error it carried out of the previous all-reduce to its next input; :meth:`begin_forward`
        clears the carry). ``sequence_parallel``: the residual stream is split by tokens over the ranks; the
        row-parallel outputs are reduce-scattered into it and the normalized rows all-gathered before the next
        column-parallel GEMM (:meth:`reduce_scatter`, :meth:`all_gather`; the reference's TP groups with
        reduce-scatter / all-gather, flashnext/kaggle/code_dataset/fnext/base/host_dp.py:131-144)."""
        self.sp = sequence_parallel
        if comm == "q4":     # shorthand: 4-bit payload with rotation and error feedback
            comm, q_bits, hadamard, error_feedback = "q8", 4, True, True
        self.rank, self.world, self.comm = rank, world, comm
        self.q_bits, self.hadamard, self.error_feedback = q_bits, hadamard, error_feedback
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.H = hidden
        self.max_tokens = max_tokens
        self.slot = max_tokens * hidden
        self.timeout_ns = timeout_ns or native.DEFAULT_TIMEOUT_NS * 4
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        if comm == "fused":
            import torch.distributed._symmetric_memory as symm
            W = world

            def alloc(shape, dtype):
                t = symm.empty(*shape, dtype=dtype, device=self.device)
                t.zero_()
                h = symm.rendezvous(t, self.group)
                ptrs = [h.get_buffer(r, tuple(shape), dtype).data_ptr() for r in range(W)]
                return t, torch.tensor(ptrs, dtype=torch.int64, device=self.device)

            self.buf, self.buf_ptrs = alloc((2, W, self.slot), torch.float32)
            self.flags, self.flag_ptrs = alloc((2, W), torch.int64)
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        elif comm == "q8":
            if self.device.type == "cuda":
                import torch.distributed._symmetric_memory as symm
                sms = torch.cuda.get_device_properties(self.device).multi_processor_count
                groups = -(-self.slot // (world * 128))
                self.qar_grid = max(1, min(sms, groups))
                nbytes = native.C().tp_qar_bytes(self.slot, world, self.qar_grid)
                self.qbuf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
                self.qbuf.zero_()
                hd = symm.rendezvous(self.qbuf, self.group)
                self.qbases = torch.tensor([hd.get_buffer(r, (nbytes,), torch.uint8).data_ptr() for r in range(world)],
                                           dtype=torch.int64, device=self.device)
                torch.cuda.synchronize(self.device)
                dist.barrier(group=self.group)
            self.carry = torch.zeros(self.slot, dtype=torch.float32, device=self.device) if error_feedback else None
        elif comm != "nccl":
            raise ValueError(comm)

    # ------------------------------------------------------------------------------------ sequence parallel
    def sp_rows(self, T: int):
        """(padded token count, rows per rank) of a T-token residual split over the ranks."""
        Tl = -(-T // self.world)
        return Tl * self.world, Tl

    def reduce_scatter(self, partial: torch.Tensor) -> torch.Tensor:
        """This rank's token rows [Tl, H] of the sum over ranks of partial [T, H] (fp32; T padded to world * Tl)."""
        T, H = partial.shape
        Tp, Tl = self.sp_rows(T)
        x = partial.float()
        if Tp != T:
            x = torch.nn.functional.pad(x, (0, 0, 0, Tp - T))
        x = x.contiguous()
        out = torch.empty(Tl, H, dtype=torch.float32, device=x.device)
        if x.is_cuda:
            dist.reduce_scatter_tensor(out, x, group=self.group)
        else:   # gloo has no reduce-scatter
            dist.all_reduce(x, group=self.group)
            out.copy_(x[self.rank * Tl:(self.rank + 1) * Tl])
        return out

    def all_gather(self, x_loc: torch.Tensor, T: int) -> torch.Tensor:
        """The first T rows of every rank's [Tl, C] rows stacked in rank order."""
        x_loc = x_loc.contiguous()
        Tl = x_loc.shape[0]
        if x_loc.is_cuda:
            out = torch.empty(Tl * self.world, *x_loc.shape[1:], dtype=x_loc.dtype, device=x_loc.device)
            dist.all_gather_into_tensor(out, x_loc, group=self.group)
        else:
            parts = [torch.empty_like(x_loc) for _ in range(self.world)]
            dist.all_gather(parts, x_loc, group=self.group)
            out = torch.cat(parts)
        return out[:T]

    # ------------------------------------------------------------------------------------ fused GEMM path
    def begin(self):
        if self.comm in ("fused", "q8"):
            native.C().tp_epoch(self.epoch)

    def begin_forward(self):
        """Start of a forward pass: the error-feedback chain restarts (errors never cross forward passes)."""
        if getattr(self, "carry", None) is not None:
            self.carry.zero_()

    def fan(self):
        """wgemm fan-out arguments: write the GEMM output into slot [rank] of every rank's buffer."""
        return (self.buf_ptrs, self.rank, self.slot, self.epoch)

    def finish_into(self, h: torch.Tensor, T: int):
        """h[:T] += sum of all ranks' partials (after a fan-out GEMM or a push)."""
        n = T * self.H
        native.C().tp_signal(self.flag_ptrs, self.rank, self.epoch)
        native.C().tp_reduce(self.buf, self.flags, self.world, n, self.slot, self.epoch, h,
                             True, native.err_word(self.device), self.timeout_ns)

    # ------------------------------------------------------------------------------------ generic partial
    def allreduce_add(self, h: torch.Tensor, partial: torch.Tensor):
        """h += all-reduce(partial) for fp32 [T, H] tensors."""
        T = partial.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} rows > TP buffer capacity {self.max_tokens}")
        if self.comm == "q8":
            n = T * self.H
            if not partial.is_cuda:   # CPU ranks: the same quantized arithmetic through gathered partials
                x = partial.reshape(-1).float()
                if self.carry is not None:
                    x = x + self.carry[:n]
                parts = [torch.empty_like(x) for _ in range(self.world)]
                dist.all_gather(parts, x.contiguous(), group=self.group)
                out, carry = qar_reference(parts, self.q_bits, self.hadamard, rank=self.rank)
                if self.carry is not None:
                    self.carry[:n] = carry
                h += out.view_as(h)
                return
            self.begin()
            native.C().tp_qar(partial.contiguous(), h, n, self.qbases, self.rank, self.slot, self.qar_grid,
                              self.epoch, native.err_word(self.device), self.timeout_ns, self.q_bits, self.hadamard,
                              self.carry)
            return
        if self.comm == "nccl" or not partial.is_cuda:
            dist.all_reduce(partial, group=self.group)
            h += partial
            return
        self.begin()
        native.C().tp_push(partial.contiguous(), self.buf_ptrs, self.rank, self.slot, self.epoch)
        self.finish_into(h, T)

    def linear_allreduce_add(self, model, x16, ws, h):
        """h += all-reduce(x16 @ W_rank^T) with the GEMM epilogue writing into the peers (fused path)."""
        from ..ops import wgemm
        T = x16.shape[0]
        if self.comm in ("nccl", "q8") or not x16.is_cuda:
            self.allreduce_add(h, model._mm(x16, ws))
            return
        if T > self.max_tokens:
            raise ValueError(f"{T} rows > TP buffer capacity {self.max_tokens}")
        self.begin()
        dummy = torch.empty(T, ws.rows, dtype=torch.float32, device=x16.device)
        wgemm.matmul(x16, ws, out=dummy, fan=self.fan())
        self.finish_into(h, T)


def _quant(x: torch.Tensor, bits: int = 8):
    """Per 128-element group: (codes, scale) with scale = absmax / qmax (1 for an all-zero group), qmax 127 or 7,
    and codes = round-half-even(x * (1 / scale)) clamped to +-qmax; x is [groups, 128]."""
    qmax = 127.0 if bits == 8 else 7.0
    amax = x.abs().amax(-1, keepdim=True)
    s = torch.where(amax > 0, amax / qmax, torch.ones_like(amax))
    return torch.round(x * (1.0 / s)).clamp(-qmax, qmax), s


def hadamard128(device=None) -> torch.Tensor:
    """Orthonormal Sylvester Walsh-Hadamard matrix of order 128 (symmetric: its own inverse)."""
    h = torch.ones(1, 1)
    while h.shape[0] < 128:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / 128 ** 0.5).to(device)


def qar_reference(partials: list, bits: int = 8, had: bool = False, rank: int = None):
    """The quantized two-shot all-reduce of csrc/k_tp.cu in torch (same chunking, rounding and summation order):
    every rank's partial (optionally rotated by the 128-point Walsh-Hadamard transform) quantized per 128-element
    group, dequantized and summed in rank order per owner chunk, the sum quantized again, rotated back. Returns the
    fp32 sum every rank adds, or with ``rank`` given (sum, that rank's error-feedback carry: its quantization error
    everywhere plus, on its own chunk, the re-quantization error of the sum)."""
    W = len(partials)
    shape, n = partials[0].shape, partials[0].numel()
    chunk = ((n + W - 1) // W + 127) // 128 * 128
    pad = W * chunk - n
    Hm = hadamard128(partials[0].device) if had else None
    rot = (lambda v: v @ Hm) if had else (lambda v: v)
    xs = [rot(torch.nn.functional.pad(p.reshape(-1).float(), (0, pad)).view(-1, 128)) for p in partials]
    acc = torch.zeros_like(xs[0])
    errs = []
    for x in xs:                                  # rank order, as every owner sums its sources
        q, s = _quant(x, bits)
        acc = acc + q * s
        errs.append(x - q * s)
    q, s = _quant(acc, bits)
    out = rot(q * s).reshape(-1)[:n].view(shape)
    if rank is None:
        return out
    carry = rot(errs[rank]).reshape(-1)
    g0, g1 = rank * chunk // 128, (rank + 1) * chunk // 128
    carry.view(-1, 128)[g0:g1] += rot(acc - q * s)[g0:g1]
    return out, carry[:n]


def sharded_speculative_accept(local_logits: torch.Tensor, v0: int, drafts, temps, seeds, steps, group=None):
    """:func:`..ops.sampling.speculative_accept` with the LM head split over the TP group: every rank reduces
    its vocabulary slice to five numbers per (sequence, verify position): its max and exp-sum at the temperature,
    the draft's logit when it owns the draft, and its best Gumbel-max candidate (value, global index) excluding
    the draft. One all-gather of [world, B, k + 1, 5] replaces gathering the logits (the reference's
    shard_sample.py:67-119 likewise exchanges a few floats per row); every rank then decides the same accepted
    count and next token, equal to the unsharded result."""
    from ..ops.sampling import _decide, _row_candidates
    B, k1, _ = local_logits.shape
    mine = torch.stack([_row_candidates(local_logits[b], drafts[b], float(temps[b]), int(seeds[b]), int(steps[b]),
                                        v0) for b in range(B)])          # [B, k1, 5]
    world = dist.get_world_size(group)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine.contiguous(), group=group)
    allc = torch.stack(parts)                                           # [W, B, k1, 5], ranks in vocab order
    acc, nxt = [], []
    for b in range(B):
        a, t = _decide(allc[:, b].cpu(), drafts[b], float(temps[b]), int(seeds[b]), int(steps[b]), k1 - 1)
        acc.append(a)
        nxt.append(t)
    return acc, nxt


def vocab_range(V: int, rank: int, world: int):
    """[v0, v1) of the vocabulary whose LM-head rows this rank holds when the head is split over the TP group."""
    return rank * V // world, (rank + 1) * V // world


def sharded_pick(local_logits: torch.Tensor, v0: int, group=None, temperature: float = 0.0, seed: int = 0,
                 step: int = 0) -> torch.Tensor:
    """Next token per row when every TP rank holds the logits of its own vocabulary slice [v0, v0 + V_local).

    The reference samples on the vocab-parallel logits shard and all-gathers 8 floats per row instead of the
    logits (dotsnote/engine/arcstats_pkg/arcstats/shard_sample.py:3-14, 67, 119). Here each rank reduces its
    slice to one (value, global index) pair per row: the max logit for greedy decoding, or for temperature
    sampling the Gumbel-max key logit / T - log(-log u) with u drawn from the sampler's counter hash at the
    token's GLOBAL index (ops.sampling.uniform_torch). The pairs are all-gathered and the largest value wins,
    lowest index on ties. Because the noise of a token does not depend on which rank holds it, the result
    equals the token the unsharded CPU sampler (ops.sampling's torch path, top-k and top-p off) picks. The GPU
    sampler kernel evaluates the same noise with its own logf, which may differ from torch.log in the last bit,
    so a near-tie between two tokens can resolve differently there. Top-k / top-p sampling over a split head is
    :func:`sharded_sample`. Returns int32 [T]."""
    from ..ops import sampling
    x = local_logits.float()
    T, Vl = x.shape
    if temperature > 0:
        u = sampling.uniform_torch(seed, step, torch.arange(v0, v0 + Vl, device=x.device))
        x = x * (1.0 / temperature) - torch.log(-torch.log(u))[None, :]
    if Vl:
        idx = x.argmax(-1)   # first index among equal values
        val = x.gather(1, idx[:, None])[:, 0]
    else:
        val, idx = x.new_full((T,), -float("inf")), torch.zeros(T, dtype=torch.long, device=x.device)
    pair = torch.stack([val, (idx + v0).float()], 1).contiguous()          # indices < 2^24 are exact in fp32
    world = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        allp = torch.empty(world, T, 2, dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(allp, pair, group=group)
    else:
        parts = [torch.empty_like(pair) for _ in range(world)]
        dist.all_gather(parts, pair, group=group)
        allp = torch.stack(parts)
    best = allp[:, :, 0].argmax(0)   # ranks hold increasing vocabulary ranges: the first max has the lowest index
    return allp[best, torch.arange(T, device=pair.device), 1].to(torch.int32)


def sharded_sample(local_logits: torch.Tensor, v0: int, vocab: int, group=None, temperature: float = 1.0,
                   top_k: int = 0, top_p: float = 1.0, seed: int = 0, step: int = 0) -> torch.Tensor:
    """Top-k / top-p sampling when every TP rank holds the logits of its own vocabulary slice [v0, v0 + V_local)
    of a `vocab`-token head. The rule is the unsharded sampler's (ops.sampling._sample_row): the K = min(top_k or
    CAND, CAND, vocab) highest logits in (value desc, index asc) order, their fp32 cumulative exp((v - v_max) / T),
    the top-p cut relative to that mass, one uniform from the counter hash at index `vocab` scaled by the kept
    mass, the first candidate whose cumulative mass exceeds it. The global top K lies in the union of the ranks'
    local top K, so each rank sends K (value, global index) pairs per row (an all-gather of world x K x 2 floats)
    instead of the logits, and every rank draws the same token. On CPU ranks it returns the CPU sampler's token; on
    GPU ranks the cumulative sums run as a parallel scan whose last bit can differ, so a near-tie may resolve
    differently from the CPU. Greedy and full-vocabulary sampling (top_k 0, top_p 1) go to :func:`sharded_pick`.
    Returns int32 [T]."""
    from ..ops import sampling
    import numpy as np
    if temperature <= 0 or (top_k <= 0 and top_p >= 1.0):
        return sharded_pick(local_logits, v0, group, temperature, seed, step)
    x = local_logits.float()
    T, Vl = x.shape
    K = min(top_k if top_k > 0 else sampling.CAND, sampling.CAND, vocab)
    kl = min(K, Vl)
    vals = x.new_full((T, K), -float("inf"))
    idx = torch.full((T, K), vocab, dtype=torch.float32, device=x.device)    # padding sorts after real tokens
    if kl:
        # local top kl in (value desc, index asc): stable sort on the values of the index-ordered slice
        order = torch.sort(x, dim=-1, descending=True, stable=True).indices[:, :kl]
        vals[:, :kl] = x.gather(1, order)
        idx[:, :kl] = (order + v0).float()
    pair = torch.stack([vals, idx], -1).contiguous()                          # [T, K, 2]
    world = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        allp = torch.empty(world, T, K, 2, dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(allp, pair, group=group)
    else:
        parts = [torch.empty_like(pair) for _ in range(world)]
        dist.all_gather(parts, pair, group=group)
        allp = torch.stack(parts)
    cand = allp.permute(1, 0, 2, 3).reshape(T, world * K, 2)
    out = torch.empty(T, dtype=torch.int32)
    u = float(sampling.uniform(seed, step, [vocab])[0])
    for r in range(T):
        v, gi = cand[r, :, 0], cand[r, :, 1]
        o1 = torch.argsort(gi, stable=True)                                   # index asc, then value desc (stable)
        o2 = o1[torch.sort(v[o1], descending=True, stable=True).indices][:K]
        vs, ids = v[o2], gi[o2].long()
        if x.is_cuda:
            cum = torch.cumsum(torch.exp((vs - vs[0]) / temperature), 0)
            cut = K - 1 if top_p >= 1.0 else int(torch.nonzero(cum >= top_p * cum[-1])[0])
            lim = u * float(cum[cut])
            hit = torch.nonzero(cum[: cut + 1] > lim)
            out[r] = int(ids[int(hit[0]) if len(hit) else cut])
        else:
            vv = vs.numpy()
            cum = np.cumsum(np.exp((vv - vv[0]) / np.float32(temperature)).astype(np.float32), dtype=np.float32)
            cut = K - 1 if top_p >= 1.0 else int(np.argmax(cum >= np.float32(top_p) * cum[-1]))
            lim = sampling.uniform(seed, step, [vocab])[0] * cum[cut]
            hit = cum[: cut + 1] > lim
            out[r] = int(ids[int(np.argmax(hit)) if hit.any() else cut])
    return out.to(local_logits.device)


def shard_d3_weights(W: dict, cfg, rank: int, world: int, shard_vocab: bool = False) -> dict:
    """Dense-form D3 weights of one TP rank: the rank's attention heads (q_b, kv_b, g rows; o columns) and its
    contiguous share of every MoE layer's experts (router and correction bias stay whole: routing is global)."""
    import copy
    dn, dr, dv = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
    out = {k: v for k, v in W.items() if k != "layers"}
    if shard_vocab:   # this rank's rows of the LM head; next tokens through sharded_pick (D3Model.pick)
        v0, v1 = vocab_range(cfg.vocab_size, rank, world)
        out["lm_head"] = W["lm_head"][v0:v1]
        out["vocab_range"] = (v0, v1)
    out["layers"] = []
    for l, L in enumerate(W["layers"]):
        H = cfg.heads_of(l)
        h0, h1 = rank * H // world, (rank + 1) * H // world
        if getattr(cfg, "dense_fp8", False) and ((h1 - h0) * (dn + dr) % 128 or (h1 - h0) * dv % 128):
            # a shard boundary inside a 128x128 FP8 block would re-quantize the block with a different scale
            raise ValueError(f"layer {l}: {h1 - h0} heads per rank do not cover whole 128-wide FP8 blocks")
        a = dict(L["attn"])
        a["q_b"] = a["q_b"][h0 * (dn + dr):h1 * (dn + dr)]
        a["kv_b"] = a["kv_b"][h0 * (dn + dv):h1 * (dn + dv)]
        a["o"] = a["o"][:, h0 * dv:h1 * dv]
        a["g"] = a["g"][h0:h1]
        L2 = dict(L)
        L2["attn"] = a
        if "moe" in L:
            m = dict(L["moe"])
            lay = m["lowbit"]
            E = len(lay.blobs)
            e0, e1 = rank * E // world, (rank + 1) * E // world
            lay2 = copy.copy(lay)
            lay2.blobs = lay.blobs[e0:e1]
            lay2.experts = lay.experts[e0:e1]
            m["lowbit"] = lay2
            m["experts_dense"] = m["experts_dense"][e0:e1]
            m["expert_range"] = (e0, e1)
            L2["moe"] = m
        out["layers"].append(L2)
    return out

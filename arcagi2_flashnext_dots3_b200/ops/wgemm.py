"""Weight sets for the tcgen05 weight-dequant GEMM and its torch reference.

A :class:`WeightSet` holds one projection for E experts (E = 1 for a dense layer) in the runtime tile-block
layout (:mod:`..formats.runtime`): one uint8 buffer with every expert's blocks, per-expert byte offsets and
formats (2/3/4 = GPTQ codes, 8 = FP8 128x128 block-scaled, 16 = fp16). Experts of different bit widths share a
buffer, so a mixed 4/3-bit MoE layer is one launch (the reference needs one Marlin launch plus one Triton launch
on a side stream for that, flashnext/kaggle/code_dataset/fnext/moe/hyb_fuse.py:122-165).

``matmul`` / ``grouped`` dispatch on the device of the activations: CUDA tensors go to the kernel (the extension
is mandatory there), CPU tensors to a plain fp32 torch reference that dequantizes the same blocks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..formats import runtime as rt
from . import native

EPI_STORE, EPI_SILU_MUL = 0, 1


@dataclass
class WeightSet:
    blob: torch.Tensor          # uint8 [total bytes]
    exp_off: torch.Tensor       # int64 [E]
    exp_fmt: torch.Tensor       # int8 [E]
    rows: int                   # valid rows per expert (before padding to 128)
    K: int
    fmts: tuple                 # python copy of exp_fmt
    silu_pairs: bool = False    # rows are [gate; up] permuted for the silu*up epilogue
    _dense_cache: dict = None
    _f8: tuple = None           # (e4m3 row-major codes, block scales) for the kind::f8f6f4 dense GEMM

    @property
    def row_tiles(self) -> int:
        return (self.rows + 127) // 128

    @property
    def kg(self) -> int:
        return self.K // 128

    @property
    def n_experts(self) -> int:
        return len(self.fmts)

    @property
    def max_block_bytes(self) -> int:
        return max(rt.block_bytes(f) for f in set(self.fmts))

    def nbytes(self) -> int:
        return self.blob.numel()

    def to(self, device):
        return WeightSet(self.blob.to(device), self.exp_off.to(device), self.exp_fmt.to(device), self.rows,
                         self.K, self.fmts, self.silu_pairs)

    def f8_operands(self):
        """Row-major e4m3 codes [row_tiles*128, K] and fp32 scales [row_tiles, KG] of a dense FP8 set (cached)."""
        if self._f8 is None:
            n = self.row_tiles * self.kg * rt.block_bytes(8)
            blob = self.blob[:n].view(self.row_tiles, self.kg, rt.block_bytes(8))
            self._f8 = rt.fp8_rowmajor(blob, self.rows, self.K)
        return self._f8

    # ------------------------------------------------------------------ reference dequant
    def dense(self, e: int = 0) -> torch.Tensor:
        """fp32 [rows, K] weight of expert e in runtime row order (cached)."""
        if self._dense_cache is None:
            self._dense_cache = {}
        if e not in self._dense_cache:
            f = self.fmts[e]
            n = self.row_tiles * self.kg * rt.block_bytes(f)
            off = int(self.exp_off[e])
            blob = self.blob[off: off + n].view(self.row_tiles, self.kg, rt.block_bytes(f))
            self._dense_cache[e] = rt.unpack_blocks(blob, f, self.rows, self.K)
        return self._dense_cache[e]


def build_weight_set(blobs: list, fmts: list, rows: int, K: int, silu_pairs=False, device=None) -> WeightSet:
    """Concatenate per-expert runtime blocks ([tiles, KG, block_bytes] uint8) into one WeightSet."""
    offs, total = [], 0
    for b in blobs:
        offs.append(total)
        total += b.numel()
    dev = device or blobs[0].device
    blob = torch.empty(total, dtype=torch.uint8, device=dev)
    for o, b in zip(offs, blobs):
        blob[o: o + b.numel()] = b.reshape(-1).to(dev)
    return WeightSet(blob, torch.tensor(offs, dtype=torch.int64, device=dev),
                     torch.tensor(fmts, dtype=torch.int8, device=dev), rows, K, tuple(int(f) for f in fmts),
                     silu_pairs)


def dense_fp8(w: torch.Tensor, device=None) -> WeightSet:
    """FP8 block-scaled WeightSet from a dense weight [R, K] (quantized here)."""
    w8, sc = rt.quantize_fp8_blocks(w)
    return build_weight_set([rt.pack_fp8(w8, sc)], [8], w.shape[0], w.shape[1], device=device)


def dense_fp8_from_ckpt(w8: torch.Tensor, scale: torch.Tensor, device=None) -> WeightSet:
    return build_weight_set([rt.pack_fp8(w8, scale)], [8], w8.shape[0], w8.shape[1], device=device)


def dense_f16(w: torch.Tensor, device=None, silu_pairs=False) -> WeightSet:
    return build_weight_set([rt.pack_f16(w)], [16], w.shape[0], w.shape[1], silu_pairs=silu_pairs, device=device)


def pick_n_tile(max_tokens: int) -> int:
    for n in (16, 32, 64):
        if max_tokens <= n:
            return n
    return 128


SMALL_WEIGHT_BYTES = 8 << 20
_OLD_DENSE_PLAN = __import__("os").environ.get("FW_DENSE_PLAN") == "old"   # comparison switch
L2_REUSE_BYTES = 48 << 20   # weights up to this size are re-read from L2 when split over several token tiles
MIN_UNITS = 80              # work units (token tile x row tile x K split) that keep the SMs busy enough


def dense_n_tile(T: int, ws: WeightSet) -> int:
    return dense_plan(T, ws)[0]


def dense_plan(T: int, ws: WeightSet):
    """(token tile, K splits) of a dense GEMM. Parallelism comes first from token tiles (when the weight stays in
    L2 across them), then from K splits, since every split adds a partial sum that one CTA of the tile reduces at
    the end. The widest tile that reaches MIN_UNITS work units wins, then the fewest splits; measured on the FN
    decode shapes at 64 tokens (tile x split sweep, CUDA-graph timed): gdn_out 53 -> 30 us, attn_o 52 -> 27 us,
    router 21 -> 13 us, hc_down 24 -> 17 us."""
    widest = pick_n_tile(T)
    ns = [n for n in (128, 64, 32, 16) if n <= widest] if ws.nbytes() <= L2_REUSE_BYTES else [widest]
    for n in ns:
        for ks in (1, 2, 4, 8):
            if ks > ws.kg:
                break
            if (T + n - 1) // n * ws.row_tiles * ks >= MIN_UNITS:
                return n, ks
    return ns[-1], min(8, ws.kg)


F8_DENSE = __import__("os").environ.get("FW_DENSE_F8", "1") != "0"   # dense FP8 sets on kind::f8f6f4
F8_MAX_SPLITS = 8           # cluster size along K (portable limit)
F8_SMS = 148


_F8_CLUSTERS = {}


def f8_max_clusters(nt: int, s: int) -> int:
    """Co-resident clusters of `s` CTAs of the FP8 GEMM with token tile `nt` on this GPU (the driver's occupancy
    query, cached). Without a GPU: the B200 layout of 8 GPCs of about 18 SMs, one CTA per SM."""
    key = (nt, s)
    if key not in _F8_CLUSTERS:
        if torch.cuda.is_available():
            _F8_CLUSTERS[key] = int(native.C().f8_max_clusters(nt, s))
        else:
            _F8_CLUSTERS[key] = 8 * (18 // s)
    return _F8_CLUSTERS[key]


def f8_plan(T: int, ws: WeightSet):
    """(token tile, K splits) of the FP8 dense GEMM: the narrowest of 32/64/128 tokens that holds T (all of a
    decode batch in one tile, so the weights stream once), then the most K splits (a cluster of CTAs per row
    tile, reduced in distributed shared memory) for which every cluster of the grid is resident at once: at most
    one wave of the SMs, and no more clusters than the GPCs can hold (a cluster's CTAs share a GPC, so clusters of
    7 on 18-SM GPCs fit two per GPC and 20 of them would take two waves)."""
    nt = 32 if T <= 32 else 64 if T <= 64 else 128
    units = ws.row_tiles * ((T + nt - 1) // nt)
    best = 1
    for s in range(2, min(F8_MAX_SPLITS, ws.kg) + 1):
        if units * s <= F8_SMS and units <= f8_max_clusters(nt, s):
            best = s
    return nt, best


def f8_ok(ws: WeightSet, fan) -> bool:
    return F8_DENSE and fan is None and ws.fmts == (8,)


def f8_linear(x: torch.Tensor, ws: WeightSet, out: torch.Tensor, epi: int = EPI_STORE, accumulate=False,
              alpha=1.0, nt: int = 0, splits: int = 0) -> torch.Tensor:
    """Dense FP8 GEMM on tcgen05 `kind::f8f6f4` (csrc/k_f8gemm.cu): x [T, K] quantized per (token, 128-column
    group) to e4m3, weights read as their e4m3 codes. Two launches (quantize, GEMM)."""
    w8, sc = ws.f8_operands()
    if not nt or not splits:
        p_nt, p_s = f8_plan(x.shape[0], ws)
        nt, splits = nt or p_nt, splits or p_s
    native.C().f8_linear(x.contiguous(), w8, sc, ws.rows, out, epi, accumulate, alpha, nt, splits,
                         native.err_word(x.device), native.DEFAULT_TIMEOUT_NS)
    return out


def f8_reference(x: torch.Tensor, ws: WeightSet, epi: int = EPI_STORE) -> torch.Tensor:
    """fp32 emulation of :func:`f8_linear`: the same per-group e4m3 activation codes and scales, exact products,
    fp32 sums (differs from the kernel only in the order of the fp32 additions)."""
    T, K = x.shape
    xg = x.float().view(T, K // 128, 128)
    amax = xg.abs().amax(-1, keepdim=True)
    # a tensor / tensor division rounds once, as the kernel's 448.f / m does (torch evaluates 448.0 / amax as
    # reciprocal(amax) * 448, which rounds twice and now and then moves a code across an e4m3 rounding boundary)
    inv = torch.where(amax > 0, torch.full_like(amax, 448.0) / amax, torch.zeros_like(amax))
    x8 = (xg * inv).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    xq = (x8 * (amax / 448.0)).view(T, K)
    w = ws.dense(0) if not x.is_cuda else ws.dense(0).to(x.device)
    return _ref_apply(xq @ w.t(), epi)


def matmul(x16: torch.Tensor, ws: WeightSet, out: torch.Tensor = None, epi: int = EPI_STORE,
           out_dtype=torch.float32, accumulate=False, alpha=1.0, n_tile=None, k_splits: int = 0,
           fan=None, f8: bool = True) -> torch.Tensor:
    """Dense y = x @ W^T (or silu(gate)*up for a silu_pairs weight). x16: fp16 [T, K]. FP8 weight sets run on the
    kind::f8f6f4 GEMM with e4m3 activations unless ``f8`` is False (or a launch plan is given): then the weights
    are dequantized to fp16 for the kind::f16 GEMM and the activations keep fp16 (the LM heads use this, so
    argmax and sampling see unquantized activations)."""
    T = x16.shape[0]
    cols = ws.rows // 2 if epi == EPI_SILU_MUL else ws.rows
    if out is None:
        out = torch.zeros(T, cols, dtype=out_dtype, device=x16.device) if accumulate else \
            torch.empty(T, cols, dtype=out_dtype, device=x16.device)
    if not x16.is_cuda:
        y = _ref_apply(x16.float() @ ws.dense(0).t(), epi) * alpha
        if accumulate:
            out += y.to(out.dtype)
        else:
            out.copy_(y.to(out.dtype))
        return out
    if f8 and f8_ok(ws, fan) and n_tile is None and k_splits == 0:
        return f8_linear(x16, ws, out, epi, accumulate, alpha)
    if n_tile is None and k_splits == 0 and not _OLD_DENSE_PLAN:
        n_tile, k_splits = dense_plan(T, ws)
    n = n_tile or dense_n_tile(T, ws)
    f_ptrs, f_me, f_slot, f_epoch = fan if fan is not None else (None, 0, 0, None)
    native.C().wgemm(ws.blob, ws.exp_off, ws.exp_fmt, ws.row_tiles, ws.kg, None, None, 0, T, x16, 0, out, 0,
                     cols, epi, accumulate, alpha, n, ws.max_block_bytes, native.err_word(x16.device),
                     native.DEFAULT_TIMEOUT_NS, k_splits, None, f_ptrs, f_me, f_slot, f_epoch)
    return out


def grouped(xs16: torch.Tensor, ws: WeightSet, items: torch.Tensor, n_items: torch.Tensor, max_items: int,
            out: torch.Tensor, epi: int = EPI_STORE, n_tile: int = 16, row_dst: torch.Tensor = None) -> torch.Tensor:
    """Grouped (MoE) GEMM: for each item (expert e, token start t0, count n) computes rows t0..t0+n of out
    from rows t0..t0+n of xs16 with expert e's weights. With `row_dst` (int64 [rows] device addresses, fp32
    rows of out's width) every output row is stored at its own address instead (possibly on a peer GPU)."""
    cols = ws.rows // 2 if epi == EPI_SILU_MUL else ws.rows
    if not xs16.is_cuda:
        it = items[: int(n_items.reshape(-1)[0])].tolist()
        for e, t0, n, _ in it:
            y = _ref_apply(xs16[t0: t0 + n].float() @ ws.dense(e).t(), epi)
            out[t0: t0 + n] = y.to(out.dtype)
        return out
    native.C().wgemm(ws.blob, ws.exp_off, ws.exp_fmt, ws.row_tiles, ws.kg, items, n_items, max_items, -1, xs16, 0,
                     out, 0, cols, epi, False, 1.0, n_tile, ws.max_block_bytes, native.err_word(xs16.device),
                     native.DEFAULT_TIMEOUT_NS, 1, row_dst, None, 0, 0, None)
    return out


GEMV_MAX_TOK = 8  # items of at most this many tokens can run on the CUDA-core grouped GEMV (csrc/k_gemv.cu)


MOE_I8 = __import__("os").environ.get("FW_MOE_I8", "0") == "1"   # decode MoE on tcgen05 kind::i8 (csrc/k_moe_i8.cu)


def moe_decode_desc() -> str:
    """The decode MoE experts' compute path, as the benchmark reports it."""
    return ("4/3-bit codes x int8 activations (per 128-column group) on tcgen05 kind::i8, int32 accumulate per "
            "group, fp32 scale folds" if MOE_I8 else
            "4/3-bit codes x int8 activations (per 128-column group) on dp4a, fp32 accumulate")


def gemv_grouped(xs16: torch.Tensor, ws: WeightSet, items: torch.Tensor, n_items: torch.Tensor, max_items: int,
                 out: torch.Tensor, epi: int = EPI_STORE, row_dst: torch.Tensor = None, kernel: str = "auto"
                 ) -> torch.Tensor:
    """Same contract as :func:`grouped` for plans built with n_tile <= 8 (decode-sized expert groups): activations
    are quantized to int8 per 128-column group, then every item (expert, first row, count <= 8) is computed by
    integer dot products straight from the packed codes. ``kernel``: "dp4a" = the CUDA-core GEMV (csrc/k_gemv.cu),
    "i8" = tcgen05 kind::i8 MMA with the widened codes in tensor memory (csrc/k_moe_i8.cu), "auto" = the one
    FW_MOE_I8 selects; both give the same bits."""
    cols = ws.rows // 2 if epi == EPI_SILU_MUL else ws.rows
    if not xs16.is_cuda:
        return grouped(xs16, ws, items, n_items, max_items, out, epi=epi, row_dst=row_dst)
    if any(f > 4 for f in ws.fmts):
        raise ValueError("the grouped GEMV handles 2/3/4-bit experts only")
    use_i8 = kernel == "i8" or (kernel == "auto" and MOE_I8)
    R, K = xs16.shape
    Rq = max(R, 16) if use_i8 else R      # the MMA's 16-row activation box may reach past the last pair
    xq = torch.empty(Rq, K, dtype=torch.int8, device=xs16.device)
    xsc = torch.empty(Rq, K // 128, dtype=torch.float32, device=xs16.device)
    xsum = torch.empty(Rq, K // 128, dtype=torch.int32, device=xs16.device)
    native.C().gemv_quant(xs16, xq, xsc, xsum)
    fn = native.C().moe_i8 if use_i8 else native.C().gemv_grouped
    fn(ws.blob, ws.exp_off, ws.exp_fmt, ws.row_tiles, ws.kg, items, n_items, max_items, xq, xsc, xsum, out, cols,
       epi, row_dst, native.err_word(xs16.device), native.DEFAULT_TIMEOUT_NS)
    return out


def _ref_apply(y: torch.Tensor, epi: int) -> torch.Tensor:
    if epi == EPI_STORE:
        return y
    # runtime row order: tile t = [gate 64t..64t+63 | up 64t..64t+63]
    T, R = y.shape
    v = y.view(T, R // 128, 2, 64)
    g, u = v[:, :, 0], v[:, :, 1]
    return (torch.nn.functional.silu(g) * u).reshape(T, R // 2)

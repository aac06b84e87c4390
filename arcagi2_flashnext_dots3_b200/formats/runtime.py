"""Conversion of checkpoint weights into the GPU kernels' runtime "tile block" layout.

The checkpoint's planar layout (:mod:`.planar`) is optimized for the reference's Triton kernels. The tcgen05
weight-dequant GEMM (csrc/wgemm.cu) instead streams one contiguous block per (128-row tile, 128-column group)
with a 1-D TMA bulk copy, so the layout is converted once at load time (the reference does the same kind of
load-time conversion for its "pair" layout, dotsnote/engine/arcstats_pkg/arcstats/lowbit_moe.py:246 `_to_pairs`).

Block = ``words uint32 [NW][128 rows]`` + (integer formats) ``fp16 scale [128]`` + ``uint8 zero [128]`` or
(FP8) ``fp32 scale`` + 12 pad bytes. Word contents: see csrc/wgemm.h. All functions are plain torch and run on
CPU or GPU.
"""
from __future__ import annotations

import torch

G = 128
TILE = 128
FMT_WORDS = {4: 16, 3: 13, 2: 8, 8: 32, 16: 64}


def block_bytes(fmt: int) -> int:
    nw = FMT_WORDS[fmt]
    return nw * 512 + (384 if fmt <= 4 else 16 if fmt == 8 else 0)


def _pad_rows(t: torch.Tensor, rows: int) -> torch.Tensor:
    if t.shape[0] == rows:
        return t
    pad = torch.zeros((rows - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    return torch.cat([t, pad], 0)


def gate_up_perm(inter: int, device="cpu") -> torch.Tensor:
    """Row order putting gate rows 64t..64t+63 and the matching up rows in tile t (for the silu*up epilogue)."""
    if inter % 64:
        raise ValueError("intermediate size must be a multiple of 64")
    t = torch.arange(inter // 64, device=device)
    g = (t[:, None] * 64 + torch.arange(64, device=device)[None]).view(-1, 64)
    return torch.cat([g, g + inter], 1).reshape(-1)


def _words_q(q: torch.Tensor, bits: int) -> torch.Tensor:
    """codes int [R, KG, 128] -> uint32 words [R, KG, NW] (as int64 to avoid sign issues)."""
    R, KG, _ = q.shape
    q = q.to(torch.int64)
    pairs = q.view(R, KG, 64, 2)
    lo, hi = pairs[..., 0], pairs[..., 1]
    if bits == 4:
        lo = lo.view(R, KG, 16, 4)
        hi = hi.view(R, KG, 16, 4)
        sh = (4 * torch.arange(4, device=q.device)).view(1, 1, 1, 4)
    elif bits == 2:
        lo = lo.view(R, KG, 8, 8)
        hi = hi.view(R, KG, 8, 8)
        sh = (2 * torch.arange(8, device=q.device)).view(1, 1, 1, 8)
    else:
        z = torch.zeros(R, KG, 1, dtype=torch.int64, device=q.device)
        lo = torch.cat([lo, z], -1).view(R, KG, 13, 5)
        hi = torch.cat([hi, z], -1).view(R, KG, 13, 5)
        sh = (3 * torch.arange(5, device=q.device)).view(1, 1, 1, 5)
    w = ((lo << sh) | (hi << (sh + 16))).sum(-1)
    return w


def pack_q(q: torch.Tensor, s: torch.Tensor, z: torch.Tensor, bits: int) -> torch.Tensor:
    """codes [R, K] + fp16 scales [R, K/128] + uint8 zeros [R, K/128] -> uint8 blocks [tiles, KG, block_bytes]."""
    R, K = q.shape
    KG = K // G
    Rp = (R + TILE - 1) // TILE * TILE
    q = _pad_rows(q.to(torch.int32), Rp).view(Rp, KG, G)
    s = _pad_rows(s.to(torch.float16), Rp)
    z = _pad_rows(z.to(torch.uint8), Rp)
    T = Rp // TILE
    w = _words_q(q, bits)                                   # [Rp, KG, NW] int64 (uint32 values)
    NW = w.shape[-1]
    w = w.view(T, TILE, KG, NW).permute(0, 2, 3, 1)         # [T, KG, NW, 128]
    w32 = torch.where(w >= 2**31, w - 2**32, w).to(torch.int32).contiguous()
    words = w32.view(torch.uint8).reshape(T, KG, NW * 512)
    sb = s.view(T, TILE, KG).permute(0, 2, 1).contiguous().view(torch.uint8).reshape(T, KG, 256)
    zb = z.view(T, TILE, KG).permute(0, 2, 1).contiguous().reshape(T, KG, 128)
    return torch.cat([words, sb, zb], -1).contiguous()


def pack_planar_blob(planes: dict, s: torch.Tensor, z: torch.Tensor, bits: int, row_perm=None) -> torch.Tensor:
    """Planar checkpoint planes -> runtime blocks (optionally reordering rows first)."""
    from .planar import unpack_planar
    K = s.shape[1] * G
    q = unpack_planar(planes, bits, K)
    if row_perm is not None:
        q, s, z = q[row_perm], s[row_perm], z[row_perm]
    return pack_q(q, s, z, bits)


def quantize_fp8_blocks(w: torch.Tensor):
    """Dense weight [R, K] -> (e4m3 [R, K], fp32 scale [ceil(R/128), K/128]) with 128x128 block absmax scaling
    (the checkpoint's `weight_scale_inv` convention: w = w8 * scale)."""
    R, K = w.shape
    Rp = (R + TILE - 1) // TILE * TILE
    wp = _pad_rows(w.float(), Rp).view(Rp // TILE, TILE, K // G, G)
    amax = wp.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / 448.0
    w8 = (wp / scale[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return w8.view(Rp, K)[:R].contiguous(), scale.float()


def dequant_fp8_blocks(w8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    R, K = w8.shape
    s = scale.repeat_interleave(TILE, 0)[:R].repeat_interleave(G, 1)[:, :K]
    return w8.float() * s


def pack_fp8(w8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3 [R, K] + fp32 block scales [R/128, K/128] -> uint8 blocks [tiles, KG, 16400]."""
    R, K = w8.shape
    KG = K // G
    Rp = (R + TILE - 1) // TILE * TILE
    T = Rp // TILE
    b = _pad_rows(w8.view(torch.uint8), Rp).view(T, TILE, KG, 32, 4).permute(0, 2, 3, 1, 4)
    words = b.contiguous().reshape(T, KG, 32 * 512)
    sc = torch.zeros(T, KG, 4, dtype=torch.float32, device=w8.device)
    sc[..., 0] = scale[:T, :KG].float()
    return torch.cat([words, sc.view(torch.uint8).reshape(T, KG, 16)], -1).contiguous()


def fp8_rowmajor(blob: torch.Tensor, R: int, K: int):
    """FP8 tile blocks [tiles, KG, 16400] -> (e4m3 codes as uint8 [tiles*128, K] in row-major order, rows past R
    zero; fp32 block scales [tiles, KG]): the operand layout of the tcgen05 `kind::f8f6f4` dense GEMM, whose TMA
    loads read 128-column groups of 128 rows straight from it."""
    T, KG, _ = blob.shape
    codes = blob[..., : 32 * 512].reshape(T, KG, 32, TILE, 4).permute(0, 3, 1, 2, 4).reshape(T * TILE, KG * 128)
    scale = blob[..., 32 * 512: 32 * 512 + 4].contiguous().view(torch.float32).reshape(T, KG)
    return codes.contiguous(), scale.contiguous()


def pack_f16(w: torch.Tensor) -> torch.Tensor:
    """Dense fp16 [R, K] -> uint8 blocks [tiles, KG, 32768]."""
    R, K = w.shape
    KG = K // G
    Rp = (R + TILE - 1) // TILE * TILE
    T = Rp // TILE
    h = _pad_rows(w.to(torch.float16), Rp).view(torch.int16).view(T, TILE, KG, 64, 2).permute(0, 2, 3, 1, 4)
    return h.contiguous().view(torch.uint8).reshape(T, KG, 32768).contiguous()


def unpack_blocks(blob: torch.Tensor, fmt: int, R: int, K: int) -> torch.Tensor:
    """Inverse of the packers (for tests): fp32 dense weight [R, K] with scales applied."""
    T, KG, _ = blob.shape
    NW = FMT_WORDS[fmt]
    words = blob[..., : NW * 512].contiguous().view(torch.int32).view(T, KG, NW, TILE).to(torch.int64) & 0xFFFFFFFF
    words = words.permute(0, 3, 1, 2).reshape(T * TILE, KG, NW)
    if fmt == 16:
        v = words.to(torch.int32).contiguous().view(torch.float16).view(T * TILE, KG, 128)
        return v.reshape(T * TILE, K)[:R].float()
    if fmt == 8:
        b = blob[..., : 32 * 512].contiguous().view(T, KG, 32, TILE, 4).permute(0, 3, 1, 2, 4)
        v = b.reshape(T * TILE, KG, 128).contiguous().view(torch.float8_e4m3fn).float()
        sc = blob[..., 32 * 512: 32 * 512 + 4].contiguous().view(torch.float32).view(T, KG)
        v = v * sc.repeat_interleave(TILE, 0)[:, :, None]
        return v.reshape(T * TILE, K)[:R]
    ppw = {4: 4, 3: 5, 2: 8}[fmt]
    bits = fmt
    sh = (bits * torch.arange(ppw, device=words.device)).view(1, 1, 1, ppw)
    mask = (1 << bits) - 1
    lo = (words[..., None] >> sh) & mask
    hi = (words[..., None] >> (sh + 16)) & mask
    pairs = torch.stack([lo, hi], -1).reshape(T * TILE, KG, NW * ppw * 2)[..., :128]
    sb = blob[..., NW * 512: NW * 512 + 256].contiguous().view(torch.float16).view(T, KG, TILE)
    zb = blob[..., NW * 512 + 256: NW * 512 + 384].contiguous().view(T, KG, TILE)
    s = sb.permute(0, 2, 1).reshape(T * TILE, KG).float()
    z = zb.permute(0, 2, 1).reshape(T * TILE, KG).float()
    w = (pairs.float() - z[..., None]) * s[..., None]
    return w.reshape(T * TILE, K)[:R]


def tensor_core_operands(blob: torch.Tensor, fmt: int, R: int, K: int) -> torch.Tensor:
    """fp16 [R, K]: the weight values exactly as the GEMM's dequant stage writes them into shared memory for the
    tensor core. FP8 blocks: fp16(e4m3) times the block scale rounded to fp16, one fp16 rounding of the product;
    integer formats: (q - z), exact in fp16, times the fp16 group scale, one rounding; fp16 blocks: unchanged.
    Rows gathered from this tensor into an fp16 weight set give the same products as the source blocks, whatever
    block scale their source tile had."""
    if fmt == 16:
        return unpack_blocks(blob, fmt, R, K).half()
    T, KG, _ = blob.shape
    if fmt == 8:
        b = blob[..., : 32 * 512].contiguous().view(T, KG, 32, TILE, 4).permute(0, 3, 1, 2, 4)
        v = b.reshape(T * TILE, KG, 128).contiguous().view(torch.float8_e4m3fn).half()
        sc = blob[..., 32 * 512: 32 * 512 + 4].contiguous().view(torch.float32).view(T, KG).half()
        out = v * sc.repeat_interleave(TILE, 0)[:, :, None]
        return out.reshape(T * TILE, K)[:R].contiguous()
    NW = FMT_WORDS[fmt]
    qz = unpack_qz(blob, fmt, R, K).half()
    sb = blob[..., NW * 512: NW * 512 + 256].contiguous().view(torch.float16).view(T, KG, TILE)
    s = sb.permute(0, 2, 1).reshape(T * TILE, KG)[:R]
    return (qz.view(R, KG, 128) * s[:, :, None]).reshape(R, K).contiguous()


def unpack_qz(blob: torch.Tensor, fmt: int, R: int, K: int) -> torch.Tensor:
    """(q - z) as fp32 [R, K] of an integer-format expert's blocks [tiles, KG, bytes] (scales not applied)."""
    T, KG, _ = blob.shape
    NW = FMT_WORDS[fmt]
    words = blob[..., : NW * 512].contiguous().view(torch.int32).view(T, KG, NW, TILE).to(torch.int64) & 0xFFFFFFFF
    words = words.permute(0, 3, 1, 2).reshape(T * TILE, KG, NW)
    ppw = {4: 4, 3: 5, 2: 8}[fmt]
    sh = (fmt * torch.arange(ppw, device=words.device)).view(1, 1, 1, ppw)
    mask = (1 << fmt) - 1
    lo = (words[..., None] >> sh) & mask
    hi = (words[..., None] >> (sh + 16)) & mask
    q = torch.stack([lo, hi], -1).reshape(T * TILE, KG, NW * ppw * 2)[..., :128]
    zb = blob[..., NW * 512 + 256: NW * 512 + 384].contiguous().view(T, KG, TILE)
    z = zb.permute(0, 2, 1).reshape(T * TILE, KG).float()
    return (q.float() - z[..., None]).reshape(T * TILE, K)[:R]


def block_scales(blob: torch.Tensor, fmt: int, R: int) -> torch.Tensor:
    """fp32 [R, KG] scales stored in an integer-format expert's blocks."""
    T, KG, _ = blob.shape
    NW = FMT_WORDS[fmt]
    sb = blob[..., NW * 512: NW * 512 + 256].contiguous().view(torch.float16).view(T, KG, TILE)
    return sb.permute(0, 2, 1).reshape(T * TILE, KG)[:R].float()

"""Planar low-bit expert weight layout (checkpoint format L0) and its torch reference dequantizer.

The on-disk layout is the reference's, kept bit-compatible so its `lowbit-LNN.pt` files load unchanged
(format described in dotsnote/engine/arcstats_pkg/arcstats/lowbit_moe.py:1-30 and produced by
flashnext/kaggle/code_dataset/fnext/moe/lowbit_kernels.py:225 `_pack_planar`; read back by
flashnext/training/student/student_fn.py:88 `_qz`). For a projection W [R, K] (y = x @ W^T) every row stores,
per group of G = 128 input columns:

* 4-bit: ``p4`` = 32 int16 words; 4-bit field j (j < 4) of word w is column 32*j + w.
* 2/3-bit: ``p2`` = 16 int16 words; 2-bit field j (j < 8) of word w is column 16*j + w.
* 3-bit only: ``p1`` = 16 uint8 bytes; bit j of byte w is bit 2 of column 16*j + w.
* ``s`` fp16 [R, K/G] scales, ``z`` uint8 [R, K/G] zero points; w = s * (q - z).

Everything here is plain torch and runs on CPU or GPU. The GPU kernels use a different runtime layout
(:mod:`.runtime`), converted once at load time.
"""
from __future__ import annotations

import torch

G = 128


def _to_i16(w: torch.Tensor) -> torch.Tensor:
    w = w.to(torch.int32)
    return torch.where(w >= 32768, w - 65536, w).to(torch.int16)


def pack_planar(q: torch.Tensor, bits: int) -> dict:
    """Pack integer codes q [R, K] (values in [0, 2**bits)) into the planar layout.

    Returns ``{"p4": int16 [R, K/4]}`` for 4-bit, ``{"p2": int16 [R, K/8]}`` for 2-bit and additionally
    ``"p1": uint8 [R, K/8]`` for 3-bit.
    """
    if bits not in (2, 3, 4):
        raise ValueError(f"bits must be 2, 3 or 4, got {bits}")
    R, K = q.shape
    if K % G:
        raise ValueError(f"K={K} is not a multiple of the group size {G}")
    q = q.to(torch.int32)
    if bits == 4:
        f = q.view(R, K // G, 4, 32)
        w = torch.zeros(R, K // G, 32, dtype=torch.int32, device=q.device)
        for j in range(4):
            w |= (f[:, :, j, :] & 15) << (4 * j)
        return {"p4": _to_i16(w).view(R, K // 4)}
    f = q.view(R, K // G, 8, 16)
    w = torch.zeros(R, K // G, 16, dtype=torch.int32, device=q.device)
    for j in range(8):
        w |= (f[:, :, j, :] & 3) << (2 * j)
    out = {"p2": _to_i16(w).view(R, K // 8)}
    if bits == 3:
        h = torch.zeros(R, K // G, 16, dtype=torch.int32, device=q.device)
        for j in range(8):
            h |= ((f[:, :, j, :] >> 2) & 1) << j
        out["p1"] = h.to(torch.uint8).view(R, K // 8)
    return out


def unpack_planar(planes: dict, bits: int, K: int) -> torch.Tensor:
    """Inverse of :func:`pack_planar`: integer codes int32 [R, K]."""
    KG = K // G
    if bits == 4:
        p4 = planes["p4"]
        R = p4.shape[0]
        w = p4.reshape(R, KG, 1, 32).to(torch.int32) & 0xFFFF
        j = torch.arange(4, device=p4.device, dtype=torch.int32).view(1, 1, 4, 1)
        return ((w >> (4 * j)) & 15).reshape(R, K)
    p2 = planes["p2"]
    R = p2.shape[0]
    w = p2.reshape(R, KG, 1, 16).to(torch.int32) & 0xFFFF
    j = torch.arange(8, device=p2.device, dtype=torch.int32).view(1, 1, 8, 1)
    q = (w >> (2 * j)) & 3
    if bits == 3:
        h = planes["p1"].reshape(R, KG, 1, 16).to(torch.int32) & 0xFF
        q = q | (((h >> j) & 1) << 2)
    return q.reshape(R, K)


def dequant(planes: dict, bits: int, s: torch.Tensor, z: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """Dense weight [R, K] = s * (q - z), computed in fp32 then cast (the reference's `deq`)."""
    R, KG = s.shape
    q = unpack_planar(planes, bits, KG * G).view(R, KG, G).float()
    w = (q - z.float()[..., None]) * s.float()[..., None]
    return w.reshape(R, KG * G).to(dtype)


def quantize_rtn(w: torch.Tensor, bits: int, symmetric: bool = False, clip_search: int = 0):
    """Round-to-nearest group quantization of w [R, K] into (codes, s fp16, z uint8).

    ``symmetric`` fixes z = 2**(bits-1) and s = absmax / (2**(bits-1) - 0.5)-style grid; asymmetric picks
    [min, max] per group. ``clip_search`` > 0 tries that many shrink ratios of the range per group and keeps the
    one with the lowest squared error (the MSE clip search used by the reference's GPTQ builder,
    flashnext/training/prune_gptq/gptq_fn.py:152).
    """
    R, K = w.shape
    KG = K // G
    wf = w.float().view(R, KG, G)
    qmax = (1 << bits) - 1

    def grid(ratio):
        if symmetric:
            amax = wf.abs().amax(-1) * ratio
            s = (amax / (qmax / 2.0)).clamp_min(1e-8)
            z = torch.full_like(s, float(1 << (bits - 1)))
        else:
            lo = (wf.amin(-1) * ratio).clamp_max(0)
            hi = (wf.amax(-1) * ratio).clamp_min(0)
            s = ((hi - lo) / qmax).clamp_min(1e-8)
            z = torch.round(-lo / s).clamp(0, qmax)
        s = s.half().float()
        return s, z

    def codes(s, z):
        return torch.clamp(torch.round(wf / s[..., None]) + z[..., None], 0, qmax)

    s, z = grid(1.0)
    q = codes(s, z)
    if clip_search:
        err = ((q - z[..., None]) * s[..., None] - wf).pow(2).sum(-1)
        for i in range(1, clip_search):
            r = 1.0 - 0.05 * i
            s2, z2 = grid(r)
            q2 = codes(s2, z2)
            e2 = ((q2 - z2[..., None]) * s2[..., None] - wf).pow(2).sum(-1)
            better = e2 < err
            s = torch.where(better, s2, s)
            z = torch.where(better, z2, z)
            q = torch.where(better[..., None], q2, q)
            err = torch.where(better, e2, err)
    return q.view(R, K).to(torch.int32), s.half(), z.to(torch.uint8)


def bytes_per_row(bits: int, K: int) -> int:
    """Bytes one packed row occupies including its fp16 scales and uint8 zeros."""
    KG = K // G
    body = {4: 64, 3: 48, 2: 32}[bits] * KG
    return body + 3 * KG

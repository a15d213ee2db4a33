"""Packed operand rows: the HBM layout the emulator kernels read.

A row holds the K elements of one dot-product operand as a little-endian bit
string, element k at bits [k*bits, (k+1)*bits): 32 bits for TF32 (the whole
F32 container), 16 for BF16 (the high half of its F32 container) and F16, 8
for E4M3/E5M2/U8/S8, 6 for E2M3/E3M2 and 4 for E2M1.  Only bits the
reference model reads are dropped (it masks every word the same way), so
packing is lossless for the arithmetic.  Rows are padded to a multiple of 4
bytes (16 when ``align16``) and stored back to back.
"""

from __future__ import annotations

import numpy as np

from . import _native as nat


def row_bytes(fmt: int, k: int) -> int:
    return (k * nat.FORMAT_BITS[fmt] + 7) // 8


def row_stride(fmt: int, k: int, align16: bool = False) -> int:
    a = 16 if align16 else 4
    return (row_bytes(fmt, k) + a - 1) // a * a


def _element_values(words: np.ndarray, fmt: int) -> np.ndarray:
    w = np.asarray(words, dtype=np.uint32)
    if fmt == nat.FMT_BF16:
        return w >> np.uint32(16)
    bits = nat.FORMAT_BITS[fmt]
    if bits == 32:
        return w
    return w & np.uint32((1 << bits) - 1)


def pack_rows(words, fmt: int, stride: int | None = None) -> np.ndarray:
    """[R, K] raw container words -> [R, stride] uint8 packed rows (host)."""
    w = np.asarray(words)
    if w.ndim != 2:
        raise ValueError("pack_rows expects a [rows, K] array of words")
    rows, k = w.shape
    stride = row_stride(fmt, k) if stride is None else stride
    if stride < row_bytes(fmt, k) or stride % 4:
        raise ValueError("row stride too small or not a multiple of 4 bytes")
    v = _element_values(w, fmt)
    bits = nat.FORMAT_BITS[fmt]
    if bits == 32:
        body = v.astype("<u4").view(np.uint8).reshape(rows, 4 * k)
    elif bits == 16:
        body = v.astype("<u2").view(np.uint8).reshape(rows, 2 * k)
    elif bits == 8:
        body = v.astype(np.uint8)
    elif bits == 6:
        k4 = (k + 3) // 4 * 4
        x = np.zeros((rows, k4), dtype=np.uint32)
        x[:, :k] = v
        x = x.reshape(rows, k4 // 4, 4)
        g = x[:, :, 0] | (x[:, :, 1] << 6) | (x[:, :, 2] << 12) | (x[:, :, 3] << 18)
        body = np.stack([g & 0xFF, (g >> 8) & 0xFF, (g >> 16) & 0xFF], axis=2).astype(np.uint8)
        body = body.reshape(rows, k4 // 4 * 3)[:, : row_bytes(fmt, k)]
    else:  # 4 bits
        k2 = (k + 1) // 2 * 2
        x = np.zeros((rows, k2), dtype=np.uint8)
        x[:, :k] = v
        body = (x[:, 0::2] | (x[:, 1::2] << 4)).astype(np.uint8)
    out = np.zeros((rows, stride), dtype=np.uint8)
    out[:, : body.shape[1]] = body
    return out


def unpack_rows(packed, fmt: int, k: int) -> np.ndarray:
    """Inverse of pack_rows for the bits the model reads: [R, stride] -> [R, K]
    uint32 container words (BF16 back in the high half)."""
    p = np.asarray(packed, dtype=np.uint8)
    rows = p.shape[0]
    bits = nat.FORMAT_BITS[fmt]
    if bits == 32:
        v = np.ascontiguousarray(p[:, : 4 * k]).view("<u4").astype(np.uint32)
    elif bits == 16:
        v = np.ascontiguousarray(p[:, : 2 * k]).view("<u2").astype(np.uint32)
    elif bits == 8:
        v = p[:, :k].astype(np.uint32)
    elif bits == 6:
        k4 = (k + 3) // 4 * 4
        nb = k4 // 4 * 3
        b = np.zeros((rows, nb), dtype=np.uint32)
        take = min(nb, p.shape[1])
        b[:, :take] = p[:, :take]
        b = b.reshape(rows, k4 // 4, 3)
        g = b[:, :, 0] | (b[:, :, 1] << 8) | (b[:, :, 2] << 16)
        v = np.stack([g & 0x3F, (g >> 6) & 0x3F, (g >> 12) & 0x3F, (g >> 18) & 0x3F], axis=2)
        v = v.reshape(rows, k4)[:, :k].astype(np.uint32)
    else:
        nb = (k + 1) // 2
        b = p[:, :nb].astype(np.uint32)
        v = np.stack([b & 0xF, b >> 4], axis=2).reshape(rows, 2 * nb)[:, :k]
    if fmt == nat.FMT_BF16:
        v = v << np.uint32(16)
    return v.astype(np.uint32)


def pack_rows_device(words, fmt: int, stride: int | None = None, stream=None):
    """[R, K] uint32 words already on the GPU (a torch tensor) -> packed rows on
    the same device, using the library's packing kernel."""
    import torch

    from .runtime import current_stream_handle

    if words.dim() != 2:
        raise ValueError("pack_rows_device expects a [rows, K] tensor of words")
    w = words.contiguous()
    if w.dtype != torch.int32 and w.dtype != torch.uint32:
        w = w.to(torch.int64).bitwise_and(0xFFFFFFFF).to(torch.uint32) if w.dtype != torch.uint32 else w
    rows, k = w.shape
    stride = row_stride(fmt, k) if stride is None else stride
    out = torch.empty((rows, stride), dtype=torch.uint8, device=w.device)
    rc = nat.load().t5e_pack_rows(fmt, w.data_ptr(), rows, k, out.data_ptr(), stride,
                                  current_stream_handle(w.device) if stream is None else stream)
    nat.check(rc, "t5e_pack_rows")
    return out

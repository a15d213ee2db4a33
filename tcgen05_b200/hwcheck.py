"""Cross-check of the emulator against the B200's own tensor cores.

``hardware_tiles`` runs real ``tcgen05.mma`` instructions (kind::tf32,
kind::f16, kind::f8f6f4 with any pair of E4M3/E5M2/E2M3/E3M2/E2M1 operands,
kind::i8) on tiles D = A B + C of M = 128, N = 16 and one instruction's K,
with F32, F16 or S32 accumulators, through ``t5e_tcgen05_tiles``;
``cross_check`` evaluates the same tiles with the emulator (``mma_batch``)
and counts the words on which the two differ.  This is the comparison the
reference's hardware harness makes between its probe runners and its model
(hardware_validation/mma_probe.py), here between the hardware and this
library.  Every word agrees, except that on the F16 x F16 -> F16 path the
reference (and so the emulator) reports NaN and infinities with F32 words
where the B200 writes F16 words; that pairing is counted separately.

``cross_check_block_scaled`` does the same for the block-scaled kinds, and
``cross_check_sparse`` for the sparse ones (tcgen05.mma.sp): the cases of a
sparse validation path, one uniform tile per case.

    python -m tcgen05_b200.hwcheck [--tiles 64] [--seed 0]
"""

from __future__ import annotations

import argparse
import ctypes
import itertools
import json

import numpy as np

from . import _native as nat
from . import packing, runtime

M, N = 128, 16

# instruction kinds and descriptor format codes (the tcgen05 instruction
# descriptor: bits 4-5 accumulator format, 7-9 A format, 10-12 B format,
# 17-22 N/8, 24-28 M/16, bit 3 saturation)
KINDS = {"tf32": 0, "bf16": 1, "f16": 1, "e4m3": 2, "e5m2": 2, "e2m3": 2, "e3m2": 2, "e2m1": 2, "u8": 3, "s8": 3}
FORMAT_CODES = {"tf32": 2, "bf16": 1, "f16": 0, "e4m3": 0, "e5m2": 1, "e2m3": 3, "e3m2": 4, "e2m1": 5, "u8": 0, "s8": 1}
K_OF_KIND = {0: 8, 1: 16, 2: 32, 3: 32}
C_FORMATS = {"f16": 0, "f32": 1, "s32": 2}
SUB_BYTE = ("e2m3", "e3m2", "e2m1")

# Set once a launch reports an expired wait.  The kernel then frees its tensor
# memory while the tcgen05.mma it committed may still be writing there, so a
# later launch in this process could read columns that product overwrites:
# every result after a timeout is untrusted, and no further hardware tiles
# are launched in the process.
_WAIT_EXPIRED = False


def _refuse_after_timeout() -> None:
    if _WAIT_EXPIRED:
        raise RuntimeError("an earlier tcgen05.mma product in this process did not complete within the kernel's "
                           "bounded wait; no further hardware tiles are launched in this process")


def _check_wait(err) -> None:
    global _WAIT_EXPIRED
    if int(err.item()):
        _WAIT_EXPIRED = True
        raise RuntimeError("a tcgen05.mma product did not complete within the kernel's bounded wait; results of "
                           "this process's hardware tiles are untrusted from here on")


def default_d_type(a_format: str) -> str:
    return "s32" if KINDS[a_format] == 3 else "f32"


def instr_desc(a_format: str, b_format: str | None = None, *, saturate: bool = False,
               d_type: str | None = None) -> tuple[int, int]:
    """(kind, instruction descriptor) for an M=128, N=16 dense tile of K-major
    operands; d_type is the accumulator: f32 (default for floating-point
    kinds), f16 (kind::f16 with F16 operands, or kind::f8f6f4) or s32
    (kind::i8)."""
    b_format = b_format or a_format
    if a_format not in KINDS or b_format not in KINDS or KINDS[a_format] != KINDS[b_format]:
        raise ValueError(f"no tcgen05 kind takes {a_format} x {b_format} here")
    kind = KINDS[a_format]
    if kind in (0, 1) and a_format != b_format:
        raise ValueError("kind::tf32 and kind::f16 take one format for A and B")
    d_type = d_type or default_d_type(a_format)
    allowed = {0: ("f32",), 1: ("f32", "f16") if a_format == "f16" else ("f32",), 2: ("f32", "f16"), 3: ("s32",)}
    if d_type not in allowed[kind]:
        raise ValueError(f"{a_format} x {b_format} does not accumulate into {d_type}")
    if saturate and kind != 3:
        raise ValueError("saturation applies to kind::i8 only")
    desc = (C_FORMATS[d_type] << 4) | (FORMAT_CODES[a_format] << 7) | (FORMAT_CODES[b_format] << 10) \
        | ((N >> 3) << 17) | ((M >> 4) << 24) | ((1 if saturate else 0) << 3)
    return kind, desc


def smem_rows(words, fmt: str) -> np.ndarray:
    """[R, K] container words -> [R, 32] bytes, the operand rows the kernel
    stages: one instruction's K packed little-endian, except that an
    E2M3/E3M2/E2M1 row of 32 elements is two 16-byte chunks of 16 packed
    elements followed by zero padding (the f8f6f4 shared-memory form of the
    6- and 4-bit types)."""
    w = np.asarray(words, dtype=np.uint32)
    rows, k = w.shape
    fid = nat.FORMAT_IDS[fmt]
    if fmt in SUB_BYTE:
        if k != 32:
            raise ValueError("f8f6f4 rows hold 32 elements")
        return packing.pack_rows(w.reshape(rows * 2, 16), fid, stride=16).reshape(rows, 32)
    out = packing.pack_rows(w, fid)
    if out.shape[1] != 32:
        raise ValueError(f"{fmt} rows of {k} elements are not 32 bytes")
    return out


def hardware_tiles(a, b, c, a_format: str, b_format: str | None = None, *, saturate: bool = False,
                   d_type: str | None = None, device=None):
    """D words of T tiles computed by tcgen05.mma: a [T, 128, K], b [T, K, 16]
    (row-major B), c [T, 128, 16] container words (uint32 numpy arrays; F16
    accumulators in the low 16 bits, and the hardware leaves the upper 16
    bits of an F16 accumulator column zero)."""
    _refuse_after_timeout()
    import torch

    b_format = b_format or a_format
    d_type = d_type or default_d_type(a_format)
    kind, desc = instr_desc(a_format, b_format, saturate=saturate, d_type=d_type)
    k = K_OF_KIND[kind]
    a = np.asarray(a, dtype=np.uint32)
    b = np.asarray(b, dtype=np.uint32)
    t = a.shape[0]
    if a.shape != (t, M, k) or b.shape != (t, k, N) or np.asarray(c).shape != (t, M, N):
        raise ValueError(f"tiles must be A [T,{M},{k}], B [T,{k},{N}], C [T,{M},{N}]")
    dev = runtime.require_device(device)
    a_rows = smem_rows(a.reshape(t * M, k), a_format)
    b_rows = smem_rows(np.ascontiguousarray(b.transpose(0, 2, 1)).reshape(t * N, k), b_format)
    c_words = np.asarray(c, dtype=np.uint32).reshape(-1)
    if d_type == "f16":
        c_words = c_words & 0xFFFF
    a_dev = runtime.to_device(a_rows, dev)
    b_dev = runtime.to_device(b_rows, dev)
    c_dev = runtime.to_device(c_words, dev)
    d_dev = torch.zeros(t * M * N, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = nat.load()
    stream = ctypes.c_void_p(runtime.current_stream_handle(dev))
    rc = lib.t5e_tcgen05_tiles(kind, desc, a_dev.data_ptr(), b_dev.data_ptr(), c_dev.data_ptr(), d_dev.data_ptr(),
                               t, err.data_ptr(), stream)
    nat.check(rc, "t5e_tcgen05_tiles")
    torch.cuda.synchronize(dev)
    _check_wait(err)
    return d_dev.cpu().numpy().view(np.uint32).reshape(t, M, N)


# The reference model's F16 x F16 -> F16 path (kind::f16 with an F16
# accumulator: Tcgen05MixedRawWindowMmaModel without a product decoder,
# tcgen05_model/model.py:579-583, so eval falls back to the base class,
# model.py:644-646 and 383-429) reports special results with its F32 words, while the
# B200 writes F16 words there; finite results agree.  The emulator keeps the
# reference's words, and the cross-check counts this pairing on its own.
REFERENCE_F32_SPECIAL_FOR_F16 = {0x7FFF: 0x7FFF_FFFF, 0x7C00: 0x7F80_0000, 0xFC00: 0xFF80_0000}


def cross_check(a, b, c, a_format: str, b_format: str | None = None, *, saturate: bool = False,
                d_type: str | None = None, device=None) -> dict:
    """Hardware and emulator words (full 32-bit words) for the same tiles, and
    their differences.  ``mismatches`` counts every differing word except, on
    the F16 x F16 -> F16 path, a hardware F16 special word facing the
    reference's F32 word for the same special value; those are counted in
    ``reference_f32_special_words``."""
    from .simulator import mma_batch

    b_format = b_format or a_format
    d_type = d_type or default_d_type(a_format)
    hw = hardware_tiles(a, b, c, a_format, b_format, saturate=saturate, d_type=d_type, device=device)
    c_in = np.asarray(c, dtype=np.uint32) & 0xFFFF if d_type == "f16" else c
    emu = mma_batch(a, b, c_in, a_format=a_format, b_format=None if b_format == a_format else b_format,
                    d_type=d_type, saturate=saturate, device=device)
    emu = np.asarray(emu, dtype=np.uint32)
    hw_flat, emu_flat = hw.reshape(-1), emu.reshape(-1)
    differ = hw_flat != emu_flat
    explained = np.zeros_like(differ)
    if a_format == b_format == "f16" and d_type == "f16":
        for hw_word, ref_word in REFERENCE_F32_SPECIAL_FOR_F16.items():
            explained |= (hw_flat == hw_word) & (emu_flat == ref_word)
    diff = np.flatnonzero(differ & ~explained)
    return {"a_format": a_format, "b_format": b_format, "d_type": d_type, "saturate": saturate,
            "cases": int(hw.size), "mismatches": int(diff.size),
            "reference_f32_special_words": int((differ & explained).sum()), "first": [int(i) for i in diff[:8]],
            "hardware": hw, "emulator": emu}


def random_tiles(a_format: str, b_format: str | None, tiles: int, seed: int, d_type: str | None = None):
    """Tiles of container words: half raw words (NaN/Inf/subnormals
    included), half finite, as the validation paths draw them."""
    from . import workloads

    b_format = b_format or a_format
    d_type = d_type or default_d_type(a_format)
    k = K_OF_KIND[KINDS[a_format]]
    rng = np.random.Generator(np.random.PCG64(seed))
    half = tiles // 2

    def words(fmt, n):
        raw = workloads.format_words(fmt, rng, half * n)
        fin = workloads.format_words(fmt, rng, (tiles - half) * n, True)
        return np.concatenate([raw, fin]).astype(np.uint32)

    a = words(a_format, M * k).reshape(tiles, M, k)
    b = words(b_format, k * N).reshape(tiles, k, N)
    if d_type == "s32":
        c = rng.integers(0, 1 << 32, size=tiles * M * N, dtype=np.uint64).astype(np.uint32)
    elif d_type == "f16":
        c = np.concatenate([workloads.f16_words(rng, half * M * N),
                            workloads.f16_words(rng, (tiles - half) * M * N, True)]).astype(np.uint32)
    else:
        c = np.concatenate([workloads.f32_words(rng, half * M * N),
                            workloads.f32_words(rng, (tiles - half) * M * N, True)]).astype(np.uint32)
    return a, b, c.reshape(tiles, M, N)


F8F6F4 = ("e4m3", "e5m2", "e2m3", "e3m2", "e2m1")

# (A format, B format, saturate, accumulator): every dense kind, every
# f8f6f4 operand pair into F32 and into F16, and the integer signedness and
# saturation modes
PAIRS = (("tf32", "tf32", False, "f32"), ("bf16", "bf16", False, "f32"), ("f16", "f16", False, "f32"),
         ("f16", "f16", False, "f16")) \
    + tuple((fa, fb, False, d) for d in ("f32", "f16") for fa, fb in itertools.product(F8F6F4, F8F6F4)) \
    + (("u8", "s8", False, "s32"), ("s8", "u8", False, "s32"), ("u8", "u8", False, "s32"), ("s8", "s8", True, "s32"))


# ---- block-scaled kinds ------------------------------------------------
#
# Tiles of M = 128, N = 128 and one instruction's K: 32 f8f6f4 elements
# (kind::mxf8f6f4, one UE8M0 scale per row and column), or 64 packed E2M1
# (kind::mxf4: two UE8M0 scales; kind::mxf4nvf4: two UE8M0 or four UE4M3 /
# UE8M0 scales).  The emulator side is the matching make_model descriptor:
# scaling, kind and scale_vec as the reference names them.
BS_N = 128
BS_KINDS = {"mxf8f6f4": 4, "mxf4": 5, "mxf4nvf4-2x": 6, "mxf4nvf4-4x": 7}
BS_K = {"mxf8f6f4": 32, "mxf4": 64, "mxf4nvf4-2x": 64, "mxf4nvf4-4x": 64}
BS_BLOCKS = {"mxf8f6f4": 1, "mxf4": 2, "mxf4nvf4-2x": 2, "mxf4nvf4-4x": 4}
MXF4_E2M1 = 1  # the E2M1 code of the mxf4 kinds (packed operands)


def block_scaled_desc(kind: str, a_format: str, b_format: str | None = None, scale: str = "ue8m0") -> tuple[int, int]:
    """(kind id, block-scaled instruction descriptor): formats at bits 7-9 and
    10-12, N/8 at 17-22, the scale format at bit 23 (1 = UE8M0, 0 = UE4M3),
    M/16 at 24-28, scale factor ids 0."""
    b_format = b_format or a_format
    if kind not in BS_KINDS:
        raise ValueError(f"unknown block-scaled kind {kind}")
    if kind == "mxf8f6f4":
        if a_format not in FORMAT_CODES or KINDS.get(a_format) != 2 or KINDS.get(b_format) != 2:
            raise ValueError("kind::mxf8f6f4 takes f8f6f4 operands")
        fa, fb = FORMAT_CODES[a_format], FORMAT_CODES[b_format]
    else:
        if a_format != "e2m1" or b_format != "e2m1":
            raise ValueError(f"kind::{kind} takes E2M1 operands")
        fa = fb = MXF4_E2M1
    if scale not in ("ue8m0", "ue4m3") or (scale == "ue4m3" and kind != "mxf4nvf4-4x"):
        raise ValueError(f"{kind} does not take {scale} scales")
    desc = (fa << 7) | (fb << 10) | ((BS_N >> 3) << 17) | ((1 if scale == "ue8m0" else 0) << 23) | ((M >> 4) << 24)
    return BS_KINDS[kind], desc


def block_scaled_model_args(kind: str, scale: str) -> dict:
    """make_model keywords of the emulator path a block-scaled kind runs."""
    if kind == "mxf8f6f4":
        return dict(scaling="ue8m0", kind="mxf8f6f4")
    if kind == "mxf4":
        return dict(scaling="ue8m0", kind="mxf4")
    if kind == "mxf4nvf4-2x":
        return dict(scaling="ue8m0", kind="mxf4nvf4", scale_vec=2)
    return dict(scaling="ue4m3", scale_vec=4) if scale == "ue4m3" else dict(scaling="ue8m0", kind="mxf4nvf4",
                                                                           scale_vec=4)


def block_scaled_rows(words, fmt: str, kind: str) -> np.ndarray:
    """[R, K] words -> [R, 32] operand bytes: the f8f6f4 form for
    kind::mxf8f6f4, 64 packed E2M1 otherwise."""
    if kind == "mxf8f6f4":
        return smem_rows(words, fmt)
    w = np.asarray(words, dtype=np.uint32)
    out = packing.pack_rows(w, nat.FORMAT_IDS["e2m1"])
    if out.shape[1] != 32:
        raise ValueError("mxf4 rows hold 64 E2M1 elements")
    return out


def scale_words(scales) -> np.ndarray:
    """[R, blocks] scale bytes -> R words, block j in byte j."""
    s = np.asarray(scales, dtype=np.uint32)
    w = np.zeros(s.shape[0], dtype=np.uint32)
    for j in range(s.shape[1]):
        w |= (s[:, j] & 0xFF) << (8 * j)
    return w


def hardware_block_scaled_tiles(a, b, c, scale_a, scale_b, kind: str, a_format: str, b_format: str | None = None,
                                scale: str = "ue8m0", device=None):
    """D words of T block-scaled tiles computed by tcgen05.mma: a [T, 128, K],
    b [T, K, 128] (row-major B), c [T, 128, 128] F32 words, scale_a
    [T, 128, blocks] (per A row), scale_b [T, 128, blocks] (per B column)."""
    _refuse_after_timeout()
    import torch

    b_format = b_format or a_format
    kid, desc = block_scaled_desc(kind, a_format, b_format, scale)
    k, blocks = BS_K[kind], BS_BLOCKS[kind]
    a = np.asarray(a, dtype=np.uint32)
    b = np.asarray(b, dtype=np.uint32)
    t = a.shape[0]
    shapes = (a.shape, b.shape, np.asarray(c).shape, np.asarray(scale_a).shape, np.asarray(scale_b).shape)
    if shapes != ((t, M, k), (t, k, BS_N), (t, M, BS_N), (t, M, blocks), (t, BS_N, blocks)):
        raise ValueError(f"tiles must be A [T,{M},{k}], B [T,{k},{BS_N}], C [T,{M},{BS_N}], scales [T,128,{blocks}]")
    dev = runtime.require_device(device)
    a_dev = runtime.to_device(block_scaled_rows(a.reshape(t * M, k), a_format, kind), dev)
    b_dev = runtime.to_device(block_scaled_rows(np.ascontiguousarray(b.transpose(0, 2, 1)).reshape(t * BS_N, k),
                                                b_format, kind), dev)
    c_dev = runtime.to_device(np.asarray(c, dtype=np.uint32).reshape(-1), dev)
    sa_dev = runtime.to_device(scale_words(np.asarray(scale_a).reshape(t * M, blocks)), dev)
    sb_dev = runtime.to_device(scale_words(np.asarray(scale_b).reshape(t * BS_N, blocks)), dev)
    d_dev = torch.zeros(t * M * BS_N, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = nat.load()
    stream = ctypes.c_void_p(runtime.current_stream_handle(dev))
    rc = lib.t5e_tcgen05_block_scaled_tiles(kid, desc, a_dev.data_ptr(), b_dev.data_ptr(), c_dev.data_ptr(),
                                            d_dev.data_ptr(), sa_dev.data_ptr(), sb_dev.data_ptr(), t,
                                            err.data_ptr(), stream)
    nat.check(rc, "t5e_tcgen05_block_scaled_tiles")
    torch.cuda.synchronize(dev)
    _check_wait(err)
    return d_dev.cpu().numpy().view(np.uint32).reshape(t, M, BS_N)


def cross_check_block_scaled(a, b, c, scale_a, scale_b, kind: str, a_format: str, b_format: str | None = None,
                             scale: str = "ue8m0", device=None) -> dict:
    """Hardware and emulator words of the same block-scaled tiles."""
    from .simulator import mma_batch

    b_format = b_format or a_format
    hw = hardware_block_scaled_tiles(a, b, c, scale_a, scale_b, kind, a_format, b_format, scale, device=device)
    emu = mma_batch(a, b, c, a_format=a_format, b_format=None if b_format == a_format else b_format,
                    scale_a=scale_a, scale_b=scale_b, device=device, **block_scaled_model_args(kind, scale))
    emu = np.asarray(emu, dtype=np.uint32)
    diff = np.flatnonzero(hw.reshape(-1) != emu.reshape(-1))
    return {"kind": kind, "a_format": a_format, "b_format": b_format, "scale": scale, "cases": int(hw.size),
            "mismatches": int(diff.size), "first": [int(i) for i in diff[:8]], "hardware": hw, "emulator": emu}


def random_block_scaled_tiles(kind: str, a_format: str, b_format: str | None, tiles: int, seed: int,
                              scale: str = "ue8m0"):
    """Tiles as random_tiles draws them, plus scales over the reference
    generators' ranges: UE8M0 over all 256 bytes (0xFF is NaN), UE4M3 over
    0x00-0x7F (0x7F is NaN)."""
    from . import workloads

    b_format = b_format or a_format
    k, blocks = BS_K[kind], BS_BLOCKS[kind]
    rng = np.random.Generator(np.random.PCG64(seed))
    half = tiles // 2

    def words(fmt, n):
        raw = workloads.format_words(fmt, rng, half * n)
        fin = workloads.format_words(fmt, rng, (tiles - half) * n, True)
        return np.concatenate([raw, fin]).astype(np.uint32)

    a = words(a_format, M * k).reshape(tiles, M, k)
    b = words(b_format, k * BS_N).reshape(tiles, k, BS_N)
    c = np.concatenate([workloads.f32_words(rng, half * M * BS_N),
                        workloads.f32_words(rng, (tiles - half) * M * BS_N, True)]).astype(np.uint32)
    top = 256 if scale == "ue8m0" else 128
    sa = rng.integers(0, top, size=(tiles, M, blocks), dtype=np.uint64).astype(np.uint32)
    sb = rng.integers(0, top, size=(tiles, BS_N, blocks), dtype=np.uint64).astype(np.uint32)
    return a, b, c.reshape(tiles, M, BS_N), sa, sb


# (kind, A format, B format, scale format): every mxf8f6f4 operand pair and
# every mxf4 / mxf4nvf4 form
BS_PAIRS = tuple(("mxf8f6f4", fa, fb, "ue8m0") for fa, fb in itertools.product(F8F6F4, F8F6F4)) + (
    ("mxf4", "e2m1", "e2m1", "ue8m0"), ("mxf4nvf4-2x", "e2m1", "e2m1", "ue8m0"),
    ("mxf4nvf4-4x", "e2m1", "e2m1", "ue8m0"), ("mxf4nvf4-4x", "e2m1", "e2m1", "ue4m3"))


# ---- sparse kinds ------------------------------------------------------
#
# tcgen05.mma.sp on uniform tiles, one case per tile (t5e_tcgen05_sparse_cases):
# the sparse validation paths' own cases (sweep.host_cases), A compressed in
# the order its metadata selects (a 2:4 selector's low index first, as the
# reference harness packs it, hardware_validation/src/
# tcgen05_block_scaled_sparse_probe.cu:304-321), B at the logical K.  The
# emulator side is mma_dot_batch on the same logical cases with their
# metadata.
SP_KINDS = {"tf32": 8, "f16": 9, "f8f6f4": 10, "mxf8f6f4": 11, "mxf4": 12, "mxf4nvf4-2x": 13, "mxf4nvf4-4x": 14}
SP_N = 8
SP_SCALED = ("mxf8f6f4", "mxf4", "mxf4nvf4-2x", "mxf4nvf4-4x")
SP_PACKED_E2M1 = ("mxf4", "mxf4nvf4-2x", "mxf4nvf4-4x")
# metadata word pattern per kind (t5e_tcgen05_sparse_cases' meta_layout): the
# reference harness's patterns, 16-bit halves by lane for kind::tf32 and
# kind::f16, the two words in alternate columns otherwise
SP_LAYOUT = {"tf32": 1, "f16": 1}


def sparse_kind(spec) -> tuple[str, str | None]:
    """(sparse instruction kind, scale format or None) of a sparse validation path."""
    fam, fmt = spec.family, spec.descriptor["a_format"]
    if fam == "sparse":
        return ("tf32" if fmt == "tf32" else "f16" if fmt in ("bf16", "f16") else "f8f6f4"), None
    if fam == "sparse-mx":
        return "mxf8f6f4", "ue8m0"
    if fam == "sparse-nvfp4":
        return "mxf4nvf4-4x", "ue4m3"
    if fam == "sparse-fp4block":
        kind = spec.params[0]
        return ("mxf4nvf4-4x" if kind.startswith("mxf4nvf4-4x") else kind), \
            ("ue4m3" if kind.endswith("ue4m3") else "ue8m0")
    raise ValueError(f"{spec.name} is not a sparse path")


def sparse_desc(kind: str, a_format: str, scale: str | None = None) -> int:
    """Sparse instruction descriptor of a uniform tile: the sparse flag (bit
    2), formats, N = 8, M = 64 (M = 128 for the block-scaled kinds), an F32
    accumulator or the scale format."""
    if kind not in SP_KINDS:
        raise ValueError(f"unknown sparse kind {kind}")
    scaled = kind in SP_SCALED
    fa = MXF4_E2M1 if kind in SP_PACKED_E2M1 else FORMAT_CODES[a_format]
    desc = (1 << 2) | (fa << 7) | (fa << 10) | ((SP_N >> 3) << 17) | (((128 if scaled else 64) >> 4) << 24)
    if scaled:
        return desc | ((1 if scale == "ue8m0" else 0) << 23)
    return desc | (C_FORMATS["f32"] << 4)


def operand_bytes(words, fmt: str, kind: str) -> np.ndarray:
    """[R, K] words -> [R, bytes] operand rows: packed E2M1 for the mxf4
    kinds, 16-byte chunks of 16 packed elements (zero padded) for
    E2M3/E3M2/E2M1 in the f8f6f4 kinds, packed little-endian otherwise."""
    w = np.asarray(words, dtype=np.uint32)
    rows, k = w.shape
    if kind in SP_PACKED_E2M1:
        return packing.pack_rows(w, nat.FORMAT_IDS["e2m1"])
    fid = nat.FORMAT_IDS[fmt]
    if fmt in SUB_BYTE:
        if k % 16:
            raise ValueError("f8f6f4 sub-byte rows hold whole 16-element chunks")
        return packing.pack_rows(w.reshape(rows * (k // 16), 16), fid, stride=16).reshape(rows, k)
    return packing.pack_rows(w, fid)


def compress_a(a, meta, k: int, mode: str) -> np.ndarray:
    """Logical A rows [n, k] -> the k/2 elements each row's metadata selects,
    in selector order: 1:2 takes element 1 of a pair for selector 0xE and
    element 0 otherwise; 2:4 the two 2-bit indices of a nibble, low first;
    pairwise 4:8 the two pairs a nibble names, low first."""
    a = np.asarray(a, dtype=np.uint32)
    meta = np.asarray(meta, dtype=np.uint32)
    n = a.shape[0]
    rows = np.arange(n)
    size = {"1of2": 2, "2of4": 4, "4of8": 8}[mode]
    out = np.zeros((n, k // 2), dtype=np.uint32)
    for ch in range(k // size):
        sel = (meta[:, 0 if ch < 8 else 1] >> np.uint32(4 * (ch % 8))) & 0xF
        if mode == "1of2":
            out[:, ch] = a[rows, 2 * ch + (sel == 0xE)]
        elif mode == "2of4":
            for j in range(2):
                out[:, 2 * ch + j] = a[rows, 4 * ch + ((sel >> np.uint32(2 * j)) & 3)]
        else:
            for j in range(4):
                pair = (sel >> np.uint32(2 * (j // 2))) & 3
                out[:, 4 * ch + j] = a[rows, 8 * ch + 2 * pair + (j & 1)]
    return out


def hardware_sparse_cases(cases, spec, *, layout: int | None = None, dump: bool = False, device=None) -> dict:
    """Run a sparse path's cases (a ``workloads.Cases`` of logical words and
    metadata) as uniform tcgen05.mma.sp tiles: {"d": words, "disagree":
    per-case counts, "dump": [n, 128, 8] TMEM words or None}."""
    _refuse_after_timeout()
    import torch

    from . import sweep

    kind, scale = sparse_kind(spec)
    fmt = spec.descriptor["a_format"]
    desc = sparse_desc(kind, fmt, scale)
    layout = SP_LAYOUT.get(kind, 0) if layout is None else layout
    mode = sweep.sparse_mode(spec)
    n, k = cases.a.shape
    a_rows = operand_bytes(compress_a(cases.a, cases.meta, k, mode), fmt, kind)
    b_rows = operand_bytes(cases.b, fmt, kind)
    if a_rows.shape[1] != 32 or b_rows.shape[1] != 64:
        raise ValueError(f"{spec.name}: operand rows of {a_rows.shape[1]} / {b_rows.shape[1]} bytes, expected 32 / 64")
    meta = np.zeros((n, 2), dtype=np.uint32)
    meta[:, : cases.meta.shape[1]] = cases.meta
    if cases.meta.shape[1] == 1:
        meta[:, 1] = cases.meta[:, 0]
    dev = runtime.require_device(device)
    scales_dev = None
    if kind in SP_SCALED:
        blocks = sweep.scale_blocks(spec)
        sw = np.stack([scale_words(cases.scale_a[:, :blocks]), scale_words(cases.scale_b[:, :blocks])], axis=1)
        scales_dev = runtime.to_device(np.ascontiguousarray(sw).reshape(-1), dev)
    a_dev = runtime.to_device(np.ascontiguousarray(a_rows), dev)
    b_dev = runtime.to_device(np.ascontiguousarray(b_rows), dev)
    c_dev = runtime.to_device(np.asarray(cases.c, dtype=np.uint32), dev)
    m_dev = runtime.to_device(meta.reshape(-1), dev)
    d_dev = torch.zeros(n, dtype=torch.int32, device=dev)
    bad_dev = torch.zeros(n, dtype=torch.int32, device=dev)
    dump_dev = torch.zeros(n * 128 * SP_N, dtype=torch.int32, device=dev) if dump else None
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = nat.load()
    stream = ctypes.c_void_p(runtime.current_stream_handle(dev))
    ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
    rc = lib.t5e_tcgen05_sparse_cases(SP_KINDS[kind], desc, layout, a_dev.data_ptr(), b_dev.data_ptr(),
                                      c_dev.data_ptr(), m_dev.data_ptr(), ptr(scales_dev), d_dev.data_ptr(),
                                      bad_dev.data_ptr(), ptr(dump_dev), n, err.data_ptr(), stream)
    nat.check(rc, "t5e_tcgen05_sparse_cases")
    torch.cuda.synchronize(dev)
    _check_wait(err)
    out = {"d": d_dev.cpu().numpy().view(np.uint32), "disagree": bad_dev.cpu().numpy(), "dump": None}
    if dump:
        out["dump"] = dump_dev.cpu().numpy().view(np.uint32).reshape(n, 128, SP_N)
    return out


def cross_check_sparse(spec, n: int = 1024, *, layout: int | None = None, device=None) -> dict:
    """Hardware and emulator words of the first n cases of a sparse path."""
    from . import sweep
    from .simulator import mma_dot_batch

    cases = sweep.host_cases(spec, 0, n, n)
    hw = hardware_sparse_cases(cases, spec, layout=layout, device=device)
    d = spec.descriptor
    kw = {key: d[key] for key in ("a_format", "b_format", "d_type", "saturate", "scaling", "scale_vec", "kind")}
    emu = np.asarray(mma_dot_batch(cases.a, cases.b, cases.c, scale_a=cases.scale_a, scale_b=cases.scale_b,
                                   sparse_metadata=cases.meta, device=device, **kw), dtype=np.uint32)
    diff = np.flatnonzero(hw["d"] != emu)
    kind, scale = sparse_kind(spec)
    return {"path": spec.name, "kind": kind, "scale": scale, "layout": SP_LAYOUT.get(kind, 0) if layout is None
            else layout, "cases": n, "mismatches": int(diff.size), "first": [int(i) for i in diff[:8]],
            "nonuniform_tiles": int((hw["disagree"] != 0).sum()), "hardware": hw["d"], "emulator": emu}


def sparse_paths():
    """The sparse validation paths, in workload order."""
    from . import workloads

    return [p for p in workloads.validation_paths() if p.family.startswith("sparse")]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tiles", type=int, default=64)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--sparse-cases", type=int, default=1024)
    args = ap.parse_args(argv)
    failed = 0
    for i, (fa, fb, sat, d) in enumerate(PAIRS):
        a, b, c = random_tiles(fa, fb, args.tiles, args.seed + i, d)
        r = cross_check(a, b, c, fa, fb, saturate=sat, d_type=d)
        failed += r["mismatches"] != 0
        print(json.dumps({k: v for k, v in r.items() if k not in ("hardware", "emulator")}), flush=True)
    bs_failed = 0
    for i, (kind, fa, fb, scale) in enumerate(BS_PAIRS):
        a, b, c, sa, sb = random_block_scaled_tiles(kind, fa, fb, max(2, args.tiles // 8), args.seed + 1000 + i,
                                                    scale)
        r = cross_check_block_scaled(a, b, c, sa, sb, kind, fa, fb, scale)
        bs_failed += r["mismatches"] != 0
        print(json.dumps({k: v for k, v in r.items() if k not in ("hardware", "emulator")}), flush=True)
    sp_failed = 0
    for spec in sparse_paths():
        r = cross_check_sparse(spec, args.sparse_cases)
        sp_failed += r["mismatches"] != 0 or r["nonuniform_tiles"] != 0
        print(json.dumps({k: v for k, v in r.items() if k not in ("hardware", "emulator")}), flush=True)
    print(json.dumps({"pairs": len(PAIRS), "pairs_with_mismatches": failed, "block_scaled_pairs": len(BS_PAIRS),
                      "block_scaled_pairs_with_mismatches": bs_failed, "sparse_paths": len(sparse_paths()),
                      "sparse_paths_with_mismatches": sp_failed}), flush=True)
    return 1 if failed or bs_failed or sp_failed else 0


if __name__ == "__main__":
    raise SystemExit(main())

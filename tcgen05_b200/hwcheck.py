"""Cross-check of the emulator against the B200's own tensor cores.

``hardware_tiles`` runs real ``tcgen05.mma`` instructions (kind::tf32,
kind::f16, kind::f8f6f4 with E4M3/E5M2 operands, kind::i8) on tiles
D = A B + C of M = 128, N = 16 and one instruction's K, through
``t5e_tcgen05_tiles``; ``cross_check`` evaluates the same tiles with the
emulator (``mma_batch``) and counts the words on which the two differ.  This
is the comparison the reference's hardware harness makes between its probe
runners and its model (hardware_validation/mma_probe.py), here between the
hardware and this library.

    python -m tcgen05_b200.hwcheck [--tiles 64] [--seed 0]
"""

from __future__ import annotations

import argparse
import ctypes
import json

import numpy as np

from . import _native as nat
from . import packing, runtime

M, N = 128, 16

# instruction kinds and descriptor format codes (the tcgen05 instruction
# descriptor: bits 4-5 accumulator format, 7-9 A format, 10-12 B format,
# 17-22 N/8, 24-28 M/16, bit 3 saturation)
KINDS = {"tf32": 0, "bf16": 1, "f16": 1, "e4m3": 2, "e5m2": 2, "u8": 3, "s8": 3}
FORMAT_CODES = {"tf32": 2, "bf16": 1, "f16": 0, "e4m3": 0, "e5m2": 1, "u8": 0, "s8": 1}
K_OF_KIND = {0: 8, 1: 16, 2: 32, 3: 32}
C_F32, C_S32 = 1, 2


def instr_desc(a_format: str, b_format: str | None = None, *, saturate: bool = False) -> tuple[int, int]:
    """(kind, instruction descriptor) for an M=128, N=16 tile with an F32
    (floating-point kinds) or S32 (kind::i8) accumulator."""
    b_format = b_format or a_format
    if a_format not in KINDS or b_format not in KINDS or KINDS[a_format] != KINDS[b_format]:
        raise ValueError(f"no tcgen05 kind takes {a_format} x {b_format} here")
    kind = KINDS[a_format]
    if kind in (0, 1) and a_format != b_format:
        raise ValueError("kind::tf32 and kind::f16 take one format for A and B")
    c_fmt = C_S32 if kind == 3 else C_F32
    desc = (c_fmt << 4) | (FORMAT_CODES[a_format] << 7) | (FORMAT_CODES[b_format] << 10) | ((N >> 3) << 17) \
        | ((M >> 4) << 24) | ((1 if saturate else 0) << 3)
    if saturate and kind != 3:
        raise ValueError("saturation applies to kind::i8 only")
    return kind, desc


def hardware_tiles(a, b, c, a_format: str, b_format: str | None = None, *, saturate: bool = False, device=None):
    """D words of T tiles computed by tcgen05.mma: a [T, 128, K], b [T, K, 16]
    (row-major B), c [T, 128, 16] container words (uint32 numpy arrays)."""
    import torch

    b_format = b_format or a_format
    kind, desc = instr_desc(a_format, b_format, saturate=saturate)
    k = K_OF_KIND[kind]
    a = np.asarray(a, dtype=np.uint32)
    b = np.asarray(b, dtype=np.uint32)
    t = a.shape[0]
    if a.shape != (t, M, k) or b.shape != (t, k, N) or np.asarray(c).shape != (t, M, N):
        raise ValueError(f"tiles must be A [T,{M},{k}], B [T,{k},{N}], C [T,{M},{N}]")
    dev = runtime.require_device(device)
    fa, fb = nat.FORMAT_IDS[a_format], nat.FORMAT_IDS[b_format]
    a_rows = packing.pack_rows(a.reshape(t * M, k), fa)
    b_rows = packing.pack_rows(np.ascontiguousarray(b.transpose(0, 2, 1)).reshape(t * N, k), fb)
    assert a_rows.shape[1] == 32 and b_rows.shape[1] == 32
    a_dev = runtime.to_device(a_rows, dev)
    b_dev = runtime.to_device(b_rows, dev)
    c_dev = runtime.to_device(np.asarray(c, dtype=np.uint32).reshape(-1), dev)
    d_dev = torch.zeros(t * M * N, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = nat.load()
    stream = ctypes.c_void_p(runtime.current_stream_handle(dev))
    rc = lib.t5e_tcgen05_tiles(kind, desc, a_dev.data_ptr(), b_dev.data_ptr(), c_dev.data_ptr(), d_dev.data_ptr(),
                               t, err.data_ptr(), stream)
    nat.check(rc, "t5e_tcgen05_tiles")
    torch.cuda.synchronize(dev)
    if int(err.item()):
        raise RuntimeError("a tcgen05.mma product did not complete within the kernel's bounded wait")
    return d_dev.cpu().numpy().view(np.uint32).reshape(t, M, N)


def cross_check(a, b, c, a_format: str, b_format: str | None = None, *, saturate: bool = False, device=None) -> dict:
    """Hardware and emulator words for the same tiles, and their differences."""
    from .simulator import mma_batch

    b_format = b_format or a_format
    hw = hardware_tiles(a, b, c, a_format, b_format, saturate=saturate, device=device)
    d_type = "s32" if KINDS[a_format] == 3 else "f32"
    emu = mma_batch(a, b, c, a_format=a_format, b_format=None if b_format == a_format else b_format, d_type=d_type,
                    saturate=saturate, device=device)
    diff = np.flatnonzero(hw.reshape(-1) != emu.reshape(-1))
    return {"a_format": a_format, "b_format": b_format, "saturate": saturate, "cases": int(hw.size),
            "mismatches": int(diff.size), "first": [int(i) for i in diff[:8]], "hardware": hw, "emulator": emu}


def random_tiles(a_format: str, b_format: str | None, tiles: int, seed: int):
    """Tiles of container words: half raw words (NaN/Inf/subnormals
    included), half finite, as the validation paths draw them."""
    from . import workloads

    b_format = b_format or a_format
    k = K_OF_KIND[KINDS[a_format]]
    rng = np.random.Generator(np.random.PCG64(seed))
    half = tiles // 2

    def words(fmt, n):
        raw = workloads.format_words(fmt, rng, half * n)
        fin = workloads.format_words(fmt, rng, (tiles - half) * n, True)
        return np.concatenate([raw, fin]).astype(np.uint32)

    a = words(a_format, M * k).reshape(tiles, M, k)
    b = words(b_format, k * N).reshape(tiles, k, N)
    if KINDS[a_format] == 3:
        c = rng.integers(0, 1 << 32, size=tiles * M * N, dtype=np.uint64).astype(np.uint32)
    else:
        c = np.concatenate([workloads.f32_words(rng, half * M * N),
                            workloads.f32_words(rng, (tiles - half) * M * N, True)]).astype(np.uint32)
    return a, b, c.reshape(tiles, M, N)


PAIRS = (("tf32", "tf32", False), ("bf16", "bf16", False), ("f16", "f16", False), ("e4m3", "e4m3", False),
         ("e5m2", "e5m2", False), ("e4m3", "e5m2", False), ("u8", "s8", False), ("s8", "s8", True))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tiles", type=int, default=64)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    failed = 0
    for i, (fa, fb, sat) in enumerate(PAIRS):
        a, b, c = random_tiles(fa, fb, args.tiles, args.seed + i)
        r = cross_check(a, b, c, fa, fb, saturate=sat)
        failed += r["mismatches"] != 0
        print(json.dumps({k: v for k, v in r.items() if k not in ("hardware", "emulator")}), flush=True)
    return 1 if failed else 0


if __name__ == "__main__":
    raise SystemExit(main())

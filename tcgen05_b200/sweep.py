"""The 46-path sweep: every modeled tcgen05 path at a fixed number of seeded
cases, sharded across the GPUs of one node (hardware_validation/
run_full_validation.py drives the same sweep on the hardware side; its
report fields and integrity checks, :235-251 and :359-405, are kept).

Cases are generated where they are evaluated.  A case's words are a
counter-based hash of (path seed, case index, word slot, stream), so any
shard of any path can be produced independently, on the GPU with torch or on
the host with numpy, bit for bit the same (one implementation, written
against either array module).  The distributions follow the reference
harness generators as restated in ``workloads.path_cases``: the first half
of a path's cases draws raw container words (NaN/Inf/subnormals included),
the second half finite ones; scales, C and sparse metadata as there.

Each rank evaluates its contiguous share of every path with the dispatching
entry point and with the generic kernel, counts the words on which they
differ, and folds every (case index, result word) into an order-independent
checksum.  The only collective is the final sum of those per-path counters,
so the report -- checksums included -- is the same at any GPU count.

    python -m tcgen05_b200.sweep [--cases-per-path N] [--output report.json]
    torchrun --nproc-per-node 8 -m tcgen05_b200.sweep ...
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from collections import Counter
from datetime import datetime, timezone

import numpy as np

from . import workloads as W

MASK32 = 0xFFFFFFFF

# stream tags of the hash
S_A, S_B, S_C, S_SA, S_SB, S_META, S_ALT = 1, 2, 3, 4, 5, 6, 7


# ------------------------------------------------------------ hashing


def _mul32(x, c: int):
    """(x * c) mod 2**32 for int64 arrays holding uint32 values, without ever
    exceeding 2**49 (so no array library's integer overflow is involved)."""
    lo = x & 0xFFFF
    hi = x >> 16
    return (lo * c + (((hi * (c & 0xFFFF)) & 0xFFFF) << 16)) & MASK32


def _fmix32(x):
    """The MurmurHash3 32-bit finaliser (a public avalanche mix)."""
    x = x & MASK32
    x = x ^ (x >> 16)
    x = _mul32(x, 0x85EBCA6B)
    x = x ^ (x >> 13)
    x = _mul32(x, 0xC2B2AE35)
    return x ^ (x >> 16)


def case_hash(xp, seed: int, stream: int, idx, slots: int):
    """[n, slots] uint32 values (as int64) for case indices idx [n]."""
    key = (seed * 0x9E3779B1 + stream * 0x7F4A7C15) & MASK32
    row = _fmix32(idx.reshape(-1, 1) ^ key)
    col = _fmix32(_arange(xp, slots, idx).reshape(1, -1) + 0x632BE5AB)
    return _fmix32(row ^ col)


def _arange(xp, n, like):
    if xp is np:
        return np.arange(n, dtype=np.int64)
    return xp.arange(n, dtype=xp.int64, device=like.device)


def _where(xp, cond, x, y):
    return np.where(cond, x, y) if xp is np else xp.where(cond, x, y)


def _take(xp, table, index):
    if xp is np:
        return np.asarray(table, dtype=np.int64)[index]
    t = xp.as_tensor(np.asarray(table, dtype=np.int64), device=index.device)
    return t[index]


# ------------------------------------------------------------ words


def _format_words(xp, fmt: str, finite, h, h2):
    """Container words of a format; ``finite`` [n, 1] selects the cases whose
    specials are redrawn finite (workloads.format_words, finite_only)."""
    if fmt in ("tf32", "bf16"):
        bad = ((h & 0x7F800000) == 0x7F800000) & finite
        return _where(xp, bad, (h & 0x807FFFFF) | ((h2 % 255) << 23), h)
    if fmt == "f16":
        w = h & 0xFFFF
        bad = (((w >> 10) & 0x1F) == 0x1F) & finite
        return _where(xp, bad, (w & ~(0x1F << 10) & 0xFFFF) | ((h2 % 0x1F) << 10), w)
    if fmt == "e4m3":
        w = h & 0xFF
        bad = ((w & 0x7F) == 0x7F) & finite
        return _where(xp, bad, (w & 0x80) | (h2 % 0x7F), w)
    if fmt == "e5m2":
        w = h & 0xFF
        bad = (((w >> 2) & 0x1F) == 0x1F) & finite
        return _where(xp, bad, (w & ~(0x1F << 2) & 0xFF) | ((h2 % 0x1F) << 2), w)
    if fmt in ("e2m3", "e3m2"):
        return h & 0x3F
    if fmt == "e2m1":
        return h & 0xF
    if fmt in ("u8", "s8"):
        return h & 0xFF
    raise ValueError(fmt)


def _f32_c(xp, seed, idx, finite):
    h = case_hash(xp, seed, S_C, idx, 2)
    return _format_words(xp, "tf32", finite, h[:, :1], h[:, 1:2]).reshape(-1)


def _f16_c(xp, seed, idx, finite):
    h = case_hash(xp, seed, S_C, idx, 2)
    return _format_words(xp, "f16", finite, h[:, :1], h[:, 1:2]).reshape(-1)


def _scales(xp, seed, stream, idx, count: int, kind: str, width: int = 4):
    """`count` random scales then unit scales (workloads._scales)."""
    unit, top = (0x38, 0x80) if kind == "ue4m3" else (0x7F, 0x100)
    h = case_hash(xp, seed, stream, idx, width) % top
    keep = _arange(xp, width, idx).reshape(1, -1) < count
    return _where(xp, keep, h, unit)


def _selectors(xp, seed, stream, idx, table):
    """[n] metadata words of eight selectors drawn from `table`."""
    h = case_hash(xp, seed, stream, idx, 8)
    picks = _take(xp, table, h % len(table))
    shifts = _arange(xp, 8, idx).reshape(1, -1) * 4
    return (picks << shifts).sum(1)


def _active(xp, meta, k: int, mode: str):
    """[n, k] selected logical positions (workloads.active_mask)."""
    csize = {"1of2": 2, "2of4": 4, "4of8": 8}[mode]
    chunks = (k + csize - 1) // csize
    pos = _arange(xp, chunks * csize, meta).reshape(1, -1)
    chunk = pos // csize
    word = _where(xp, chunk >= 8, meta[:, 1:2], meta[:, 0:1])
    sel = (word >> ((chunk % 8) * 4)) & 0xF
    off = pos % csize
    if mode == "1of2":
        act = off == _where(xp, sel == 0xE, 1, 0)
    elif mode == "2of4":
        act = (off == (sel & 3)) | (off == ((sel >> 2) & 3))
    else:
        pair = off // 2
        act = (pair == (sel & 3)) | (pair == ((sel >> 2) & 3))
    return act[:, :k]


def path_k(spec: W.PathSpec) -> int:
    """Logical K of a validation path's cases."""
    fam = spec.family
    fmt = spec.descriptor["a_format"]
    if fam == "dense":
        return {"tf32": 8, "bf16": 16, "f16": 16}.get(fmt, 32)
    if fam in ("mixed", "mx", "i8"):
        return 32
    if fam in ("fp4block", "nvfp4"):
        return 64
    if fam == "sparse":
        return {"tf32": 16, "bf16": 32, "f16": 32}.get(spec.params[0], 64)
    if fam == "sparse-mx":
        return 64
    return 128  # sparse-nvfp4, sparse-fp4block


def generate(spec: W.PathSpec, start: int, count: int, total: int, xp=np, device=None) -> dict:
    """Cases [start, start + count) of a path with `total` cases, as arrays of
    the given module (numpy, or torch on `device`): a, b [n, K] words, c [n],
    and scale_a, scale_b [n, S] / meta [n, 2] where the path has them."""
    if xp is np:
        idx = np.arange(start, start + count, dtype=np.int64)
    else:
        idx = xp.arange(start, start + count, dtype=xp.int64, device=device)
    d = spec.descriptor
    fam = spec.family
    seed = spec.seed
    k = path_k(spec)
    finite = (idx >= total // 2).reshape(-1, 1)
    out = {"a": None, "b": None, "c": None, "scale_a": None, "scale_b": None, "meta": None}

    def words(fmt, stream, kk):
        h = case_hash(xp, seed, stream, idx, kk)
        h2 = case_hash(xp, seed, S_ALT + stream, idx, kk)
        return _format_words(xp, fmt, finite, h, h2)

    if fam == "i8":
        a = case_hash(xp, seed, S_A, idx, 32) & 0xFF
        b = case_hash(xp, seed, S_B, idx, 32) & 0xFF
        c = case_hash(xp, seed, S_C, idx, 1).reshape(-1)
        edges = W._i8_edge_cases(d["a_format"], d["b_format"])
        ea = np.array([e[0] for e in edges], dtype=np.int64)
        eb = np.array([e[1] for e in edges], dtype=np.int64)
        ec = np.array([e[2] for e in edges], dtype=np.int64)
        is_edge = (idx < len(edges)).reshape(-1, 1)
        j = _where(xp, idx < len(edges), idx, 0)
        a = _where(xp, is_edge, _take(xp, ea, j), a)
        b = _where(xp, is_edge, _take(xp, eb, j), b)
        c = _where(xp, is_edge.reshape(-1), _take(xp, ec, j), c)
        out.update(a=a, b=b, c=c)
        return out
    if fam == "dense":
        out.update(a=words(d["a_format"], S_A, k), b=words(d["a_format"], S_B, k), c=_f32_c(xp, seed, idx, finite))
    elif fam == "mixed":
        c = _f16_c(xp, seed, idx, finite) if d["d_type"] == "f16" else _f32_c(xp, seed, idx, finite)
        out.update(a=words(d["a_format"], S_A, k), b=words(d["b_format"], S_B, k), c=c)
    elif fam == "mx":
        out.update(a=words(d["a_format"], S_A, k), b=words(d["a_format"], S_B, k), c=_f32_c(xp, seed, idx, finite),
                   scale_a=_scales(xp, seed, S_SA, idx, 1, "ue8m0", 1), scale_b=_scales(xp, seed, S_SB, idx, 1, "ue8m0", 1))
    elif fam in ("fp4block", "nvfp4"):
        kind = spec.params[0] if spec.params else "mxf4nvf4-4x-ue4m3"
        count = 4 if kind in ("mxf4nvf4-4x", "mxf4nvf4-4x-ue4m3") else 2
        sk = "ue4m3" if kind == "mxf4nvf4-4x-ue4m3" else "ue8m0"
        out.update(a=case_hash(xp, seed, S_A, idx, 64) & 0xF, b=case_hash(xp, seed, S_B, idx, 64) & 0xF,
                   c=_f32_c(xp, seed, idx, finite), scale_a=_scales(xp, seed, S_SA, idx, count, sk),
                   scale_b=_scales(xp, seed, S_SB, idx, count, sk))
    else:  # sparse families
        if fam == "sparse":
            fmt = spec.params[0]
            word_fmt = "e4m3" if fmt == "fp8" else fmt
            mode = "1of2" if fmt == "tf32" else "2of4"
            table = W.SELECTORS_TF32 if fmt == "tf32" else W.SELECTORS_2OF4
            lo = _selectors(xp, seed, S_META, idx, table)
            hi = lo if fmt in ("tf32", "bf16", "f16") else _selectors(xp, seed, S_META + 8, idx, table)
            a, b = words(word_fmt, S_A, k), words(word_fmt, S_B, k)
        elif fam == "sparse-mx":
            mode = "2of4"
            lo = _selectors(xp, seed, S_META, idx, W.SELECTORS_2OF4)
            hi = _selectors(xp, seed, S_META + 8, idx, W.SELECTORS_2OF4)
            a, b = words(d["a_format"], S_A, k), words(d["a_format"], S_B, k)
            out.update(scale_a=_scales(xp, seed, S_SA, idx, 2, "ue8m0"),
                       scale_b=_scales(xp, seed, S_SB, idx, 2, "ue8m0"))
        else:  # sparse-nvfp4, sparse-fp4block: pairwise 4:8 on E2M1
            mode = "4of8"
            lo = _selectors(xp, seed, S_META, idx, W.SELECTORS_2OF4)
            hi = _selectors(xp, seed, S_META + 8, idx, W.SELECTORS_2OF4)
            a, b = case_hash(xp, seed, S_A, idx, k) & 0xF, case_hash(xp, seed, S_B, idx, k) & 0xF
            if fam == "sparse-nvfp4":
                sa = case_hash(xp, seed, S_SA, idx, 4) & 0x7F
                sb = case_hash(xp, seed, S_SB, idx, 4) & 0x7F
            else:
                kind = spec.params[0]
                sk = "ue4m3" if kind == "mxf4nvf4-4x-ue4m3" else "ue8m0"
                sa, sb = _scales(xp, seed, S_SA, idx, 4, sk), _scales(xp, seed, S_SB, idx, 4, sk)
            out.update(scale_a=sa, scale_b=sb)
        meta = (lo.reshape(-1, 1) if xp is np else lo.reshape(-1, 1))
        meta = np.concatenate([meta, hi.reshape(-1, 1)], axis=1) if xp is np else xp.cat([meta, hi.reshape(-1, 1)], 1)
        act = _active(xp, meta, k, mode)
        out.update(a=_where(xp, act, a, 0), b=b, c=_f32_c(xp, seed, idx, finite), meta=meta)
    return out


_SPARSE_MODE = {"1of2": 1, "2of4": 2, "4of8": 3}  # T5E_SPARSE_* of the selection modes


def sparse_mode(spec: W.PathSpec) -> str | None:
    """Selection mode of a sparse path ("1of2", "2of4", "4of8"), None if dense."""
    fam = spec.family
    if fam == "sparse":
        return "1of2" if spec.params[0] == "tf32" else "2of4"
    if fam == "sparse-mx":
        return "2of4"
    if fam in ("sparse-nvfp4", "sparse-fp4block"):
        return "4of8"
    return None


def path_model(spec: W.PathSpec):
    """The arithmetic model of a path (make_model with its descriptor)."""
    from .model import make_model

    d = spec.descriptor
    return make_model(d["a_format"], d["b_format"], d_type=d["d_type"], saturate=d["saturate"],
                      scaling=d["scaling"], scale_vec=d["scale_vec"], kind=d["kind"])


def scale_blocks(spec: W.PathSpec, model=None) -> int:
    """Scale bytes per operand row a case reaches: physical K over the
    model's scale block (0 for unscaled paths)."""
    from . import _native as nat

    desc = (model or path_model(spec)).descriptor()
    if desc.family not in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED):
        return 0
    return -(-_phys_k(spec) // desc.scale_block)


def device_batch(spec: W.PathSpec, start: int, count: int, total: int, device):
    """Cases [start, start + count) of a path with `total` cases, generated on
    `device` (``generate``) and laid out as the kernels read them:
    (model, DeviceBatch).  Sparse A rows hold only the selected elements
    (physical K, T5E_SPARSE_A_COMPRESSED), B rows the logical K; scale rows
    keep the blocks physical K reaches, metadata the words its chunks need.
    The result words equal those of the public API on ``host_cases`` of the
    same range."""
    import torch

    from . import _native as nat
    from . import packing
    from .runtime import DeviceBatch

    model = path_model(spec)
    desc = model.descriptor()
    g = generate(spec, start, count, total, torch, device)
    k = path_k(spec)
    to32 = lambda x: torch.where(x >= 1 << 31, x - (1 << 32), x).to(torch.int32)  # noqa: E731
    a = g["a"]
    mode = sparse_mode(spec)
    sparse = flags = 0
    meta = None
    if mode is not None:
        act = _active(torch, g["meta"], k, mode)
        a = a[act].reshape(count, k // 2)  # every legal record selects exactly half of the logical K
        sparse = _SPARSE_MODE[mode]
        flags = nat.FLAG_SPARSE_A_COMPRESSED
        chunks = k // {"1of2": 2, "2of4": 4, "4of8": 8}[mode]
        meta = to32(g["meta"][:, : -(-chunks // 8)]).contiguous()
    f16 = desc.d_type == nat.D_F16
    c = g["c"] & 0xFFFF if f16 else g["c"]
    c = torch.where(c >= 1 << 15, c - (1 << 16), c).to(torch.int16) if f16 else to32(c)
    db = DeviceBatch(n=count, k=k, a=packing.pack_rows_device(to32(a), desc.a_format),
                     b=packing.pack_rows_device(to32(g["b"]), desc.b_format), c=c.contiguous(),
                     metadata=meta, flags=flags, sparse=sparse)
    blocks = scale_blocks(spec, model)
    if blocks:
        db.scale_a = g["scale_a"][:, :blocks].to(torch.uint8).contiguous()
        db.scale_b = g["scale_b"][:, :blocks].to(torch.uint8).contiguous()
    return model, db


MATRIX_SEED = 92901  # counter-hash seed of the matrix configuration's tile words


def matrix_tiles(first_tile: int, tiles: int, device, m: int = 128, n: int = 256, k: int = 16):
    """Tiles [first_tile, first_tile + tiles) of the matrix configuration
    (BF16 A [m x k] and B [k x n] words, F32 C words, uniformly random
    32-bit patterns, NaN/Inf/subnormals included) on `device` in the
    kernels' layout: (model, DeviceBatch).  Every word is the counter hash of
    its global row or case index, so any split of the tiles over GPUs
    evaluates the same cases.  BF16 rows keep the high half of each word."""
    import torch

    from .model import make_model
    from .runtime import DeviceBatch

    def rows(stream, first, count, words):
        idx = torch.arange(first, first + count, dtype=torch.int64, device=device)
        h = case_hash(torch, MATRIX_SEED, stream, idx, words)
        return torch.where(h >= 1 << 31, h - (1 << 32), h).to(torch.int32)

    a = rows(S_A, first_tile * m, tiles * m, k)        # [rows, k] raw words
    b = rows(S_B, first_tile * n, tiles * n, k)        # [columns, k] raw words (B rows are its columns)
    c = rows(S_C, first_tile * m * n, tiles * m * n, 1).reshape(-1)
    pack = lambda w: (w >> 16).to(torch.int16).view(torch.uint8).reshape(w.shape[0], 2 * k)  # noqa: E731
    db = DeviceBatch(n=tiles * m * n, k=k, a=pack(a).contiguous(), b=pack(b).contiguous(), c=c.contiguous(),
                     tile_m=m, tile_n=n)
    return make_model("bf16"), db


def path_work(spec: W.PathSpec, cases: int, model=None) -> tuple[int, int]:
    """(element-MACs, algorithmic bytes) of `cases` cases of a path.  MACs are
    the physical products; bytes follow the per-path formula: packed A at
    physical K, packed B at logical K, C and D (2 bytes each for F16 D, else
    4), one byte per scale block each operand reaches, half a byte per
    metadata chunk."""
    from . import _native as nat

    model = model or path_model(spec)
    desc = model.descriptor()
    k = path_k(spec)
    kp = _phys_k(spec)
    bits = nat.FORMAT_BITS
    cd = 2 if desc.d_type == nat.D_F16 else 4
    per = -(-kp * bits[desc.a_format] // 8) + -(-k * bits[desc.b_format] // 8) + 2 * cd
    per += 2 * scale_blocks(spec, model)
    mode = sparse_mode(spec)
    if mode is not None:
        per += k // {"1of2": 2, "2of4": 4, "4of8": 8}[mode] // 2
    return cases * kp, cases * per


def host_cases(spec: W.PathSpec, start: int, count: int, total: int) -> W.Cases:
    """The numpy mirror of `generate` as public-API cases (for the oracle)."""
    g = generate(spec, start, count, total, np)
    u32 = lambda x: None if x is None else np.asarray(x, dtype=np.int64).astype(np.uint32)  # noqa: E731
    u8 = lambda x: None if x is None else np.asarray(x, dtype=np.int64).astype(np.uint8)  # noqa: E731
    return W.Cases(spec.descriptor, u32(g["a"]), u32(g["b"]), u32(g["c"]), u8(g["scale_a"]), u8(g["scale_b"]),
                   u32(g["meta"]), name=spec.name)


def result_checksum(xp, idx, words):
    """Order-independent fold of (case index, result word) pairs: the sum of
    a 32-bit hash of each pair."""
    h = _fmix32(_fmix32(idx & MASK32) ^ (words & MASK32))
    return int(h.sum()) if xp is np else int(h.sum().item())


# ------------------------------------------------------------ the sweep


def _device_eval(spec, g, device, generic: bool):
    """Result words (int64 tensor of uint32 values) of generated device cases."""
    import torch

    from . import simulator

    d = spec.descriptor
    kw = {key: d[key] for key in ("a_format", "b_format", "d_type", "saturate", "scaling", "scale_vec", "kind")}
    to32 = lambda x: torch.where(x >= 1 << 31, x - (1 << 32), x).to(torch.int32)  # noqa: E731
    meta = None if g["meta"] is None else to32(g["meta"])
    sa = None if g["scale_a"] is None else g["scale_a"].to(torch.uint8)
    sb = None if g["scale_b"] is None else g["scale_b"].to(torch.uint8)
    res = simulator.mma_dot_batch(to32(g["a"]), to32(g["b"]), to32(g["c"]), scale_a=sa, scale_b=sb,
                                  sparse_metadata=meta, device=device, check=True, generic=generic, **kw)
    return res.view(torch.int32).to(torch.int64) & MASK32


def _evaluate_shard_gpu(spec, lo: int, hi: int, total: int, device, chunk: int):
    """(cases, mismatches, checksum, seconds) of cases [lo, hi) on this rank's
    GPU; seconds is the device time of the evaluations through the
    dispatching entry point (packing of the generated words included)."""
    import torch

    cases = mism = chk = 0
    ms = 0.0
    for s0 in range(lo, hi, chunk):
        s1 = min(hi, s0 + chunk)
        g = generate(spec, s0, s1 - s0, total, torch, device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fast = _device_eval(spec, g, device, generic=False)
        e1.record()
        slow = _device_eval(spec, g, device, generic=True)
        mism += int((fast != slow).sum().item())
        idx = torch.arange(s0, s1, dtype=torch.int64, device=device)
        chk += result_checksum(torch, idx, fast)
        cases += s1 - s0
        ms += e0.elapsed_time(e1)
    return cases, mism, chk, ms / 1e3


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous share [lo, hi) of `total` cases for `rank` of `world`."""
    return total * rank // world, total * (rank + 1) // world


def integrity(requested: list[str], results: list[dict]) -> tuple[list[str], list[str]]:
    """(failed paths, integrity errors): missing, duplicate and unexpected
    paths, as run_full_validation.py:359-379 checks them."""
    counts = Counter(r["path"] for r in results)
    missing = sorted(set(requested) - set(counts))
    duplicate = sorted(p for p, c in counts.items() if c != 1)
    unexpected = sorted(set(counts) - set(requested))
    errors = []
    if missing:
        errors.append(f"missing paths: {', '.join(missing)}")
    if duplicate:
        errors.append(f"duplicate paths: {', '.join(duplicate)}")
    if unexpected:
        errors.append(f"unexpected paths: {', '.join(unexpected)}")
    failed = sorted({r["path"] for r in results if r["failed"]} | set(missing))
    return failed, errors


def run_sweep(cases_per_path: int, *, paths=None, rank: int = 0, world: int = 1, device=None, chunk: int = 1 << 18,
              evaluate=None, group=None) -> dict:
    """Evaluate this rank's share of every path and sum the per-path counters
    over the ranks (torch.distributed, when world > 1).  ``evaluate(spec, lo,
    hi, total)`` -> (cases, mismatches, checksum) defaults to the GPU
    evaluation; every rank returns the same report."""
    import torch

    paths = list(W.validation_paths() if paths is None else paths)
    if evaluate is None:
        def evaluate(spec, lo, hi, total):
            return _evaluate_shard_gpu(spec, lo, hi, total, device, chunk)
    t0 = time.perf_counter()
    counters = torch.zeros((len(paths), 3), dtype=torch.int64)
    kernel_s = 0.0
    for p, spec in enumerate(paths):
        lo, hi = shard(cases_per_path, rank, world)
        res = evaluate(spec, lo, hi, cases_per_path)
        counters[p, 0] = res[0]
        counters[p, 1] = res[1]
        counters[p, 2] = res[2]  # below 2**63: at most 2**31 cases of 32-bit hashes
        kernel_s += res[3] if len(res) > 3 else 0.0
    elapsed = torch.tensor([time.perf_counter() - t0, kernel_s], dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        backend = dist.get_backend(group)
        dev = device if backend == "nccl" else torch.device("cpu")
        c = counters.to(dev)
        e = elapsed.to(dev)
        dist.all_reduce(c, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(e, op=dist.ReduceOp.MAX, group=group)
        counters, elapsed = c.cpu(), e.cpu()
    results = []
    for p, spec in enumerate(paths):
        cases, mism, chk = (int(v) for v in counters[p])
        results.append({"path": spec.name, "cases": cases, "mismatches": mism, "position_failures": 0,
                        "checksum": f"{chk & 0xFFFFFFFFFFFFFFFF:016x}",
                        "failed": mism != 0 or cases != cases_per_path})
    failed, errors = integrity([s.name for s in paths], results)
    macs = sum(r["cases"] * _phys_k(s) for r, s in zip(results, paths))
    seconds = float(elapsed[0])
    kernel_seconds = float(elapsed[1])
    return {
        "generated_at": datetime.now(timezone.utc).isoformat(),
        "cases_per_path": cases_per_path,
        "requested_path_count": len(paths),
        "path_count": len(results),
        "total_cases": sum(r["cases"] for r in results),
        "devices": world,
        "failed_paths": failed,
        "integrity_errors": errors,
        "results": results,
        "elapsed_s": seconds,
        "element_macs": macs,
        "element_macs_per_s": macs / seconds if seconds > 0 else None,
        "kernel_seconds_max_rank": kernel_seconds,
        "kernel_element_macs_per_s": macs / kernel_seconds if kernel_seconds > 0 else None,
    }


def _phys_k(spec: W.PathSpec) -> int:
    """Products formed per case: K, halved for the sparse paths."""
    k = path_k(spec)
    return k // 2 if spec.family.startswith("sparse") else k


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="46-path sweep of the tcgen05 emulator")
    ap.add_argument("--cases-per-path", type=int, default=1_000_000)
    ap.add_argument("--chunk", type=int, default=1 << 18)
    ap.add_argument("--paths", default=None, help="comma-separated subset of path names")
    ap.add_argument("--output", default=None)
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    paths = W.validation_paths()
    if args.paths:
        wanted = set(args.paths.split(","))
        paths = [p for p in paths if p.name in wanted]
    report = run_sweep(args.cases_per_path, paths=paths, rank=rank, world=world, device=device, chunk=args.chunk)
    if rank == 0:
        text = json.dumps(report, indent=2, sort_keys=True)
        if args.output:
            with open(args.output, "w") as f:
                f.write(text + "\n")
        print(f"SUMMARY paths={report['path_count']} cases={report['total_cases']} "
              f"failed={len(report['failed_paths'])} devices={world} seconds={report['elapsed_s']:.3f} "
              f"element_macs_per_s={report['element_macs_per_s']:.4g} "
              f"kernel_element_macs_per_s={report['kernel_element_macs_per_s'] or 0:.4g}", flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 1 if report["failed_paths"] or report["integrity_errors"] else 0


if __name__ == "__main__":
    sys.exit(main())

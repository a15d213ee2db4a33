"""Seeded synthetic inputs: the reference's 46 hardware-validation paths and
the benchmark configurations.

The 46 paths follow the reference manifest
(hardware_validation/run_full_validation.py:43-224) and the input
distributions of its case generators (hardware_validation/mma_probe.py):
raw words, a finite-only half, random UE8M0/UE4M3 scales over their whole
encoding (NaN included) and random legal sparse metadata.  Inputs come from
numpy's PCG64 instead of Python's Mersenne Twister, so the cases are new
draws from the same distributions.  Every case is expressed through the
public ``mma_dot`` arguments (logical-K words, scale tuples, metadata).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SELECTORS_TF32 = np.array([0x4, 0xE], dtype=np.uint32)
SELECTORS_2OF4 = np.array([0x4, 0x8, 0xC, 0x9, 0xD, 0x6, 0xE], dtype=np.uint32)
# the six distinct 2-of-4 patterns (0x6 and 0x9 select the same pair)
SELECTORS_SIX = np.array([0x4, 0x8, 0xC, 0x9, 0xD, 0xE], dtype=np.uint32)


# --------------------------------------------------------------- words


def f32_words(rng, n, finite_only=False):
    """mma_probe.py:258-262: uniform 32-bit words; finite-only redraws the
    exponent of an Inf/NaN word uniformly in 0..254."""
    w = rng.integers(0, 1 << 32, size=n, dtype=np.uint64).astype(np.uint32)
    if finite_only:
        bad = (w & 0x7F800000) == 0x7F800000
        e = rng.integers(0, 255, size=n, dtype=np.uint32)
        w = np.where(bad, (w & 0x807FFFFF) | (e << 23), w)
    return w.astype(np.uint32)


def f16_words(rng, n, finite_only=False):
    """mma_probe.py:799-803."""
    w = rng.integers(0, 1 << 16, size=n, dtype=np.uint32)
    if finite_only:
        bad = ((w >> 10) & 0x1F) == 0x1F
        e = rng.integers(0, 0x1F, size=n, dtype=np.uint32)
        w = np.where(bad, (w & ~np.uint32(0x1F << 10)) | (e << 10), w)
    return w.astype(np.uint32)


def e4m3_words(rng, n, finite_only=False):
    """mma_probe.py:895-899."""
    w = rng.integers(0, 256, size=n, dtype=np.uint32)
    if finite_only:
        bad = (w & 0x7F) == 0x7F
        r = rng.integers(0, 0x7F, size=n, dtype=np.uint32)
        w = np.where(bad, (w & 0x80) | r, w)
    return w.astype(np.uint32)


def e5m2_words(rng, n, finite_only=False):
    """mma_probe.py:994-998."""
    w = rng.integers(0, 256, size=n, dtype=np.uint32)
    if finite_only:
        bad = ((w >> 2) & 0x1F) == 0x1F
        e = rng.integers(0, 0x1F, size=n, dtype=np.uint32)
        w = np.where(bad, (w & ~np.uint32(0x1F << 2)) | (e << 2), w)
    return w.astype(np.uint32)


def format_words(fmt, rng, n, finite_only=False):
    """Random container words of a format (mma_probe.py:991-1003, :1291-1300)."""
    if fmt in ("tf32", "bf16"):
        return f32_words(rng, n, finite_only)
    if fmt == "f16":
        return f16_words(rng, n, finite_only)
    if fmt == "e4m3":
        return e4m3_words(rng, n, finite_only)
    if fmt == "e5m2":
        return e5m2_words(rng, n, finite_only)
    if fmt in ("e2m3", "e3m2"):
        return rng.integers(0, 64, size=n, dtype=np.uint32)
    if fmt == "e2m1":
        return rng.integers(0, 16, size=n, dtype=np.uint32)
    if fmt in ("u8", "s8"):
        return rng.integers(0, 256, size=n, dtype=np.uint32)
    raise ValueError(fmt)


def metadata_words(rng, n, selectors):
    """n uint32 words of eight uniformly chosen selectors (mma_probe.py:2734-2759)."""
    picks = selectors[rng.integers(0, len(selectors), size=(n, 8))]
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, :]
    return np.bitwise_or.reduce(picks << shifts, axis=1).astype(np.uint32)


def active_mask(meta, k, mode):
    """[n, k] boolean map of the selected logical positions for metadata
    records [n, W] (the reference's sparse_active_indices, vectorised)."""
    n = meta.shape[0]
    csize = {"1of2": 2, "2of4": 4, "4of8": 8}[mode]
    chunks = (k + csize - 1) // csize
    mask = np.zeros((n, chunks * csize), dtype=bool)
    rows = np.arange(n)
    for c in range(chunks):
        sel = (meta[:, c // 8] >> np.uint32((c & 7) * 4)) & 0xF
        if mode == "1of2":
            mask[rows, 2 * c + (sel == 0xE)] = True
            continue
        f = (sel & 3).astype(np.int64)
        g = ((sel >> 2) & 3).astype(np.int64)
        if mode == "2of4":
            mask[rows, 4 * c + f] = True
            mask[rows, 4 * c + g] = True
        else:
            for p in (f, g):
                mask[rows, 8 * c + 2 * p] = True
                mask[rows, 8 * c + 2 * p + 1] = True
    return mask[:, :k]


# --------------------------------------------------------------- cases


@dataclass
class Cases:
    """A batch of cases in public-API form plus the descriptor keywords."""

    desc: dict
    a: np.ndarray                 # [n, k] uint32 logical words
    b: np.ndarray
    c: np.ndarray                 # [n] uint32
    scale_a: np.ndarray | None = None   # [n, ns] uint8
    scale_b: np.ndarray | None = None
    meta: np.ndarray | None = None      # [n, W] uint32
    name: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def n(self):
        return self.a.shape[0]

    @property
    def k(self):
        return self.a.shape[1]

    def concat(self, other: "Cases") -> "Cases":
        def cat(x, y):
            return None if x is None else np.concatenate([x, y])

        return Cases(self.desc, cat(self.a, other.a), cat(self.b, other.b), cat(self.c, other.c),
                     cat(self.scale_a, other.scale_a), cat(self.scale_b, other.scale_b), cat(self.meta, other.meta),
                     self.name)

    def subset(self, idx) -> "Cases":
        def take(x):
            return None if x is None else x[idx]

        return Cases(self.desc, take(self.a), take(self.b), take(self.c), take(self.scale_a), take(self.scale_b),
                     take(self.meta), self.name)

    def digest(self) -> str:
        import hashlib

        h = hashlib.sha256()
        for x in (self.a, self.b, self.c, self.scale_a, self.scale_b, self.meta):
            h.update(b"-" if x is None else np.ascontiguousarray(x).tobytes())
        return h.hexdigest()


def _scales(rng, n, count, kind):
    """_scale_tuple (mma_probe.py:2243-2255): `count` random scales, the rest
    of four unit scales."""
    unit, hi = (0x38, 0x80) if kind == "ue4m3" else (0x7F, 0x100)
    s = np.full((n, 4), unit, dtype=np.uint8)
    s[:, :count] = rng.integers(0, hi, size=(n, count), dtype=np.uint32).astype(np.uint8)
    return s


def _i8_edge_cases(a_type, b_type):
    """mma_probe.py:1117-1139."""
    pos_a = 0x7F if a_type == "s8" else 0xFF
    pos_b = 0x7F if b_type == "s8" else 0xFF
    neg_a = 0x80 if a_type == "s8" else None
    neg_b = 0x80 if b_type == "s8" else None
    cases = [((0,) * 32, (0,) * 32, 0), ((1,) * 32, (1,) * 32, 0), ((pos_a,) * 32, (pos_b,) * 32, 0),
             ((pos_a,) * 32, (pos_b,) * 32, 0x7FFF_FFF0), ((pos_a,) * 32, (pos_b,) * 32, 0x8000_0010)]
    if neg_a is not None:
        cases.append(((neg_a,) * 32, (pos_b,) * 32, 0x8000_0010))
        cases.append(((pos_a,) * 16 + (neg_a,) * 16, (pos_b,) * 32, 0x7FFF_FFF0))
    if neg_b is not None:
        cases.append(((pos_a,) * 32, (neg_b,) * 32, 0x8000_0010))
        cases.append(((pos_a,) * 32, (pos_b,) * 16 + (neg_b,) * 16, 0x7FFF_FFF0))
    return cases


@dataclass(frozen=True)
class PathSpec:
    name: str
    family: str
    desc: tuple
    seed: int
    params: tuple = ()

    @property
    def descriptor(self) -> dict:
        return dict(self.desc)


def _spec(name, family, seed, params=(), **desc):
    full = dict(a_format="tf32", b_format=None, d_type="f32", saturate=False, scaling=None, scale_vec=None, kind=None)
    full.update(desc)
    return PathSpec(name, family, tuple(sorted(full.items())), seed, tuple(params))


def validation_paths() -> tuple[PathSpec, ...]:
    """The 46 named paths, seeds as in run_full_validation.py:57-221."""
    p = []
    dense = [("dense-tf32", "tf32"), ("dense-bf16", "bf16"), ("dense-f16", "f16"), ("dense-e4m3", "e4m3"),
             ("dense-e5m2", "e5m2"), ("dense-e2m3", "e2m3"), ("dense-e3m2", "e3m2"), ("dense-e2m1", "e2m1")]
    for i, (name, fmt) in enumerate(dense):
        p.append(_spec(name, "dense", 92101 + 2 * i, a_format=fmt))
    seed = 92201
    for saturate in (False, True):
        for at, bt in (("u8", "u8"), ("s8", "u8"), ("u8", "s8"), ("s8", "s8")):
            p.append(_spec(f"i8-{at}-{bt}-{'saturate' if saturate else 'wrap'}", "i8", seed,
                           a_format=at, b_format=bt, d_type="s32", saturate=saturate))
            seed += 1
    seed = 92301
    for fmt in ("e4m3", "e5m2", "e2m3", "e3m2", "e2m1"):
        p.append(_spec(f"dense-mx-{fmt}", "mx", seed, a_format=fmt, scaling="ue8m0", kind="mxf8f6f4", scale_vec=1))
        seed += 2
    for kind in ("mxf4", "mxf4nvf4-2x", "mxf4nvf4-4x", "mxf4nvf4-4x-ue4m3"):
        p.append(_spec(f"dense-{kind}", "fp4block", seed, (kind,), **_fp4_desc(kind)))
        seed += 2
    for fmt, fseed in (("tf32", 92401), ("bf16", 92403), ("f16", 92405), ("fp8", 92407), ("e5m2", 92409),
                       ("e2m3", 92501), ("e3m2", 92503), ("e2m1", 92505)):
        p.append(_spec(f"sparse-{fmt}", "sparse", fseed, (fmt,), a_format="e4m3" if fmt == "fp8" else fmt))
    p.append(_spec("sparse-nvfp4", "sparse-nvfp4", 92507, (), a_format="e2m1", scaling="ue4m3", scale_vec=4))
    seed = 92601
    for fmt in ("e4m3", "e5m2", "e2m3", "e3m2", "e2m1"):
        p.append(_spec(f"sparse-mx-{fmt}", "sparse-mx", seed, a_format=fmt, scaling="ue8m0", kind="mxf8f6f4",
                       scale_vec=1))
        seed += 2
    for kind in ("mxf4", "mxf4nvf4-2x", "mxf4nvf4-4x", "mxf4nvf4-4x-ue4m3"):
        p.append(_spec(f"sparse-{kind}", "sparse-fp4block", seed, (kind,), **_fp4_desc(kind)))
        seed += 2
    p.append(_spec("mixed-e4m3-e2m1-f32", "mixed", 92703, a_format="e4m3", b_format="e2m1", d_type="f32"))
    p.append(_spec("mixed-e2m1-e4m3-f16", "mixed", 92705, a_format="e2m1", b_format="e4m3", d_type="f16"))
    p.append(_spec("dense-nvfp4", "nvfp4", 92801, a_format="e2m1", scaling="ue4m3", scale_vec=4))
    assert len(p) == 46
    return tuple(p)


def _fp4_desc(kind):
    if kind == "mxf4":
        return dict(a_format="e2m1", scaling="ue8m0", kind="mxf4", scale_vec=2)
    if kind == "mxf4nvf4-2x":
        return dict(a_format="e2m1", scaling="ue8m0", kind="mxf4nvf4", scale_vec=2)
    if kind == "mxf4nvf4-4x":
        return dict(a_format="e2m1", scaling="ue8m0", kind="mxf4nvf4", scale_vec=4)
    return dict(a_format="e2m1", scaling="ue4m3", kind="mxf4nvf4", scale_vec=4)


def _half(spec: PathSpec, rng, n: int, finite: bool) -> Cases:
    d = spec.descriptor
    fam = spec.family
    if fam == "dense":
        fmt = d["a_format"]
        k = {"tf32": 8, "bf16": 16, "f16": 16}.get(fmt, 32)
        a = format_words(fmt, rng, n * k, finite).reshape(n, k)
        b = format_words(fmt, rng, n * k, finite).reshape(n, k)
        return Cases(d, a, b, f32_words(rng, n, finite))
    if fam == "mixed":
        k = 32
        a = format_words(d["a_format"], rng, n * k, finite).reshape(n, k)
        b = format_words(d["b_format"], rng, n * k, finite).reshape(n, k)
        c = f16_words(rng, n, finite) if d["d_type"] == "f16" else f32_words(rng, n, finite)
        return Cases(d, a, b, c)
    if fam == "mx":
        fmt = d["a_format"]
        a = format_words(fmt, rng, n * 32, finite).reshape(n, 32)
        b = format_words(fmt, rng, n * 32, finite).reshape(n, 32)
        c = f32_words(rng, n, finite)
        return Cases(d, a, b, c, _scales(rng, n, 1, "ue8m0")[:, :1], _scales(rng, n, 1, "ue8m0")[:, :1])
    if fam in ("fp4block", "nvfp4"):
        kind = spec.params[0] if spec.params else "mxf4nvf4-4x-ue4m3"
        count = 4 if kind in ("mxf4nvf4-4x", "mxf4nvf4-4x-ue4m3") else 2
        sk = "ue4m3" if kind == "mxf4nvf4-4x-ue4m3" else "ue8m0"
        a = rng.integers(0, 16, size=(n, 64), dtype=np.uint32)
        b = rng.integers(0, 16, size=(n, 64), dtype=np.uint32)
        c = f32_words(rng, n, finite)
        return Cases(d, a, b, c, _scales(rng, n, count, sk), _scales(rng, n, count, sk))
    if fam == "sparse":
        fmt = spec.params[0]
        word_fmt = "e4m3" if fmt == "fp8" else fmt
        k = {"tf32": 16, "bf16": 32, "f16": 32}.get(fmt, 64)
        mode = "1of2" if fmt == "tf32" else "2of4"
        sel = SELECTORS_TF32 if fmt == "tf32" else SELECTORS_2OF4
        lo = metadata_words(rng, n, sel)
        hi = metadata_words(rng, n, sel) if fmt not in ("tf32", "bf16", "f16") else lo
        meta = np.stack([lo, hi], axis=1)
        act = active_mask(meta, k, mode)
        a = np.where(act, format_words(word_fmt, rng, n * k, finite).reshape(n, k), 0).astype(np.uint32)
        b = format_words(word_fmt, rng, n * k, finite).reshape(n, k)
        return Cases(d, a, b, f32_words(rng, n, finite), meta=meta)
    if fam == "sparse-nvfp4":
        lo = metadata_words(rng, n, SELECTORS_2OF4)
        hi = metadata_words(rng, n, SELECTORS_2OF4)
        meta = np.stack([lo, hi], axis=1)
        act = active_mask(meta, 128, "4of8")
        a = np.where(act, rng.integers(0, 16, size=(n, 128), dtype=np.uint32), 0).astype(np.uint32)
        b = rng.integers(0, 16, size=(n, 128), dtype=np.uint32)
        sa = rng.integers(0, 0x80, size=(n, 4), dtype=np.uint32).astype(np.uint8)
        sb = rng.integers(0, 0x80, size=(n, 4), dtype=np.uint32).astype(np.uint8)
        return Cases(d, a, b, f32_words(rng, n, finite), sa, sb, meta)
    if fam == "sparse-mx":
        fmt = d["a_format"]
        lo = metadata_words(rng, n, SELECTORS_2OF4)
        hi = metadata_words(rng, n, SELECTORS_2OF4)
        meta = np.stack([lo, hi], axis=1)
        act = active_mask(meta, 64, "2of4")
        a = np.where(act, format_words(fmt, rng, n * 64, finite).reshape(n, 64), 0).astype(np.uint32)
        b = format_words(fmt, rng, n * 64, finite).reshape(n, 64)
        c = f32_words(rng, n, finite)
        return Cases(d, a, b, c, _scales(rng, n, 2, "ue8m0"), _scales(rng, n, 2, "ue8m0"), meta)
    if fam == "sparse-fp4block":
        kind = spec.params[0]
        sk = "ue4m3" if kind == "mxf4nvf4-4x-ue4m3" else "ue8m0"
        lo = metadata_words(rng, n, SELECTORS_2OF4)
        hi = metadata_words(rng, n, SELECTORS_2OF4)
        meta = np.stack([lo, hi], axis=1)
        act = active_mask(meta, 128, "4of8")
        a = np.where(act, rng.integers(0, 16, size=(n, 128), dtype=np.uint32), 0).astype(np.uint32)
        b = rng.integers(0, 16, size=(n, 128), dtype=np.uint32)
        c = f32_words(rng, n, finite)
        return Cases(d, a, b, c, _scales(rng, n, 4, sk), _scales(rng, n, 4, sk), meta)
    raise ValueError(fam)


def path_cases(spec: PathSpec, n: int, seed: int | None = None) -> Cases:
    """n cases of a validation path: a raw half then a finite-only half
    (run_full_validation.py:33-40); integer paths start with the reference's
    edge cases (mma_probe.py:1117-1139) and draw C as a raw 32-bit word."""
    seed = spec.seed if seed is None else seed
    if spec.family == "i8":
        d = spec.descriptor
        rng = np.random.Generator(np.random.PCG64(seed))
        edges = _i8_edge_cases(d["a_format"], d["b_format"])[:n]
        m = n - len(edges)
        a = rng.integers(0, 256, size=(m, 32), dtype=np.uint32)
        b = rng.integers(0, 256, size=(m, 32), dtype=np.uint32)
        c = rng.integers(0, 1 << 32, size=m, dtype=np.uint64).astype(np.uint32)
        if edges:
            a = np.concatenate([np.array([e[0] for e in edges], dtype=np.uint32), a])
            b = np.concatenate([np.array([e[1] for e in edges], dtype=np.uint32), b])
            c = np.concatenate([np.array([e[2] for e in edges], dtype=np.uint32), c])
        out = Cases(d, a, b, c)
        out.name = spec.name
        return out
    raw = n // 2
    first = _half(spec, np.random.Generator(np.random.PCG64(seed)), raw, False)
    second = _half(spec, np.random.Generator(np.random.PCG64(seed + 1)), n - raw, True)
    out = first.concat(second)
    out.name = spec.name
    return out


# ------------------------------------------------------- bench configs


def finite_f32_c(rng, n):
    """F32 C words with the biased exponent uniform in [100, 154], sign and
    fraction uniform (the E4M3 x E5M2 configuration's C)."""
    sign = rng.integers(0, 2, size=n, dtype=np.uint32) << 31
    exp = rng.integers(100, 155, size=n, dtype=np.uint32) << 23
    frac = rng.integers(0, 1 << 23, size=n, dtype=np.uint32)
    return (sign | exp | frac).astype(np.uint32)


def finite_f16_c(rng, n):
    """F16 C words with the biased exponent uniform in [1, 30] (finite,
    normal), sign and fraction uniform."""
    sign = rng.integers(0, 2, size=n, dtype=np.uint32) << 15
    exp = rng.integers(1, 31, size=n, dtype=np.uint32) << 10
    frac = rng.integers(0, 1 << 10, size=n, dtype=np.uint32)
    return (sign | exp | frac).astype(np.uint32)


# ------------------------------------------------- regime-boundary cases
#
# Inputs aimed at the places where the scaled E2M1 models switch regime:
# C's raw exponent near the largest product raw exponent (the NVFP4
# C-dominant / product-dominant split, model.py:780-796, and the MXF4
# family's per-group C-dominant windows, model.py:964-981), groups whose
# scales sit around the 33-34 binades where their sums start to truncate,
# results in the subnormal range below the 2**-174 group floor
# (model.py:986-1003), and NaN scales in reached and unreached blocks.

BOUNDARY_KINDS = ("mxf4", "mxf4nvf4-2x", "mxf4nvf4-4x", "nvfp4")
_SCALE_OFFSETS = np.array([0, 0, -1, -2, -3, -4, -5, -10, -20, -30, -32, -33, -34, -35, -36, -40, -60],
                          dtype=np.int64)


def _boundary_c(rng, n, c_raw):
    """F32 C words with raw exponent c_raw (clipped to the F32 range), random
    sign and fraction; about 12% zero or -0, 4% subnormal, 2% infinite and
    1% NaN."""
    c_raw = np.clip(c_raw, -126, 127)
    sign = rng.integers(0, 2, size=n, dtype=np.uint64).astype(np.uint32) << np.uint32(31)
    frac = rng.integers(0, 1 << 23, size=n, dtype=np.uint64).astype(np.uint32)
    c = sign | ((c_raw + 127).astype(np.uint32) << np.uint32(23)) | frac
    u = rng.random(n)
    c = np.where(u < 0.09, 0, c)
    c = np.where((u >= 0.09) & (u < 0.12), 0x80000000, c)
    c = np.where((u >= 0.12) & (u < 0.16), sign | (frac | 1), c)
    c = np.where((u >= 0.16) & (u < 0.18), sign | 0x7F800000, c)
    c = np.where((u >= 0.18) & (u < 0.19), 0x7FC00000 | (frac & 0x3FFFFF), c)
    return c.astype(np.uint32)


def boundary_cases(kind: str, n: int, seed: int = 0, *, sparse: bool = False, floor: bool = False) -> Cases:
    """Regime-boundary cases of a scaled E2M1 descriptor: ``kind`` is one of
    BOUNDARY_KINDS (UE8M0 MXF4 2X, MXF4NVF4 2X/4X, or NVFP4 with UE4M3
    scales); K = 64 dense, or logical K = 128 with pairwise 4:8 metadata.
    ``floor`` draws small UE8M0 scales, so that the product window lies
    below 2**-174 and many results are subnormal."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nvfp4 = kind == "nvfp4"
    desc = (dict(a_format="e2m1", scaling="ue4m3", scale_vec=4) if nvfp4
            else _fp4_desc(kind))
    block = 16 if (nvfp4 or kind == "mxf4nvf4-4x") else 32
    blocks = 64 // block
    k = 128 if sparse else 64
    # elements: uniform nibbles, with about one group in six entirely zero
    a = rng.integers(0, 16, size=(n, 64), dtype=np.uint32)
    b = rng.integers(0, 16, size=(n, 64), dtype=np.uint32)
    zero_group = rng.random((n, 4)) < 0.17
    a = np.where(np.repeat(zero_group, 16, axis=1), a & 0x8, a)
    if nvfp4:
        # UE4M3 exponent fields e in 0..15 (raw exponent max(e, 1) - 7; e = 0
        # is subnormal, a zero mantissa there a zero scale), mantissa random
        base = rng.integers(0, 16, size=(n, 1), dtype=np.int64)
        ea = np.clip(base + rng.integers(-3, 1, size=(n, 4)), 0, 15)
        eb = np.clip(base + rng.integers(-3, 1, size=(n, 4)), 0, 15)
        sa = ((ea << 3) | rng.integers(0, 8, size=(n, 4))).astype(np.int64)
        sb = ((eb << 3) | rng.integers(0, 8, size=(n, 4))).astype(np.int64)
        sa = np.where(sa == 0x7F, 0x7E, sa)
        sb = np.where(sb == 0x7F, 0x7E, sb)
        sr = (np.maximum(ea, 1) - 7) + (np.maximum(eb, 1) - 7)
    else:
        lo, hi = (10, 60) if floor else (45, 215)
        base = rng.integers(lo, hi, size=(n, 1), dtype=np.int64)
        sa = np.clip(base + _SCALE_OFFSETS[rng.integers(0, _SCALE_OFFSETS.size, size=(n, 4))], 0, 254)
        sb = np.clip(base + _SCALE_OFFSETS[rng.integers(0, _SCALE_OFFSETS.size, size=(n, 4))], 0, 254)
        sr = (sa - 127) + (sb - 127)
    # C relative to a random group's scale exponent: the band [SR_g, SR_g + 4]
    # and a few binades either side
    g = rng.integers(0, 4, size=n)
    group_sr = sr[np.arange(n), (g * 16) // block]
    c = _boundary_c(rng, n, group_sr + rng.integers(-3, 8, size=n))
    if floor:
        c = np.where(rng.random(n) < 0.5, _boundary_c(rng, n, np.full(n, -126)) & 0x807FFFFF, c).astype(np.uint32)
    # NaN scales: 1% in a reached block; unreached trailing blocks hold
    # anything (they are never read)
    nan_byte = 0x7F if nvfp4 else 0xFF
    hit = rng.random((n, 4)) < 0.005
    sa = np.where(hit & (np.arange(4) < blocks), nan_byte, sa)
    if blocks < 4:
        sa[:, blocks:] = rng.integers(0, 256, size=(n, 4 - blocks))
        sb[:, blocks:] = rng.integers(0, 256, size=(n, 4 - blocks))
    scale_a = sa.astype(np.uint8)
    scale_b = sb.astype(np.uint8)
    meta = None
    if sparse:
        lo_w = metadata_words(rng, n, SELECTORS_2OF4)
        hi_w = metadata_words(rng, n, SELECTORS_2OF4)
        meta = np.stack([lo_w, hi_w], axis=1)
        act = active_mask(meta, 128, "4of8")
        la = np.zeros((n, 128), dtype=np.uint32)
        lb = rng.integers(0, 16, size=(n, 128), dtype=np.uint32)
        la[act] = a.reshape(-1)
        lb[act] = b.reshape(-1)
        a, b = la, lb
    name = ("sparse-" if sparse else "") + kind + ("-floor" if floor else "-band")
    return Cases(desc, a.astype(np.uint32), b.astype(np.uint32), c, scale_a, scale_b, meta, name=name)


# (kind, sparse, floor) of every boundary set the fixtures and tests use
BOUNDARY_SETS = tuple((kind, sparse, floor) for kind in BOUNDARY_KINDS for sparse in (False, True)
                      for floor in ((False, True) if kind != "nvfp4" else (False,)))


def config_cases(name: str, n: int, seed: int = 0) -> Cases:
    """Public-API cases of a benchmark configuration."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if name == "tf32-k8":
        return Cases(dict(a_format="tf32"), f32_words(rng, n * 8).reshape(n, 8), f32_words(rng, n * 8).reshape(n, 8),
                     f32_words(rng, n), name=name)
    if name in ("e4m3xe5m2-k32", "e4m3xe5m2-k32-f16"):
        f16 = name.endswith("f16")
        a = rng.integers(0, 256, size=(n, 32), dtype=np.uint32)
        b = rng.integers(0, 256, size=(n, 32), dtype=np.uint32)
        c = finite_f16_c(rng, n) if f16 else finite_f32_c(rng, n)
        return Cases(dict(a_format="e4m3", b_format="e5m2", d_type="f16" if f16 else "f32"), a, b, c, name=name)
    if name == "mx-e2m3xe3m2-k32":
        a = rng.integers(0, 64, size=(n, 32), dtype=np.uint32)
        b = rng.integers(0, 64, size=(n, 32), dtype=np.uint32)
        sa = rng.integers(0x70, 0x90, size=(n, 1), dtype=np.uint32).astype(np.uint8)
        sb = rng.integers(0x70, 0x90, size=(n, 1), dtype=np.uint32).astype(np.uint8)
        return Cases(dict(a_format="e2m3", b_format="e3m2", scaling="ue8m0", kind="mxf8f6f4"), a, b,
                     finite_f32_c(rng, n), sa, sb, name=name)
    if name in ("u8xs8-k32-sat", "u8xs8-k32-wrap"):
        a = rng.integers(0, 256, size=(n, 32), dtype=np.uint32)
        b = rng.integers(0, 256, size=(n, 32), dtype=np.uint32)
        u = rng.integers(0, 1 << 21, size=n, dtype=np.uint32)
        top = rng.integers(0, 2, size=n, dtype=np.uint32).astype(bool)
        c = np.where(top, np.uint32(0x7FFFFFFF) - u, np.uint32(0x80000000) + u).astype(np.uint32)
        return Cases(dict(a_format="u8", b_format="s8", d_type="s32", saturate=name.endswith("sat")), a, b, c,
                     name=name)
    if name == "nvfp4-k64":
        a = rng.integers(0, 16, size=(n, 64), dtype=np.uint32)
        b = rng.integers(0, 16, size=(n, 64), dtype=np.uint32)
        sa = rng.integers(0x01, 0x7F, size=(n, 4), dtype=np.uint32).astype(np.uint8)
        sb = rng.integers(0x01, 0x7F, size=(n, 4), dtype=np.uint32).astype(np.uint8)
        return Cases(dict(a_format="e2m1", scaling="ue4m3", scale_vec=4), a, b, finite_f32_c(rng, n), sa, sb,
                     name=name)
    if name == "nvfp4-sparse-k128":
        lo = metadata_words(rng, n, SELECTORS_SIX)
        hi = metadata_words(rng, n, SELECTORS_SIX)
        meta = np.stack([lo, hi], axis=1)
        act = active_mask(meta, 128, "4of8")
        a = np.where(act, rng.integers(0, 16, size=(n, 128), dtype=np.uint32), 0).astype(np.uint32)
        b = rng.integers(0, 16, size=(n, 128), dtype=np.uint32)
        sa = rng.integers(0x01, 0x7F, size=(n, 4), dtype=np.uint32).astype(np.uint8)
        sb = rng.integers(0x01, 0x7F, size=(n, 4), dtype=np.uint32).astype(np.uint8)
        return Cases(dict(a_format="e2m1", scaling="ue4m3", scale_vec=4), a, b, finite_f32_c(rng, n), sa, sb, meta,
                     name=name)
    raise ValueError(f"unknown configuration {name!r}")


# ------------------------------------------- configurations generated on the GPU

# Cases per configuration at the sizes the benchmark configurations state.
CONFIG_SIZES = {
    "tf32-k8": 65536,
    "e4m3xe5m2-k32": 1 << 20,
    "e4m3xe5m2-k32-f16": 1 << 20,
    "mx-e2m3xe3m2-k32": 1 << 22,
    "u8xs8-k32-sat": 1 << 22,
    "u8xs8-k32-wrap": 1 << 22,
    "nvfp4-k64": 1 << 24,
    "nvfp4-sparse-k128": 1 << 24,
    "matrix-bf16": 4096 * 128 * 256,
}


def _device_bytes(torch, gen, device, shape):
    return torch.randint(0, 256, shape, dtype=torch.uint8, device=device, generator=gen)


def _device_finite_c(torch, gen, device, n, f16=False):
    """Finite C words: F32 with biased exponent uniform in [100, 154] (or F16
    with exponent in [1, 30]), sign and fraction uniform -- the distribution
    of finite_f32_c / finite_f16_c."""
    if f16:
        sign = torch.randint(0, 2, (n,), dtype=torch.int32, device=device, generator=gen) << 15
        exp = torch.randint(1, 31, (n,), dtype=torch.int32, device=device, generator=gen) << 10
        frac = torch.randint(0, 1 << 10, (n,), dtype=torch.int32, device=device, generator=gen)
        return (sign | exp | frac).to(torch.int16)
    sign = torch.randint(0, 2, (n,), dtype=torch.int64, device=device, generator=gen) << 31
    exp = torch.randint(100, 155, (n,), dtype=torch.int64, device=device, generator=gen) << 23
    frac = torch.randint(0, 1 << 23, (n,), dtype=torch.int64, device=device, generator=gen)
    return (sign | exp | frac).to(torch.int32)


def _device_selector_words(torch, gen, device, n, selectors):
    sel = torch.as_tensor(selectors.astype(np.int64), device=device)
    picks = sel[torch.randint(0, len(selectors), (n, 8), device=device, generator=gen)]
    shifts = torch.arange(8, device=device, dtype=torch.int64) * 4
    return (picks << shifts).sum(dim=1).to(torch.int64)


def device_config(name: str, device, seed: int = 0, n: int | None = None):
    """A configuration's inputs generated directly in HBM, in the kernels'
    packed layout, from a seeded device generator: returns (model, DeviceBatch).

    Uniformly random container words of a packed format are uniformly random
    bytes, so operand rows are random bytes; scales, C and metadata follow
    the configuration's stated distributions.  (The host generators of
    config_cases produce the same distributions from numpy; the two streams
    differ.)"""
    import torch

    from . import _native as nat
    from .model import make_model
    from .runtime import DeviceBatch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    n = CONFIG_SIZES[name] if n is None else n
    if name in ("e4m3xe5m2-k32", "e4m3xe5m2-k32-f16"):
        f16 = name.endswith("f16")
        model = make_model("e4m3", "e5m2", d_type="f16" if f16 else "f32")
        return model, DeviceBatch(n=n, k=32, a=_device_bytes(torch, gen, device, (n, 32)),
                                  b=_device_bytes(torch, gen, device, (n, 32)),
                                  c=_device_finite_c(torch, gen, device, n, f16))
    if name == "tf32-k8":
        model = make_model("tf32")
        c = _device_bytes(torch, gen, device, (n, 4)).view(torch.int32).reshape(n)
        return model, DeviceBatch(n=n, k=8, a=_device_bytes(torch, gen, device, (n, 32)),
                                  b=_device_bytes(torch, gen, device, (n, 32)), c=c)
    if name == "mx-e2m3xe3m2-k32":
        model = make_model("e2m3", "e3m2", scaling="ue8m0", kind="mxf8f6f4")
        db = DeviceBatch(n=n, k=32, a=_device_bytes(torch, gen, device, (n, 24)),
                         b=_device_bytes(torch, gen, device, (n, 24)), c=_device_finite_c(torch, gen, device, n))
        db.scale_a = torch.randint(0x70, 0x90, (n, 1), dtype=torch.uint8, device=device, generator=gen)
        db.scale_b = torch.randint(0x70, 0x90, (n, 1), dtype=torch.uint8, device=device, generator=gen)
        return model, db
    if name in ("u8xs8-k32-sat", "u8xs8-k32-wrap"):
        model = make_model("u8", "s8", d_type="s32", saturate=name.endswith("sat"))
        u = torch.randint(0, 1 << 21, (n,), dtype=torch.int64, device=device, generator=gen)
        top = torch.randint(0, 2, (n,), dtype=torch.int64, device=device, generator=gen).bool()
        c = torch.where(top, 0x7FFFFFFF - u, 0x80000000 + u).to(torch.int64)
        c = torch.where(c >= 1 << 31, c - (1 << 32), c).to(torch.int32)
        return model, DeviceBatch(n=n, k=32, a=_device_bytes(torch, gen, device, (n, 32)),
                                  b=_device_bytes(torch, gen, device, (n, 32)), c=c)
    if name in ("nvfp4-k64", "nvfp4-sparse-k128"):
        model = make_model("e2m1", scaling="ue4m3", scale_vec=4)
        sparse = name == "nvfp4-sparse-k128"
        db = DeviceBatch(n=n, k=128 if sparse else 64, a=_device_bytes(torch, gen, device, (n, 32)),
                         b=_device_bytes(torch, gen, device, (n, 64 if sparse else 32)),
                         c=_device_finite_c(torch, gen, device, n))
        db.scale_a = torch.randint(0x01, 0x7F, (n, 4), dtype=torch.uint8, device=device, generator=gen)
        db.scale_b = torch.randint(0x01, 0x7F, (n, 4), dtype=torch.uint8, device=device, generator=gen)
        if sparse:
            lo = _device_selector_words(torch, gen, device, n, SELECTORS_SIX)
            hi = _device_selector_words(torch, gen, device, n, SELECTORS_SIX)
            meta = torch.stack([lo, hi], dim=1)
            db.metadata = torch.where(meta >= 1 << 31, meta - (1 << 32), meta).to(torch.int32)
            db.sparse = nat.SPARSE_4OF8
            db.flags = nat.FLAG_SPARSE_A_COMPRESSED
        return model, db
    if name == "matrix-bf16":
        tiles, m, nn = n // (128 * 256), 128, 256
        model = make_model("bf16")
        c = _device_bytes(torch, gen, device, (n, 4)).view(torch.int32).reshape(n)
        return model, DeviceBatch(n=n, k=16, a=_device_bytes(torch, gen, device, (tiles * m, 32)),
                                  b=_device_bytes(torch, gen, device, (tiles * nn, 32)), c=c, tile_m=m, tile_n=nn)
    raise ValueError(f"unknown configuration {name!r}")


def config_work(name: str, db) -> tuple[int, int]:
    """(element-MACs, algorithmic bytes) of one launch over DeviceBatch db:
    physical products per case times cases; bytes of A, B, C, D, scales and
    metadata the launch must move (matrix tiles read each A and B row once)."""
    k_phys = 64 if name == "nvfp4-sparse-k128" else db.k
    macs = db.n * k_phys
    c_bytes = db.c.element_size()
    nbytes = db.a.numel() + db.b.numel() + db.n * (c_bytes + 4)
    if db.scale_a is not None:
        nbytes += db.scale_a.numel() + db.scale_b.numel()
    if db.metadata is not None:
        nbytes += db.metadata.numel() * 4
    return macs, nbytes

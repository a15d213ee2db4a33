"""Every benchmark configuration at its full size, word for word against the
oracle: the inputs are generated in HBM as the bench generates them (packed
rows), evaluated by the library, then copied to the host in chunks, unpacked
to container words and evaluated by the oracle on every host core.

Sizes: TF32 K=8 65,536 cases; E4M3 x E5M2 K=32 2^20 cases with F32 D and
with F16 D; MXF8F6F4 E2M3 x E3M2 2^22; U8 x S8 2^22 saturating and
wrapping; NVFP4 K=64 2^24 dense and 2^24 pairwise-sparse (logical K=128,
compressed A rows); the BF16 matrix configuration, 4096 tiles of
M=128 x N=256 x K=16 (134M cases), expanded tile by tile to one row pair per
case for the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tcgen05_b200 import make_model, packing, runtime, workloads

pytestmark = pytest.mark.gpu

# the public keywords of the model each configuration is generated for
KEYWORDS = {
    "tf32-k8": dict(a_format="tf32"),
    "e4m3xe5m2-k32": dict(a_format="e4m3", b_format="e5m2", d_type="f32"),
    "e4m3xe5m2-k32-f16": dict(a_format="e4m3", b_format="e5m2", d_type="f16"),
    "mx-e2m3xe3m2-k32": dict(a_format="e2m3", b_format="e3m2", scaling="ue8m0", kind="mxf8f6f4"),
    "u8xs8-k32-sat": dict(a_format="u8", b_format="s8", d_type="s32", saturate=True),
    "u8xs8-k32-wrap": dict(a_format="u8", b_format="s8", d_type="s32", saturate=False),
    "nvfp4-k64": dict(a_format="e2m1", scaling="ue4m3", scale_vec=4),
    "nvfp4-sparse-k128": dict(a_format="e2m1", scaling="ue4m3", scale_vec=4),
}
CHUNK = 1 << 19


def _host(t):
    return t.cpu().numpy()


def _chunk_words(db, desc, lo, hi):
    """Container words of cases lo..hi in the oracle's form."""
    sparse = db.sparse != 0
    k_b = db.k
    a = packing.unpack_rows(_host(db.a[lo:hi]), desc.a_format, db.k // 2 if sparse else db.k)
    b = packing.unpack_rows(_host(db.b[lo:hi]), desc.b_format, k_b)
    c = _host(db.c[lo:hi])
    c = c.view(np.uint16).astype(np.uint32) if c.dtype == np.int16 else c.view(np.uint32)
    meta = None if db.metadata is None else _host(db.metadata[lo:hi]).view(np.uint32)
    if sparse:
        # compressed A rows hold the selected elements in logical order
        act = workloads.active_mask(meta, db.k, "4of8")
        full = np.zeros((hi - lo, db.k), dtype=np.uint32)
        full[act] = a.reshape(-1)
        a = full
    sa = None if db.scale_a is None else _host(db.scale_a[lo:hi])
    sb = None if db.scale_b is None else _host(db.scale_b[lo:hi])
    return a, b, c, sa, sb, meta


@pytest.mark.parametrize("name", list(KEYWORDS))
def test_configuration_at_full_size_matches_oracle(name):
    import torch

    dev = torch.device("cuda", 0)
    model, db = workloads.device_config(name, dev, seed=0)
    assert db.n == workloads.CONFIG_SIZES[name]
    desc = model.descriptor()
    kw = KEYWORDS[name]
    assert bytes(desc) == bytes(make_model(**{k: v for k, v in kw.items()}).descriptor())
    d, st = runtime.launch(desc, db, status=True)
    got = _host(d).view(np.uint32)
    assert not _host(st).any()
    mismatches, first = 0, None
    for lo in range(0, db.n, CHUNK):
        hi = min(db.n, lo + CHUNK)
        a, b, c, sa, sb, meta = _chunk_words(db, desc, lo, hi)
        want, ost = oracle.mma_dot_batch(a, b, c, scale_a=sa, scale_b=sb, sparse_metadata=meta, **kw)
        assert not ost.any(), f"{name}: the oracle rejected a case in {lo}..{hi}"
        diff = np.flatnonzero(got[lo:hi] != want)
        if diff.size and first is None:
            first = (lo + int(diff[0]), int(got[lo + diff[0]]), int(want[diff[0]]))
        mismatches += int(diff.size)
    assert mismatches == 0, f"{name}: {mismatches} words differ, first (case, device, oracle) = {first}"


def test_matrix_configuration_at_full_size_matches_oracle():
    import torch

    dev = torch.device("cuda", 0)
    model, db = workloads.device_config("matrix-bf16", dev, seed=0)
    desc = model.descriptor()
    tm, tn = db.tile_m, db.tile_n
    tiles = db.n // (tm * tn)
    assert tiles == 4096
    d, _ = runtime.launch(desc, db, status=False)
    got = _host(d).view(np.uint32)
    per_call = 32  # tiles per oracle call
    mismatches, first = 0, None
    for t0 in range(0, tiles, per_call):
        t1 = min(tiles, t0 + per_call)
        a_rows = packing.unpack_rows(_host(db.a[t0 * tm:t1 * tm]), desc.a_format, db.k).reshape(t1 - t0, tm, db.k)
        b_rows = packing.unpack_rows(_host(db.b[t0 * tn:t1 * tn]), desc.b_format, db.k).reshape(t1 - t0, tn, db.k)
        # case (row, col) of a tile pairs A row `row` with B row `col`
        a = np.repeat(a_rows, tn, axis=1).reshape(-1, db.k)
        b = np.tile(b_rows, (1, tm, 1)).reshape(-1, db.k)
        lo, hi = t0 * tm * tn, t1 * tm * tn
        c = _host(db.c[lo:hi]).view(np.uint32)
        want, ost = oracle.mma_dot_batch(a, b, c, a_format="bf16")
        assert not ost.any()
        diff = np.flatnonzero(got[lo:hi] != want)
        if diff.size and first is None:
            first = (lo + int(diff[0]), int(got[lo + diff[0]]), int(want[diff[0]]))
        mismatches += int(diff.size)
    assert mismatches == 0, f"matrix-bf16: {mismatches} words differ, first (case, device, oracle) = {first}"

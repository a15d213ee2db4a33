"""t5e_mma_dot_batch_noalloc: host batches evaluated through the library's
static staging array, for callers that may not allocate GPU memory.

Every GPU test compares two calls in a row of the no-allocation entry point
with t5e_mma_dot_batch (the existing entry point, on device copies of the
same packed rows): result words and per-case status bytes must be equal,
bit for bit.  The second call is a smaller batch of another path, so a word
left in the array by the first call would show.  This file is named to be
collected last: its tests must also pass after every other test has run in
the same process."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import tcgen05_b200 as t5
from tcgen05_b200 import _native as nat
from tcgen05_b200 import packing, runtime, simulator, workloads

PATHS = {p.name: p for p in workloads.validation_paths()}


def _host_batch(cases: workloads.Cases, broadcast_meta=None):
    """(model descriptor, host DeviceBatch) in the layout the C-ABI reads, as
    torch tensors in pageable host memory."""
    import torch

    d = dict(a_format="tf32", b_format=None, d_type="f32", saturate=False, scaling=None, scale_vec=None, kind=None)
    d.update(cases.desc)
    model = t5.make_model(d["a_format"], d["b_format"], d_type=d["d_type"], saturate=d["saturate"],
                          scaling=d["scaling"], scale_vec=d["scale_vec"], kind=d["kind"])
    desc = model.descriptor()
    n, k = cases.n, cases.k
    a = torch.from_numpy(packing.pack_rows(cases.a, desc.a_format))
    b = torch.from_numpy(packing.pack_rows(cases.b, desc.b_format))
    c_np = simulator._c_host(cases.c, n, model)
    c = torch.from_numpy(c_np.view(np.int16) if c_np.dtype == np.uint16 else c_np.view(np.int32))
    record = cases.meta if broadcast_meta is None else broadcast_meta
    sparse, meta, flags = simulator._prepare(model, d["a_format"], d["scaling"], d["kind"], k, n, record)
    hb = runtime.DeviceBatch(n=n, k=k, a=a, b=b, c=c, sparse=sparse, flags=flags)
    if cases.scale_a is not None and desc.family in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED):
        hb.scale_a = torch.from_numpy(np.ascontiguousarray(cases.scale_a, dtype=np.uint8))
        hb.scale_b = torch.from_numpy(np.ascontiguousarray(cases.scale_b, dtype=np.uint8))
    if meta is not None:
        hb.metadata = torch.from_numpy(np.ascontiguousarray(np.asarray(meta).astype(np.uint32).view(np.int32)))
    return desc, hb


def _noalloc(desc, hb):
    """Result words and status bytes from t5e_mma_dot_batch_noalloc."""
    import torch

    d = torch.full((hb.n,), -1, dtype=torch.int32)
    st = torch.full((hb.n,), 0xEE, dtype=torch.uint8)
    bs = runtime.make_batch_struct(hb, d, st)
    lib = nat.load()
    stream = runtime.current_stream_handle(torch.device("cuda"))
    rc = lib.t5e_mma_dot_batch_noalloc(ctypes.byref(desc), ctypes.byref(bs), ctypes.c_void_p(stream))
    nat.check(rc, "t5e_mma_dot_batch_noalloc")
    return d.numpy().view(np.uint32), st.numpy()


def _existing(desc, hb):
    """Result words and status bytes from t5e_mma_dot_batch on device copies."""
    import torch

    dev = torch.device("cuda")
    db = runtime.DeviceBatch(n=hb.n, k=hb.k, a=hb.a.to(dev), b=hb.b.to(dev), c=hb.c.to(dev), sparse=hb.sparse,
                             flags=hb.flags)
    if hb.scale_a is not None:
        db.scale_a, db.scale_b = hb.scale_a.to(dev), hb.scale_b.to(dev)
    if hb.metadata is not None:
        db.metadata = hb.metadata.to(dev)
    d, st = runtime.launch(desc, db, status=True)
    return d.cpu().numpy().view(np.uint32), st.cpu().numpy()


def _assert_same(got, want, what):
    gd, gs = got
    wd, ws = want
    bad = np.flatnonzero(gd != wd)
    assert bad.size == 0, f"{what}: {bad.size} words differ, first case {bad[0]}: {gd[bad[0]]:#010x} != {wd[bad[0]]:#010x}"
    assert np.array_equal(gs, ws), f"{what}: status bytes differ"


# a second path for each first one: another family, so the second call's
# regions start at other offsets of the array
PAIRS = [(name, list(PATHS)[(i + 17) % len(PATHS)]) for i, name in enumerate(PATHS)]


@pytest.mark.gpu
@pytest.mark.parametrize("first,second", PAIRS, ids=[f"{a}-then-{b}" for a, b in PAIRS])
def test_two_calls_in_a_row_match_existing_entry_point(first, second):
    for name, n, seed in ((first, 3000, 11), (second, 1100, 12)):
        cases = workloads.path_cases(PATHS[name], n, seed=seed)
        desc, hb = _host_batch(cases)
        _assert_same(_noalloc(desc, hb), _existing(desc, hb), name)


@pytest.mark.gpu
def test_shared_metadata_record_and_repeat():
    """Sparse metadata shared by every case (one record staged) and one word
    repeated over K."""
    spec = PATHS["sparse-fp8"]
    cases = workloads.path_cases(spec, 2048, seed=5)
    for record in ((0x4C8D9E64, 0xE6D9C844), 0x4E):
        desc, hb = _host_batch(cases, broadcast_meta=record)
        for _ in range(2):
            _assert_same(_noalloc(desc, hb), _existing(desc, hb), f"metadata {record!r}")


@pytest.mark.gpu
def test_bad_selectors_report_the_same_status():
    """Cases whose metadata selects an illegal pattern get the same status
    bytes from both entry points."""
    cases = workloads.path_cases(PATHS["sparse-nvfp4"], 1024, seed=9)
    meta = cases.meta.copy()
    meta[::7, 0] = 0xFFFFFFFF  # selector 0xF is illegal for four of eight
    cases = workloads.Cases(cases.desc, cases.a, cases.b, cases.c, cases.scale_a, cases.scale_b, meta, cases.name)
    desc, hb = _host_batch(cases)
    got = _noalloc(desc, hb)
    _assert_same(got, _existing(desc, hb), "bad selectors")
    assert (got[1][::7] != 0).all()


def _staging_bytes(hb) -> int:
    """Bytes of the array a dense batch with status bytes takes: A rows, B
    rows, C words, D words and status bytes, each region rounded up to 256."""
    per_case = (hb.a.shape[1], hb.b.shape[1], hb.c.element_size(), 4, 1)
    return sum(-(-hb.n * x // 256) * 256 for x in per_case)


def _tiled(hb, n):
    """The batch's cases repeated to n cases."""
    reps = -(-n // hb.n)
    return runtime.DeviceBatch(n=n, k=hb.k, a=hb.a.repeat(reps, 1)[:n].contiguous(),
                               b=hb.b.repeat(reps, 1)[:n].contiguous(), c=hb.c.repeat(reps)[:n].contiguous(),
                               sparse=hb.sparse, flags=hb.flags)


def _largest_fit(hb) -> int:
    per_case = hb.a.shape[1] + hb.b.shape[1] + hb.c.element_size() + 4 + 1
    n = nat.NOALLOC_STAGE_BYTES // per_case
    while _staging_bytes(_Shape(hb, n)) > nat.NOALLOC_STAGE_BYTES:
        n -= 1
    return n


class _Shape:
    """The row widths of a batch at another case count."""

    def __init__(self, hb, n):
        self.a, self.b, self.c, self.n = hb.a, hb.b, hb.c, n


@pytest.mark.gpu
def test_largest_batch_that_fits_and_first_that_does_not():
    """The largest E4M3 batch inside the array is evaluated like the
    existing entry point; one more case is rejected before any copy."""
    cases = workloads.path_cases(PATHS["dense-e4m3"], 1024, seed=3)
    desc, hb = _host_batch(cases)
    n_fit = _largest_fit(hb)
    big = _tiled(hb, n_fit)
    assert _staging_bytes(big) <= nat.NOALLOC_STAGE_BYTES
    _assert_same(_noalloc(desc, big), _existing(desc, big), "largest batch")
    over = _tiled(hb, n_fit + 1)
    assert _staging_bytes(over) > nat.NOALLOC_STAGE_BYTES
    _expect_rejected(desc, over)


def _expect_rejected(desc, hb):
    import torch

    d = torch.zeros(hb.n, dtype=torch.int32)
    st = torch.zeros(hb.n, dtype=torch.uint8)
    bs = runtime.make_batch_struct(hb, d, st)
    lib = nat.load()
    rc = lib.t5e_mma_dot_batch_noalloc(ctypes.byref(desc), ctypes.byref(bs), ctypes.c_void_p(0))
    assert rc == nat.ERR_INVALID
    assert b"staging" in lib.t5e_last_error()
    assert not d.any()


def test_oversized_batch_rejected_without_a_device():
    """The size check runs on the host before any CUDA call: a batch larger
    than the staging array is rejected on a machine with no GPU."""
    cases = workloads.path_cases(PATHS["dense-bf16"], 64, seed=1)
    desc, hb = _host_batch(cases)
    _expect_rejected(desc, _tiled(hb, _largest_fit(hb) + 1))


def test_header_and_python_agree_on_the_array_size():
    from pathlib import Path
    import re

    text = (Path(__file__).resolve().parents[1] / "include" / "t5e.h").read_text()
    m = re.search(r"#define T5E_NOALLOC_STAGE_BYTES \((\d+)u \* 1024u \* 1024u\)", text)
    assert m and int(m.group(1)) * 1024 * 1024 == nat.NOALLOC_STAGE_BYTES


@pytest.mark.gpu
def test_call_on_a_capturing_stream_is_refused_and_the_capture_survives():
    """The entry point synchronizes its stream, which a capture forbids: on a
    capturing stream it returns T5E_ERR_INVALID without queuing anything, and
    the capture (here of a plain tensor fill) still completes and replays."""
    import torch

    cases = workloads.path_cases(PATHS["dense-e4m3"], 256, seed=7)
    desc, hb = _host_batch(cases)
    d = torch.full((hb.n,), -1, dtype=torch.int32)
    bs = runtime.make_batch_struct(hb, d, None)
    lib = nat.load()
    x = torch.zeros(16, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        stream = torch.cuda.current_stream().cuda_stream
        rc = lib.t5e_mma_dot_batch_noalloc(ctypes.byref(desc), ctypes.byref(bs), ctypes.c_void_p(stream))
        x.fill_(3.0)
    assert rc == nat.ERR_INVALID
    assert "capturing" in nat.load().t5e_last_error().decode()
    g.replay()
    torch.cuda.synchronize()
    assert float(x.sum()) == 48.0
    assert int((d == -1).sum()) == hb.n  # nothing was written

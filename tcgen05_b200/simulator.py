"""Scalar, matrix and batched entry points of the tcgen05 MMA emulator.

``mma_dot`` and ``mma`` keep the signatures and ValueError behaviour of the
reference's tcgen05_model/simulator.py:80-211; ``mma_dot_batch`` and
``mma_batch`` evaluate N independent dot products or T independent tiles in
one kernel launch.  All arithmetic runs in the CUDA library; the host only
validates arguments, packs operand rows and moves buffers.
"""

from __future__ import annotations

import ctypes

from collections.abc import Sequence

import numpy as np

from . import _native as nat
from . import packing
from . import runtime
from .model import DotProduct, ScalarModel, _ModelBase, make_model, normalize_format

SPARSE_TF32_SELECTORS = frozenset((0x4, 0xE))
SPARSE_2OF4_SELECTORS = frozenset((0x4, 0x8, 0xC, 0x9, 0xD, 0x6, 0xE))


def _matrix(value: Sequence[Sequence[int]], name: str) -> tuple[tuple[int, ...], ...]:
    """Row-major matrix checks of tcgen05_model/simulator.py:13-23."""
    rows = tuple(tuple(row) for row in value)
    if not rows or not rows[0]:
        raise ValueError(f"{name} must be a non-empty matrix")
    width = len(rows[0])
    if any(len(row) != width for row in rows):
        raise ValueError(f"{name} must be rectangular")
    for word in (word for row in rows for word in row):
        if not isinstance(word, (int, np.integer)) or isinstance(word, bool) or not 0 <= word <= 0xFFFF_FFFF:
            raise ValueError(f"{name} contains a non-uint32 word: {word!r}")
    return rows


def _sparse_geometry(format_name: str, kind: str | None, nvfp4: bool = False) -> tuple[int, int]:
    """(T5E_SPARSE_* mode, chunk size) of a descriptor; validates ``kind``."""
    if kind not in (None, "mxf8f6f4", "mxf4", "mxf4nvf4", "nvfp4"):
        raise ValueError(f"unsupported sparse metadata kind: {kind!r}")
    if format_name == "tf32":
        return nat.SPARSE_1OF2, 2
    if nvfp4 or kind in ("mxf4", "mxf4nvf4", "nvfp4"):
        return nat.SPARSE_4OF8, 8
    return nat.SPARSE_2OF4, 4


def sparse_active_indices(
    format_name: str,
    k: int,
    metadata: int | Sequence[int],
    *,
    kind: str | None = None,
    nvfp4: bool = False,
) -> frozenset[int]:
    """Logical K indices selected by tcgen05 sparse metadata
    (tcgen05_model/simulator.py:26-77).

    TF32 keeps one value of each pair (selector 0x4: lower, 0xE: upper);
    BF16/F16/f8/f6/f4 keep two of each four (the selector's low and high
    2-bit fields); kind "mxf4", "mxf4nvf4" or "nvfp4" keeps two adjacent
    pairs of each eight.  Nibbles are read least significant first; an int
    metadata word repeats over K.
    """
    format_name = normalize_format(format_name)
    kind = None if kind is None else kind.lower()
    mode, chunk_size = _sparse_geometry(format_name, kind, nvfp4)
    words = (metadata,) if isinstance(metadata, (int, np.integer)) else tuple(metadata)
    if not words or any(not 0 <= word <= 0xFFFF_FFFF for word in words):
        raise ValueError("metadata must contain uint32 words")
    chunks = (k + chunk_size - 1) // chunk_size
    if isinstance(metadata, (int, np.integer)):
        words = words * ((chunks + 7) // 8)
    if len(words) * 8 < chunks:
        raise ValueError(f"{chunks} metadata nibbles are required for K={k}")
    legal = SPARSE_TF32_SELECTORS if mode == nat.SPARSE_1OF2 else SPARSE_2OF4_SELECTORS
    active: set[int] = set()
    for chunk in range(chunks):
        selector = (int(words[chunk // 8]) >> ((chunk & 7) * 4)) & 0xF
        if selector not in legal:
            raise ValueError(f"illegal sparse selector 0x{selector:x} in chunk {chunk}")
        if mode == nat.SPARSE_1OF2:
            active.add(chunk * 2 + (selector == 0xE))
            continue
        low, high = selector & 3, (selector >> 2) & 3
        if mode == nat.SPARSE_4OF8:
            for pair in (low, high):
                active.update((chunk * 8 + pair * 2, chunk * 8 + pair * 2 + 1))
        else:
            active.update((chunk * 4 + low, chunk * 4 + high))
    return frozenset(index for index in active if index < k)


# ---------------------------------------------------------------- helpers


def _is_torch(x) -> bool:
    try:
        import torch
    except ImportError:  # pragma: no cover - torch is a dependency
        return False
    return isinstance(x, torch.Tensor)


def _words_np(x, name: str) -> np.ndarray:
    """Host array of raw words checked to be uint32 values (as int64)."""
    arr = np.asarray(x)
    if arr.dtype == object or arr.dtype.kind not in "iu":
        try:
            arr = np.asarray(x, dtype=np.int64)
        except (OverflowError, TypeError, ValueError) as exc:
            raise ValueError(f"{name} contains a non-uint32 word") from exc
    if arr.dtype.kind == "u" and arr.dtype.itemsize <= 4:
        return arr.astype(np.uint32)
    if arr.size and (arr.min() < 0 or arr.max() > 0xFFFF_FFFF):
        bad = arr[(arr < 0) | (arr > 0xFFFF_FFFF)].flat[0]
        raise ValueError(f"operand is not a uint32 word: {int(bad)!r}")
    return arr.astype(np.uint32)


def _scales_np(x, name: str) -> np.ndarray:
    arr = np.asarray(x)
    if arr.dtype == object or arr.dtype.kind not in "iu":
        arr = np.asarray(x, dtype=np.int64)
    if arr.size and (arr.min() < 0 or arr.max() > 0xFF):
        bad = arr[(arr < 0) | (arr > 0xFF)].flat[0]
        raise ValueError(f"scale is not an 8-bit word: {int(bad)!r}")
    return arr.astype(np.uint8)


def _c_dtype_bytes(model) -> int:
    return 2 if model.descriptor().d_type == nat.D_F16 else 4


def _c_words_on_device(c_dev, f16: bool):
    """C words already on the device -> the dtype the kernel reads."""
    import torch

    want = 2 if f16 else 4
    if c_dev.element_size() == want and c_dev.dtype in (torch.int16, torch.uint16, torch.int32, torch.uint32):
        return c_dev.view(torch.int16 if f16 else torch.int32).contiguous()
    wide = c_dev.to(torch.int64)
    if f16:
        return wide.bitwise_and(0xFFFF).to(torch.int32).to(torch.int16).contiguous()
    return wide.bitwise_and(0xFFFFFFFF).to(torch.int32).contiguous()


def _c_host(c, n: int, model) -> np.ndarray:
    """C words as the dtype the kernel reads (uint16 for F16 C, else uint32)."""
    words = np.zeros(n, dtype=np.uint32) if c is None else _words_np(c, "C").reshape(n)
    if _c_dtype_bytes(model) == 2:
        return (words & 0xFFFF).astype(np.uint16)
    return words


def _check_scale_pair(model, k_phys: int, nsa: int | None, nsb: int | None) -> int:
    """Scale-count rules of the scaled models (model.py:725-731, :852-858);
    returns the per-operand scale count the kernel reads (0: defaults)."""
    if (nsa is None) != (nsb is None):
        raise ValueError("scale_a and scale_b must be supplied together")
    d = model.descriptor()
    if d.family not in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED):
        return -1  # scales are ignored by this family
    if nsa is None:
        return 0
    if nsa != nsb:
        raise ValueError(model._scale_count_error)
    if nsa * d.scale_block < k_phys:
        raise ValueError(model._scale_cover_error)
    return nsa


def _eval_case_arrays(model, a, b, c, sa, sb, *, device=None) -> np.ndarray:
    """Evaluate dense cases given as host word arrays (used by model.eval)."""
    a = _words_np(a, "A")
    b = _words_np(b, "B")
    n, k = a.shape
    if b.shape != (n, k):
        raise ValueError("A and B dot-product vectors must have equal length")
    if k == 0:
        raise ValueError("a dot product must contain at least one element")
    if k > nat.MAX_K:
        raise ValueError(f"K={k} exceeds the emulator's maximum of {nat.MAX_K}")
    if sa is not None:
        sa = _scales_np(sa, "scale_a").reshape(n, -1)
    if sb is not None:
        sb = _scales_np(sb, "scale_b").reshape(n, -1)
    nscale = _check_scale_pair(model, k, None if sa is None else sa.shape[1], None if sb is None else sb.shape[1])
    desc = model.descriptor()
    dev = runtime.require_device(device)
    batch = runtime.DeviceBatch(
        n=n,
        k=k,
        a=runtime.to_device(packing.pack_rows(a, desc.a_format), dev),
        b=runtime.to_device(packing.pack_rows(b, desc.b_format), dev),
        c=runtime.to_device(_c_host(c, n, model), dev),
    )
    if nscale > 0:
        batch.scale_a = runtime.to_device(sa, dev)
        batch.scale_b = runtime.to_device(sb, dev)
    d, st = runtime.launch(desc, batch)
    st_h = st.cpu().numpy()
    if st_h.any():
        first = int(np.flatnonzero(st_h)[0])
        _raise_case_status(model, int(st_h[first]))
    return d.cpu().numpy().view(np.uint32).copy()


def _raise_case_status(model, status: int, *, meta_message=None) -> None:
    if status == nat.CASE_EMPTY:
        raise ValueError("a dot product must contain at least one element")
    if status == nat.CASE_SCALE_COVER:
        raise ValueError(model._scale_cover_error)
    if status in (nat.CASE_BAD_SELECTOR, nat.CASE_META_WORDS) and meta_message is not None:
        meta_message()
    if status == nat.CASE_TIMEOUT:
        raise RuntimeError("a bounded device wait for this case's input copy expired; no result was produced")
    raise ValueError(f"invalid case (status {status})")


# ------------------------------------------------------------ scalar API


def mma_dot(
    a: Sequence[int],
    b: Sequence[int],
    c: int = 0,
    *,
    model: ScalarModel | None = None,
    a_format: str = "tf32",
    b_format: str | None = None,
    d_type: str = "f32",
    saturate: bool = False,
    scaling: str | None = None,
    scale_vec: int | None = None,
    kind: str | None = None,
    scale_a: Sequence[int] | None = None,
    scale_b: Sequence[int] | None = None,
    sparse_metadata: int | Sequence[int] | None = None,
) -> int:
    """One tcgen05 output word (tcgen05_model/simulator.py:80-140), evaluated
    on the GPU.  Sparse calls take full logical-K A/B; disabled positions are
    dropped before classification (masked for unscaled formats, compressed
    to physical K before scale-block assignment for scaled ones)."""
    a_words, b_words = tuple(a), tuple(b)
    if len(a_words) != len(b_words):
        raise ValueError("A and B dot-product vectors must have equal length")
    if sparse_metadata is not None:
        active = sparse_active_indices(
            a_format,
            len(a_words),
            sparse_metadata,
            kind="nvfp4" if (scaling or "").lower() == "ue4m3" else kind,
        )
        if scaling is None:
            a_words = tuple(word if index in active else 0 for index, word in enumerate(a_words))
            b_words = tuple(word if index in active else 0 for index, word in enumerate(b_words))
        else:
            order = sorted(active)
            a_words = tuple(a_words[index] for index in order)
            b_words = tuple(b_words[index] for index in order)
    selected = model or make_model(
        a_format,
        b_format,
        d_type=d_type,
        saturate=saturate,
        scaling=scaling,
        scale_vec=scale_vec,
        sparse=False if scaling is not None else sparse_metadata is not None,
        kind=kind,
    )
    case = DotProduct(
        a_words,
        b_words,
        c,
        None if scale_a is None else tuple(scale_a),
        None if scale_b is None else tuple(scale_b),
    )
    return selected.eval(case)


def mma(
    a: Sequence[Sequence[int]],
    b: Sequence[Sequence[int]],
    c: Sequence[Sequence[int]] | None = None,
    *,
    a_format: str = "tf32",
    b_format: str | None = None,
    d_type: str = "f32",
    saturate: bool = False,
    scaling: str | None = None,
    scale_vec: int | None = None,
    kind: str | None = None,
    scale_a: Sequence[Sequence[int]] | None = None,
    scale_b: Sequence[Sequence[int]] | None = None,
    sparse_metadata: int | Sequence[int] | None = None,
) -> tuple[tuple[int, ...], ...]:
    """``D = A @ B + C`` on row-major raw-word matrices
    (tcgen05_model/simulator.py:143-211): every output word is the scalar
    model of one row of A and one column of B, all evaluated in one launch.
    ``scale_a`` is indexed by A row, ``scale_b`` by B column."""
    a_rows, b_rows = _matrix(a, "A"), _matrix(b, "B")
    m, k, n = len(a_rows), len(a_rows[0]), len(b_rows[0])
    if len(b_rows) != k:
        raise ValueError(f"A is {m}x{k} but B has {len(b_rows)} rows")
    c_rows = tuple((0,) * n for _ in range(m)) if c is None else _matrix(c, "C")
    if len(c_rows) != m or len(c_rows[0]) != n:
        raise ValueError(f"C must be {m}x{n}")
    sa_rows = None if scale_a is None else _matrix(scale_a, "scale_a")
    sb_rows = None if scale_b is None else _matrix(scale_b, "scale_b")
    if (sa_rows is None) != (sb_rows is None):
        raise ValueError("scale_a and scale_b must be supplied together")
    if sa_rows is not None and (len(sa_rows) != m or len(sb_rows) != n):
        raise ValueError("scale_a needs one row per A row and scale_b one row per B column")
    model = make_model(
        a_format,
        b_format,
        d_type=d_type,
        saturate=saturate,
        scaling=scaling,
        scale_vec=scale_vec,
        sparse=sparse_metadata is not None,
        kind=kind,
    )
    result = mma_batch(
        np.array(a_rows, dtype=np.int64)[None],
        np.array(b_rows, dtype=np.int64)[None],
        np.array(c_rows, dtype=np.int64)[None],
        model=model,
        a_format=a_format,
        scaling=scaling,
        kind=kind,
        scale_a=None if sa_rows is None else np.array(sa_rows, dtype=np.int64)[None],
        scale_b=None if sb_rows is None else np.array(sb_rows, dtype=np.int64)[None],
        sparse_metadata=sparse_metadata,
    )
    return tuple(tuple(int(w) for w in row) for row in result[0])


# ----------------------------------------------------------- batched API


class PendingBatch:
    """Result words of a host batch that ``mma_dot_batch(..., wait=False)``
    left in flight.  ``wait()`` blocks until every word is in ``out`` and
    returns it; ``ready()`` polls.  The device buffers the batch streams
    through, and the caller's pinned host inputs the uploads read, stay
    referenced here until then, so that neither allocator can hand them out
    while a copy still uses them (a caller may drop its inputs right after
    the call); dropping an unfinished batch therefore waits for it."""

    def __init__(self, out, event=None, buffers=None):
        self.out = out
        self._event = event
        self._buffers = buffers

    def ready(self) -> bool:
        return self._buffers is None or self._event.query()

    def wait(self):
        if self._buffers is not None:
            self._event.synchronize()
            self._buffers = None
        return self.out

    def __del__(self):
        if getattr(self, "_buffers", None) is not None:
            try:
                self._event.synchronize()
            except Exception:  # interpreter shutdown: the CUDA context may already be gone
                pass


class PackedRows:
    """Operand rows already in the kernels' packed layout (see packing.py):
    ``data`` is a [rows, stride] uint8 array or tensor, ``k`` the elements per
    row (the selected count for a compressed sparse A)."""

    def __init__(self, data, k: int, compressed: bool = False):
        self.data = data
        self.k = k
        self.compressed = compressed


def _metadata_array(sparse_metadata, rows: int):
    """Metadata as ([R or 1, W] uint32 host/tensor, flags)."""
    if isinstance(sparse_metadata, (int, np.integer)):
        if not 0 <= sparse_metadata <= 0xFFFF_FFFF:
            raise ValueError("metadata must contain uint32 words")
        return np.array([[sparse_metadata]], dtype=np.uint32), nat.FLAG_META_REPEAT | nat.FLAG_META_BROADCAST
    if isinstance(sparse_metadata, (list, tuple)):
        words = tuple(sparse_metadata)
        if not words or any(not 0 <= int(w) <= 0xFFFF_FFFF for w in words):
            raise ValueError("metadata must contain uint32 words")
        return np.array([words], dtype=np.uint32), nat.FLAG_META_BROADCAST
    if _is_torch(sparse_metadata):
        t = sparse_metadata
        if t.dim() == 1:
            return t.reshape(-1, 1), nat.FLAG_META_REPEAT
        return t, 0
    arr = _words_np(sparse_metadata, "metadata")
    if arr.ndim == 1:
        return arr.reshape(-1, 1), nat.FLAG_META_REPEAT
    return arr, 0


def _operand_rows(x, fmt: int, dev, name: str):
    """Host/device words or PackedRows -> (device uint8 [R, stride], rows, k)."""
    import torch

    if isinstance(x, PackedRows):
        return runtime.to_device(x.data, dev, torch.uint8), x.data.shape[0], x.k
    if _is_torch(x) and x.is_cuda:
        if x.dim() != 2:
            raise ValueError(f"{name} must be a [N, K] array of words")
        return packing.pack_rows_device(x.to(dev), fmt), x.shape[0], x.shape[1]
    words = _words_np(x, name)
    if words.ndim != 2:
        raise ValueError(f"{name} must be a [N, K] array of words")
    return runtime.to_device(packing.pack_rows(words, fmt), dev), words.shape[0], words.shape[1]


def _prepare(model, a_format, scaling, kind, k, rows_a, sparse_metadata):
    if sparse_metadata is None:
        return 0, None, 0
    fmt = normalize_format(a_format)
    meta_kind = "nvfp4" if (scaling or "").lower() == "ue4m3" else (None if kind is None else kind.lower())
    mode, chunk = _sparse_geometry(fmt, meta_kind)
    meta, flags = _metadata_array(sparse_metadata, rows_a)
    chunks = (k + chunk - 1) // chunk
    if not (flags & nat.FLAG_META_REPEAT) and meta.shape[1] * 8 < chunks:
        raise ValueError(f"{chunks} metadata nibbles are required for K={k}")
    return mode, meta, flags


def _run(model, a_rows, b_rows, c_dev, k, dev, *, n, tile_m, tile_n, scale_a, scale_b, sparse, meta, flags,
         a_compressed, check, meta_error, generic=False):
    import torch

    desc = model.descriptor()
    batch = runtime.DeviceBatch(n=n, k=k, a=a_rows, b=b_rows, c=c_dev, tile_m=tile_m, tile_n=tile_n,
                                sparse=sparse, flags=flags | (nat.FLAG_SPARSE_A_COMPRESSED if a_compressed else 0))
    if scale_a is not None:
        batch.scale_a = runtime.to_device(scale_a, dev, torch.uint8)
        batch.scale_b = runtime.to_device(scale_b, dev, torch.uint8)
    if meta is not None:
        batch.metadata = runtime.to_device(meta, dev, torch.int32 if not _is_torch(meta) else None)
    d, st = runtime.launch(desc, batch, status=check, generic=generic)
    if check:
        st_h = st.cpu().numpy()
        if st_h.any():
            first = int(np.flatnonzero(st_h)[0])
            _raise_case_status(model, int(st_h[first]), meta_message=lambda: meta_error(first))
    return d


def _pinned(x) -> bool:
    return _is_torch(x) and not x.is_cuda and x.is_pinned()


# Batches at least this large, with every per-case array in pinned host
# memory, are streamed through the GPU in chunks (see _pipelined_batch).
# Each chunk costs tens of microseconds of host-side issue, so a few large
# chunks keep the host-to-device copies back to back.
PIPELINE_MIN_CASES = 1 << 16
PIPELINE_CHUNKS = 4
# Batches left in flight (wait=False) overlap with the next batch's upload,
# so each needs fewer chunks of its own: fewer, larger copies keep the link
# closer to its plain-copy rate (measured: 53 GB/s with 1-2 chunks, 52 with
# 4, 50 with 8, for 70 MB batches back to back).
PIPELINE_CHUNKS_IN_FLIGHT = 2

_COPY_STREAMS: dict = {}


def _copy_streams(dev):
    """The (upload, download) streams of a device, created once."""
    import torch

    key = dev.index if dev.index is not None else torch.cuda.current_device()
    pair = _COPY_STREAMS.get(key)
    if pair is None:
        pair = _COPY_STREAMS[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return pair


def _pipelined_batch(selected, desc, a, b, c, sa, sb, meta, flags, sparse, k, n, dev, out, check, meta_error,
                     generic, wait=True):
    """Host-resident batch in pinned memory -> pinned ``out``: the cases are
    cut into chunks; each chunk's operands are copied to the device on one
    stream, evaluated on the current stream once its copy has landed, and its
    result words (and status bytes) copied back on a third stream, so the
    copies in both directions overlap each other and the kernels.  The
    library's t5e_mma_dot_batch_staged runs that loop; the loop below it
    serves the generic kernel and metadata shared by every case.  With
    ``wait`` false and no per-case status to read back, the library call
    returns once everything is queued and a PendingBatch is returned."""
    import torch

    comp = torch.cuda.current_stream(dev)
    # per-case status bytes only exist for sparse selections: every other
    # per-case error (scale cover, K range) is decided for the whole batch on
    # the host before the launch
    check = check and sparse != 0
    a_dev = torch.empty(a.data.shape, dtype=torch.uint8, device=dev)
    b_dev = torch.empty(b.data.shape, dtype=torch.uint8, device=dev)
    c_dev = torch.empty(c.shape, dtype=c.dtype, device=dev)
    sa_dev = None if sa is None else torch.empty(sa.shape, dtype=torch.uint8, device=dev)
    sb_dev = None if sb is None else torch.empty(sb.shape, dtype=torch.uint8, device=dev)
    per_case_meta = meta is not None and not (flags & nat.FLAG_META_BROADCAST)
    meta_dev = None
    if meta is not None:
        meta_dev = (torch.empty(meta.shape, dtype=torch.int32, device=dev) if per_case_meta
                    else runtime.to_device(meta, dev, torch.int32))
    d_dev = torch.empty(n, dtype=torch.int32, device=dev)
    st_dev = torch.empty(n, dtype=torch.uint8, device=dev) if check else None
    st_host = torch.empty(n, dtype=torch.uint8, pin_memory=True) if check else None
    lib = nat.load()
    fn = lib.t5e_mma_dot_batch_generic if generic else lib.t5e_mma_dot_batch
    handle = ctypes.c_void_p(comp.cuda_stream)
    step = -(-n // (PIPELINE_CHUNKS if wait or check else PIPELINE_CHUNKS_IN_FLIGHT))
    step = (step + 1023) // 1024 * 1024
    sa_h = None if sa is None else sa.view(torch.uint8)
    sb_h = None if sb is None else sb.view(torch.uint8)
    a_flags = flags | (nat.FLAG_SPARSE_A_COMPRESSED if a.compressed else 0)
    if not generic and (meta is None or per_case_meta):
        # the chunk loop runs inside the library: one call streams the whole
        # batch (copies up, kernels, copies down) through the device buffers
        # above and returns with `out` filled
        db = runtime.DeviceBatch(n=n, k=k, a=a_dev, b=b_dev, c=c_dev, sparse=sparse, flags=a_flags)
        hb = runtime.DeviceBatch(n=n, k=k, a=a.data, b=b.data, c=c, sparse=sparse, flags=a_flags)
        if sa_dev is not None:
            db.scale_a, db.scale_b = sa_dev, sb_dev
            hb.scale_a, hb.scale_b = sa_h, sb_h
        if meta_dev is not None:
            db.metadata = meta_dev
            hb.metadata = meta.view(torch.int32)
        dev_struct = runtime.make_batch_struct(db, d_dev, st_dev)
        host_struct = runtime.make_batch_struct(hb, out, st_host)
        if not wait and not check:
            done = torch.cuda.Event()
            done.record(comp)  # creates the event; the library records it again after the last download
            nat.check(lib.t5e_mma_dot_batch_staged_async(ctypes.byref(desc), ctypes.byref(host_struct),
                                                         ctypes.byref(dev_struct), step, handle,
                                                         ctypes.c_void_p(done.cuda_event)),
                      "t5e_mma_dot_batch_staged_async")
            # the library's uploads read the caller's pinned inputs on its own stream, so the pinned-memory
            # allocator records no use of them: they stay referenced here, with the device buffers, until the
            # batch's event has fired, so that none can be freed and handed to a new allocation meanwhile
            return PendingBatch(out, done, (a_dev, b_dev, c_dev, sa_dev, sb_dev, meta_dev, d_dev,
                                            a.data, b.data, c, sa_h, sb_h, meta))
        nat.check(lib.t5e_mma_dot_batch_staged(ctypes.byref(desc), ctypes.byref(host_struct), ctypes.byref(dev_struct),
                                               step, handle), "t5e_mma_dot_batch_staged")
        if check:
            st_np = st_host.numpy()
            if st_np.any():
                first = int(np.flatnonzero(st_np)[0])
                _raise_case_status(selected, int(st_np[first]), meta_message=lambda: meta_error(first))
        return out
    up, down = _copy_streams(dev)
    # the device buffers above come from the allocator on the current stream:
    # the uploads wait for whatever that stream still has queued
    up.wait_stream(comp)
    for s0 in range(0, n, step):
        s1 = min(n, s0 + step)
        with torch.cuda.stream(up):
            a_dev[s0:s1].copy_(a.data[s0:s1], non_blocking=True)
            b_dev[s0:s1].copy_(b.data[s0:s1], non_blocking=True)
            c_dev[s0:s1].copy_(c[s0:s1], non_blocking=True)
            if sa_dev is not None:
                sa_dev[s0:s1].copy_(sa_h[s0:s1], non_blocking=True)
                sb_dev[s0:s1].copy_(sb_h[s0:s1], non_blocking=True)
            if per_case_meta:
                meta_dev[s0:s1].copy_(meta[s0:s1].view(torch.int32), non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(up)
        comp.wait_event(landed)
        db = runtime.DeviceBatch(n=s1 - s0, k=k, a=a_dev[s0:s1], b=b_dev[s0:s1], c=c_dev[s0:s1], sparse=sparse,
                                 flags=a_flags)
        if sa_dev is not None:
            db.scale_a, db.scale_b = sa_dev[s0:s1], sb_dev[s0:s1]
        if meta_dev is not None:
            db.metadata = meta_dev[s0:s1] if per_case_meta else meta_dev
        bs = runtime.make_batch_struct(db, d_dev[s0:s1], None if st_dev is None else st_dev[s0:s1])
        nat.check(fn(ctypes.byref(desc), ctypes.byref(bs), handle), "t5e_mma_dot_batch")
        done = torch.cuda.Event()
        done.record(comp)
        down.wait_event(done)
        with torch.cuda.stream(down):
            out[s0:s1].copy_(d_dev[s0:s1].view(out.dtype), non_blocking=True)
            if st_dev is not None:
                st_host[s0:s1].copy_(st_dev[s0:s1], non_blocking=True)
    down.synchronize()
    if check:
        st_np = st_host.numpy()
        if st_np.any():
            first = int(np.flatnonzero(st_np)[0])
            _raise_case_status(selected, int(st_np[first]), meta_message=lambda: meta_error(first))
    return out


def _raw_words_pinned(x) -> bool:
    """A pinned host tensor of raw 32-bit container words, [N, K]."""
    import torch

    return _pinned(x) and x.dim() == 2 and x.dtype in (torch.int32, torch.uint32)


def _pack_chunk(raw, fmt: int, out, stream) -> None:
    """Raw words already on the device -> packed rows in ``out`` (t5e_pack_rows)."""
    rc = nat.load().t5e_pack_rows(fmt, raw.data_ptr(), raw.shape[0], raw.shape[1], out.data_ptr(), out.shape[1],
                                  ctypes.c_void_p(stream.cuda_stream))
    nat.check(rc, "t5e_pack_rows")


def _streamed_words(parts, n: int, dev, out, wait: bool, launch, chunks: int, align: int = 1024):
    """Raw container words in pinned host memory, streamed through the GPU:
    each chunk of cases is copied up as raw words on the upload stream,
    packed into the kernels' row layout on the device (t5e_pack_rows) and
    evaluated on the current stream once its copy has landed, and its result
    words are copied down on the download stream, so that the copies of one
    chunk overlap the packing and evaluation of the others.

    ``parts`` maps a name to (host tensor, rows per case, pack format or
    None): a part has ``per`` = (num, den) rows for each case (a fraction
    for rows shared by the cases of a tile).  ``launch(dev_parts, d_dev, s0, s1)`` evaluates
    cases [s0, s1) on the current stream from the device copies (packed rows
    for the parts with a format, raw words for the others) into ``d_dev``.
    Chunks hold whole multiples of ``align`` cases.  Returns ``out`` when
    ``wait``, else a PendingBatch holding every buffer until its download has
    finished."""
    import torch

    comp = torch.cuda.current_stream(dev)
    up, down = _copy_streams(dev)
    raw = {name: torch.empty(h.shape, dtype=h.dtype, device=dev) for name, (h, _, _) in parts.items()}
    packed = {name: torch.empty((h.shape[0], packing.row_stride(fmt, h.shape[1])), dtype=torch.uint8, device=dev)
              for name, (h, _, fmt) in parts.items() if fmt is not None}
    d_dev = torch.empty(out.shape, dtype=torch.int32, device=dev)
    up.wait_stream(comp)  # the buffers above come from the allocator on the current stream
    step = -(-n // chunks)
    step = (step + align - 1) // align * align
    for s0 in range(0, n, step):
        s1 = min(n, s0 + step)
        with torch.cuda.stream(up):
            for name, (h, per, _) in parts.items():
                r0, r1 = _rows(s0, per), _rows(s1, per)
                raw[name][r0:r1].copy_(h[r0:r1], non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(up)
        comp.wait_event(landed)
        for name, (h, per, fmt) in parts.items():
            if fmt is not None:
                r0, r1 = _rows(s0, per), _rows(s1, per)
                _pack_chunk(raw[name][r0:r1], fmt, packed[name][r0:r1], comp)
        launch({**raw, **packed}, d_dev, s0, s1)
        done = torch.cuda.Event()
        done.record(comp)
        down.wait_event(done)
        with torch.cuda.stream(down):
            out.view(-1)[s0:s1].copy_(d_dev.view(-1)[s0:s1].view(out.dtype), non_blocking=True)
    finished = torch.cuda.Event()
    finished.record(down)
    # the pinned inputs are read by copies on the upload stream that the
    # pinned-memory allocator does not see: they stay referenced until the
    # batch has finished, with the device buffers
    keep = (raw, packed, d_dev, {name: h for name, (h, _, _) in parts.items()})
    if not wait:
        return PendingBatch(out, finished, keep)
    finished.synchronize()
    return out


def _words_batch(selected, desc, a, b, c, scale_a, scale_b, sparse_metadata, a_format, scaling, kind, dev, out,
                 check, generic, wait):
    """mma_dot_batch on raw container words in pinned host memory (every
    per-case array pinned): streamed through the GPU by _streamed_words, the
    operand rows packed on the device."""
    import torch

    n, k = a.shape
    if b.shape != (n, k):
        raise ValueError("A and B dot-product vectors must have equal length")
    if k > nat.MAX_K:
        raise ValueError(f"K={k} exceeds the emulator's maximum of {nat.MAX_K}")
    f16 = desc.d_type == nat.D_F16
    if c is None or not (_pinned(c) and c.numel() == n and c.element_size() == (2 if f16 else 4)):
        raise ValueError("streamed raw words need C as a pinned tensor of N words of the C/D type's width")
    sparse, meta, flags = _prepare(selected, a_format, scaling, kind, k, n, sparse_metadata)
    per_case_meta = meta is not None and not (flags & nat.FLAG_META_BROADCAST)
    if per_case_meta and not _pinned(meta):
        raise ValueError("streamed raw words need per-case metadata in pinned memory")
    one = (1, 1)
    parts = {"a": (a, one, desc.a_format), "b": (b, one, desc.b_format), "c": (c.reshape(n), one, None)}
    scaled = desc.family in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED) and scale_a is not None
    if scaled:
        if not (_pinned(scale_a) and _pinned(scale_b) and scale_a.dim() == 2 and scale_a.shape == scale_b.shape):
            raise ValueError("streamed raw words need [N, blocks] scales in pinned memory")
        if sparse == 0 and scale_a.shape[1] * desc.scale_block < k:
            raise ValueError(selected._scale_cover_error)
        parts["sa"] = (scale_a.view(torch.uint8), one, None)
        parts["sb"] = (scale_b.view(torch.uint8), one, None)
    if per_case_meta:
        parts["meta"] = (meta.view(torch.int32), one, None)
    shared_meta = None if meta is None or per_case_meta else runtime.to_device(meta, dev, torch.int32)
    check = check and sparse != 0
    st_dev = torch.empty(n, dtype=torch.uint8, device=dev) if check else None
    st_host = torch.empty(n, dtype=torch.uint8, pin_memory=True) if check else None
    lib = nat.load()
    fn = lib.t5e_mma_dot_batch_generic if generic else lib.t5e_mma_dot_batch
    handle = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def launch(dp, d_dev, s0, s1):
        db = runtime.DeviceBatch(n=s1 - s0, k=k, a=dp["a"][s0:s1], b=dp["b"][s0:s1], c=dp["c"][s0:s1],
                                 sparse=sparse, flags=flags)
        if scaled:
            db.scale_a, db.scale_b = dp["sa"][s0:s1], dp["sb"][s0:s1]
        if meta is not None:
            db.metadata = dp["meta"][s0:s1] if per_case_meta else shared_meta
        bs = runtime.make_batch_struct(db, d_dev[s0:s1], None if st_dev is None else st_dev[s0:s1])
        nat.check(fn(ctypes.byref(desc), ctypes.byref(bs), handle), "t5e_mma_dot_batch")
        if st_dev is not None:
            down = _copy_streams(dev)[1]
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(dev))
            down.wait_event(ev)
            with torch.cuda.stream(down):
                st_host[s0:s1].copy_(st_dev[s0:s1], non_blocking=True)

    chunks = PIPELINE_CHUNKS if wait or check else PIPELINE_CHUNKS_IN_FLIGHT
    res = _streamed_words(parts, n, dev, out, wait or check, launch, chunks)
    if check:
        st_np = st_host.numpy()
        if st_np.any():
            first = int(np.flatnonzero(st_np)[0])

            def meta_error() -> None:
                record = meta[0] if meta.shape[0] == 1 else meta[first]
                words = np.asarray(record.cpu() if _is_torch(record) else record).astype(np.int64).tolist()
                sparse_active_indices(a_format, k, words[0] if flags & nat.FLAG_META_REPEAT else words,
                                      kind="nvfp4" if (scaling or "").lower() == "ue4m3" else kind)

            _raise_case_status(selected, int(st_np[first]), meta_message=meta_error)
    return res


def _words_tiles(selected, desc, a, b, c, dev, out, generic, wait):
    """mma_batch on raw words in pinned host memory: tiles streamed through
    the GPU by _streamed_words, whole tiles per chunk; each chunk's B is
    transposed on the device (the kernels read B by columns) and packed."""
    import torch

    t, m, k = a.shape
    n = b.shape[2]
    if b.shape[:2] != (t, k):
        raise ValueError(f"A is {m}x{k} but B has {b.shape[1]} rows")
    if k > nat.MAX_K:
        raise ValueError(f"K={k} exceeds the emulator's maximum of {nat.MAX_K}")
    f16 = desc.d_type == nat.D_F16
    total = t * m * n
    if c.numel() != total or c.element_size() != (2 if f16 else 4) or tuple(out.shape) != (t, m, n) \
            or out.element_size() != 4:
        raise ValueError("streamed tiles need C and out as pinned [T, M, N] words")
    per_tile = m * n
    parts = {"a": (a.reshape(t * m, k), (1, n), desc.a_format), "b": (b.reshape(t * k, n), (k, per_tile), None),
             "c": (c.reshape(total), (1, 1), None)}
    lib = nat.load()
    fn = lib.t5e_mma_dot_batch_generic if generic else lib.t5e_mma_dot_batch
    comp = torch.cuda.current_stream(dev)
    handle = ctypes.c_void_p(comp.cuda_stream)

    def launch(dp, d_dev, s0, s1):
        t0, t1 = s0 // per_tile, s1 // per_tile
        cols = dp["b"][t0 * k:t1 * k].view(t1 - t0, k, n).transpose(1, 2).contiguous().view((t1 - t0) * n, k)
        b_rows = torch.empty(((t1 - t0) * n, packing.row_stride(desc.b_format, k)), dtype=torch.uint8, device=dev)
        _pack_chunk(cols, desc.b_format, b_rows, comp)
        db = runtime.DeviceBatch(n=s1 - s0, k=k, a=dp["a"][t0 * m:t1 * m], b=b_rows, c=dp["c"][s0:s1],
                                 tile_m=m, tile_n=n)
        bs = runtime.make_batch_struct(db, d_dev.view(-1)[s0:s1], None)
        nat.check(fn(ctypes.byref(desc), ctypes.byref(bs), handle), "t5e_mma_dot_batch")

    chunks = PIPELINE_CHUNKS if wait else PIPELINE_CHUNKS_IN_FLIGHT
    return _streamed_words(parts, total, dev, out, wait, launch, chunks, align=per_tile)


def _rows(case: int, per) -> int:
    """First row of a case in an array with ``per`` = (num, den) rows per
    case (fewer than one for rows shared by the cases of a tile)."""
    return case * per[0] // per[1]


def mma_dot_batch(
    a,
    b,
    c=None,
    *,
    model: ScalarModel | None = None,
    a_format: str = "tf32",
    b_format: str | None = None,
    d_type: str = "f32",
    saturate: bool = False,
    scaling: str | None = None,
    scale_vec: int | None = None,
    kind: str | None = None,
    scale_a=None,
    scale_b=None,
    sparse_metadata=None,
    device=None,
    check: bool = True,
    generic: bool = False,
    out=None,
    wait: bool = True,
):
    """N independent ``mma_dot`` evaluations in one kernel launch.

    ``a``, ``b``: [N, K] raw container words (numpy arrays or torch tensors,
    host or CUDA) or ``PackedRows``; sparse calls pass full logical-K rows
    (or a compressed ``PackedRows`` A).  ``c``: [N] words or None (zeros).
    ``scale_a``/``scale_b``: [N, blocks] 8-bit scales or None (the reference
    defaults).  ``sparse_metadata``: an int (repeated over K) or a word
    sequence shared by every case, or an array of N ints / [N, W] words.
    Returns the N result words: a uint32 numpy array for host inputs, a
    torch.uint32 CUDA tensor for device inputs, or ``out`` (a host array or
    pinned tensor of N 32-bit words) filled in place.  With ``check`` the
    per-case ValueErrors of the reference are raised.

    ``wait=False`` returns a ``PendingBatch`` instead; its ``wait()`` returns
    what the call would have.  A batch streamed from pinned host memory
    (``PackedRows`` over pinned tensors and a pinned ``out``) then returns
    as soon as its copies and kernels are queued, so that the next batch's
    upload follows on the link without a gap.  Sparse batches with
    ``check`` need their status bytes on the host and complete before
    returning, as do all other inputs.
    """
    res = _mma_dot_batch(a, b, c, model=model, a_format=a_format, b_format=b_format, d_type=d_type,
                         saturate=saturate, scaling=scaling, scale_vec=scale_vec, kind=kind, scale_a=scale_a,
                         scale_b=scale_b, sparse_metadata=sparse_metadata, device=device, check=check,
                         generic=generic, out=out, wait=wait)
    if not wait and not isinstance(res, PendingBatch):
        res = PendingBatch(res)
    return res


def _mma_dot_batch(a, b, c, *, model, a_format, b_format, d_type, saturate, scaling, scale_vec, kind, scale_a,
                   scale_b, sparse_metadata, device, check, generic, out, wait):
    import torch

    selected = model or make_model(a_format, b_format, d_type=d_type, saturate=saturate, scaling=scaling,
                                   scale_vec=scale_vec, kind=kind)
    if not isinstance(selected, _ModelBase):
        raise TypeError("model must come from tcgen05_b200.make_model or its model classes")
    desc = selected.descriptor()
    dev = runtime.require_device(device)
    if (_raw_words_pinned(a) and _raw_words_pinned(b) and out is not None and _pinned(out)
            and out.element_size() == 4 and out.numel() == a.shape[0] and a.shape[0] >= PIPELINE_MIN_CASES):
        return _words_batch(selected, desc, a, b, c, scale_a, scale_b, sparse_metadata, a_format, scaling, kind,
                            dev, out, check, generic, wait)
    host_result = not ((_is_torch(a) and a.is_cuda) or (isinstance(a, PackedRows) and _is_torch(a.data)
                                                        and a.data.is_cuda))
    streamed = (isinstance(a, PackedRows) and isinstance(b, PackedRows) and _pinned(a.data) and _pinned(b.data)
                and a.data.dim() == 2 and b.data.dim() == 2)
    if streamed:  # copied chunk by chunk below, or in one piece if the batch does not qualify
        a_rows = b_rows = None
        n, ka = a.data.shape[0], a.k
        nb, k = b.data.shape[0], b.k
    else:
        a_rows, n, ka = _operand_rows(a, desc.a_format, dev, "A")
        b_rows, nb, k = _operand_rows(b, desc.b_format, dev, "B")
    a_compressed = isinstance(a, PackedRows) and a.compressed
    if nb != n:
        raise ValueError("A and B must hold the same number of cases")
    if ka != k and not a_compressed:
        raise ValueError("A and B dot-product vectors must have equal length")
    if k < 1:
        raise ValueError("a dot product must contain at least one element")
    if k > nat.MAX_K:
        raise ValueError(f"K={k} exceeds the emulator's maximum of {nat.MAX_K}")
    sparse, meta, flags = _prepare(selected, a_format, scaling, kind, k, n, sparse_metadata)
    if (streamed and out is not None and _pinned(out) and out.element_size() == 4 and n >= PIPELINE_MIN_CASES
            and c is not None and _pinned(c) and c.element_size() == (2 if desc.d_type == nat.D_F16 else 4)
            and (scale_a is None or (_pinned(scale_a) and _pinned(scale_b) and scale_a.dim() == 2
                                     and scale_a.shape == scale_b.shape))
            and (meta is None or (flags & nat.FLAG_META_BROADCAST) or _pinned(meta))):
        if scale_a is not None and sparse == 0 and scale_a.shape[1] * desc.scale_block < k:
            raise ValueError(selected._scale_cover_error)

        def meta_error_p(first: int) -> None:
            record = meta[0] if meta.shape[0] == 1 else meta[first]
            words = np.asarray(record.cpu() if _is_torch(record) else record).astype(np.int64).tolist()
            sparse_active_indices(a_format, k, words[0] if flags & nat.FLAG_META_REPEAT else words,
                                  kind="nvfp4" if (scaling or "").lower() == "ue4m3" else kind)

        sa_p = scale_a if desc.family in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED) else None
        sb_p = scale_b if sa_p is not None else None
        return _pipelined_batch(selected, desc, a, b, c.reshape(n), sa_p, sb_p, meta, flags, sparse, k, n, dev, out,
                                check, meta_error_p, generic, wait)
    if streamed:
        a_rows, _, _ = _operand_rows(a, desc.a_format, dev, "A")
        b_rows, _, _ = _operand_rows(b, desc.b_format, dev, "B")
    if c is None:
        c_dev = torch.zeros(n, dtype=torch.int16 if desc.d_type == nat.D_F16 else torch.int32, device=dev)
    elif _is_torch(c):
        c_dev = _c_words_on_device(c.reshape(n).to(dev, non_blocking=True), desc.d_type == nat.D_F16)
    else:
        c_host = _c_host(c, n, selected)
        c_dev = runtime.to_device(c_host.view(np.int16) if c_host.dtype == np.uint16 else c_host, dev)
    if (scale_a is None) != (scale_b is None):
        raise ValueError("scale_a and scale_b must be supplied together")
    sa = sb = None
    if scale_a is not None and desc.family in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED):
        sa = scale_a if _is_torch(scale_a) else _scales_np(scale_a, "scale_a")
        sb = scale_b if _is_torch(scale_b) else _scales_np(scale_b, "scale_b")
        if sa.ndim == 1:
            sa = sa.reshape(1, -1).repeat(n, 0) if not _is_torch(sa) else sa.reshape(1, -1).expand(n, -1)
        if sb.ndim == 1:
            sb = sb.reshape(1, -1).repeat(n, 0) if not _is_torch(sb) else sb.reshape(1, -1).expand(n, -1)
        if sa.shape[1] != sb.shape[1]:
            raise ValueError(selected._scale_count_error)
        if sparse == 0 and sa.shape[1] * desc.scale_block < k:
            raise ValueError(selected._scale_cover_error)

    def meta_error(first: int) -> None:
        record = meta[0] if meta.shape[0] == 1 else meta[first]
        words = np.asarray(record.cpu() if _is_torch(record) else record).astype(np.int64).tolist()
        sparse_active_indices(a_format, k, words[0] if flags & nat.FLAG_META_REPEAT else words,
                              kind="nvfp4" if (scaling or "").lower() == "ue4m3" else kind)

    d = _run(selected, a_rows, b_rows, c_dev, k, dev, n=n, tile_m=1, tile_n=1, scale_a=sa, scale_b=sb,
             sparse=sparse, meta=meta, flags=flags, a_compressed=a_compressed, check=check, meta_error=meta_error,
             generic=generic)
    if out is not None:
        if _is_torch(out):
            out.copy_(d.view(out.dtype) if out.element_size() == 4 else d, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        else:
            out[...] = d.cpu().numpy().view(np.uint32)
        return out
    if host_result:
        return d.cpu().numpy().view(np.uint32).copy()
    return d.view(torch.uint32)


def mma_batch(
    a,
    b,
    c=None,
    *,
    model: ScalarModel | None = None,
    a_format: str = "tf32",
    b_format: str | None = None,
    d_type: str = "f32",
    saturate: bool = False,
    scaling: str | None = None,
    scale_vec: int | None = None,
    kind: str | None = None,
    scale_a=None,
    scale_b=None,
    sparse_metadata=None,
    device=None,
    check: bool = True,
    generic: bool = False,
    out=None,
    wait: bool = True,
):
    """T independent row-major tiles ``D[t] = A[t] @ B[t] + C[t]`` in one
    launch: ``a`` [T, M, K], ``b`` [T, K, N], ``c`` [T, M, N] raw words;
    ``scale_a`` [T, M, blocks], ``scale_b`` [T, N, blocks]; one metadata
    value shared by all tiles (as ``mma``), or an array of T ints / [T, W]
    words.  Returns [T, M, N] words (numpy for host inputs, torch.uint32 on
    the device for device inputs).

    Unscaled dense tiles whose A, B and C are raw words in pinned host
    memory, with a pinned [T, M, N] ``out`` of 32-bit words, are streamed
    through the GPU a group of tiles at a time (copies up, packing and
    evaluation on the device, copies down, overlapped); ``wait=False`` then
    returns a PendingBatch, as for mma_dot_batch."""
    import torch

    selected = model or make_model(a_format, b_format, d_type=d_type, saturate=saturate, scaling=scaling,
                                   scale_vec=scale_vec, kind=kind)
    desc = selected.descriptor()
    dev = runtime.require_device(device)
    if (_pinned(a) and _pinned(b) and c is not None and _pinned(c) and out is not None and _pinned(out)
            and a.dim() == 3 and b.dim() == 3 and scale_a is None and sparse_metadata is None
            and a.dtype in (torch.int32, torch.uint32) and b.dtype in (torch.int32, torch.uint32)):
        return _words_tiles(selected, desc, a, b, c, dev, out, generic, wait)
    if out is not None or not wait:
        raise ValueError("out and wait=False apply to pinned host tiles of raw words (unscaled, dense)")
    on_device = _is_torch(a) and a.is_cuda
    if on_device:
        t, m, k = a.shape
        n = b.shape[2]
        a_rows = packing.pack_rows_device(a.reshape(t * m, k).to(dev), desc.a_format)
        b_rows = packing.pack_rows_device(b.to(dev).transpose(1, 2).reshape(t * n, k), desc.b_format)
    else:
        aw = _words_np(a, "A")
        bw = _words_np(b, "B")
        t, m, k = aw.shape
        n = bw.shape[2]
        if bw.shape[:2] != (t, k):
            raise ValueError(f"A is {m}x{k} but B has {bw.shape[1]} rows")
        a_rows = runtime.to_device(packing.pack_rows(aw.reshape(t * m, k), desc.a_format), dev)
        b_rows = runtime.to_device(
            packing.pack_rows(np.ascontiguousarray(bw.transpose(0, 2, 1)).reshape(t * n, k), desc.b_format), dev)
    if k > nat.MAX_K:
        raise ValueError(f"K={k} exceeds the emulator's maximum of {nat.MAX_K}")
    total = t * m * n
    if c is None:
        c_dev = torch.zeros(total, dtype=torch.int16 if desc.d_type == nat.D_F16 else torch.int32, device=dev)
    elif _is_torch(c) and c.is_cuda:
        c_dev = c.reshape(total).to(dev)
        want = 2 if desc.d_type == nat.D_F16 else 4
        if c_dev.element_size() != want:
            c_dev = c_dev.to(torch.int64).bitwise_and(0xFFFF if want == 2 else 0xFFFFFFFF)
            c_dev = c_dev.to(torch.int32).to(torch.int16) if want == 2 else c_dev.to(torch.int32)
    else:
        c_host = _c_host(np.asarray(c).reshape(total), total, selected)
        c_dev = runtime.to_device(c_host.view(np.int16) if c_host.dtype == np.uint16 else c_host, dev)
    sa = sb = None
    if (scale_a is None) != (scale_b is None):
        raise ValueError("scale_a and scale_b must be supplied together")
    if scale_a is not None and desc.family in (nat.FAMILY_NVFP4, nat.FAMILY_BLOCK_SCALED):
        sa = scale_a.reshape(t * m, -1) if _is_torch(scale_a) else _scales_np(scale_a, "scale_a").reshape(t * m, -1)
        sb = scale_b.reshape(t * n, -1) if _is_torch(scale_b) else _scales_np(scale_b, "scale_b").reshape(t * n, -1)
        if sa.shape[1] != sb.shape[1]:
            raise ValueError(selected._scale_count_error)
        if sparse_metadata is None and sa.shape[1] * desc.scale_block < k:
            raise ValueError(selected._scale_cover_error)
    elif scale_a is not None:
        _scales_np(scale_a, "scale_a")
        _scales_np(scale_b, "scale_b")
    sparse, meta, flags = 0, None, 0
    if sparse_metadata is not None:
        if isinstance(sparse_metadata, (int, np.integer, list, tuple)):
            sparse, meta, flags = _prepare(selected, a_format, scaling, kind, k, t * m, sparse_metadata)
        else:
            per_tile = sparse_metadata if _is_torch(sparse_metadata) else _words_np(sparse_metadata, "metadata")
            sparse, meta, flags = _prepare(selected, a_format, scaling, kind, k, t, per_tile)
            # one record per tile -> one record per A row of that tile
            meta = meta.repeat_interleave(m, 0) if _is_torch(meta) else np.repeat(meta, m, axis=0)

    def meta_error(first: int) -> None:
        row = (first // (m * n)) * m + (first % (m * n)) // n
        record = meta[0] if meta.shape[0] == 1 else meta[row]
        words = np.asarray(record.cpu() if _is_torch(record) else record).astype(np.int64).tolist()
        sparse_active_indices(a_format, k, words[0] if flags & nat.FLAG_META_REPEAT else words,
                              kind="nvfp4" if (scaling or "").lower() == "ue4m3" else kind)

    d = _run(selected, a_rows, b_rows, c_dev, k, dev, n=total, tile_m=m, tile_n=n, scale_a=sa, scale_b=sb,
             sparse=sparse, meta=meta, flags=flags, a_compressed=False, check=check, meta_error=meta_error,
             generic=generic)
    if on_device:
        return d.view(torch.uint32).reshape(t, m, n)
    return d.cpu().numpy().view(np.uint32).reshape(t, m, n).copy()

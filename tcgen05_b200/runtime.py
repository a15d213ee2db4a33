"""Device plumbing: CUDA devices, streams and buffers through PyTorch, and the
one call that hands a batch to the emulator library.

PyTorch only provides memory, copies and the stream; every result word is
computed by the library's sm_100a kernels.  There is no CPU path: without a
CUDA device or without the built library these functions raise.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native as nat


def _torch():
    import torch

    return torch


def require_device(device=None):
    """The torch.device to run on; raises when no CUDA device is present."""
    torch = _torch()
    if not torch.cuda.is_available():
        raise RuntimeError(
            "tcgen05_b200 evaluates MMA arithmetic on a CUDA device (B200, sm_100a) and has no CPU "
            "fallback; no CUDA device is available"
        )
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    d = torch.device(device)
    if d.type != "cuda":
        raise RuntimeError(f"tcgen05_b200 runs on CUDA devices, not {d}")
    return d if d.index is not None else torch.device("cuda", torch.cuda.current_device())


def current_stream_handle(device) -> int:
    torch = _torch()
    return torch.cuda.current_stream(device).cuda_stream


def to_device(x, device, dtype=None):
    """numpy array or torch tensor -> contiguous torch tensor on `device`."""
    torch = _torch()
    if isinstance(x, torch.Tensor):
        t = x
    else:
        arr = np.ascontiguousarray(x)
        if arr.dtype == np.uint32:
            t = torch.from_numpy(arr.view(np.int32))
        else:
            t = torch.from_numpy(arr)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.to(device, non_blocking=True).contiguous()


@dataclass
class DeviceBatch:
    """Device-resident operands of one launch (see t5e_batch in include/t5e.h)."""

    n: int
    k: int
    a: object            # uint8 [rows, a_stride]
    b: object            # uint8 [rows, b_stride]
    c: object            # int32 [n] (F32/S32 words) or int16 [n] (F16 words)
    scale_a: object = None  # uint8 [rows, nscale]
    scale_b: object = None
    metadata: object = None  # int32 [rows, meta_words] (uint32 words)
    flags: int = 0
    tile_m: int = 1
    tile_n: int = 1
    sparse: int = 0


def make_batch_struct(db: DeviceBatch, d, status) -> nat.Batch:
    torch = _torch()
    bs = nat.Batch()
    bs.n = db.n
    bs.k = db.k
    bs.flags = db.flags
    bs.tile_m = db.tile_m
    bs.tile_n = db.tile_n
    bs.sparse = db.sparse
    bs.a = db.a.data_ptr()
    bs.a_stride = db.a.shape[1]
    bs.b = db.b.data_ptr()
    bs.b_stride = db.b.shape[1]
    bs.c = db.c.data_ptr()
    bs.c_bytes = 2 if db.c.dtype in (torch.int16, torch.uint16) else 4
    if db.scale_a is not None:
        bs.nscale = db.scale_a.shape[1]
        bs.scale_a = db.scale_a.data_ptr()
        bs.scale_b = db.scale_b.data_ptr()
    else:
        bs.nscale = 0
        bs.scale_a = None
        bs.scale_b = None
    if db.metadata is not None:
        bs.metadata = db.metadata.data_ptr()
        bs.meta_words = db.metadata.shape[1]
    else:
        bs.metadata = None
        bs.meta_words = 0
    bs.d = d.data_ptr()
    bs.status = status.data_ptr() if status is not None else None
    return bs


def launch(model: nat.Model, db: DeviceBatch, *, d=None, status=True, generic=False, stream=None):
    """Run the emulator over a device batch on the current stream of its
    device.  Returns (d, status) device tensors (status None when not asked)."""
    torch = _torch()
    device = db.a.device
    if d is None:
        d = torch.empty(db.n, dtype=torch.int32, device=device)
    st = torch.empty(db.n, dtype=torch.uint8, device=device) if status else None
    bs = make_batch_struct(db, d, st)
    lib = nat.load()
    fn = lib.t5e_mma_dot_batch_generic if generic else lib.t5e_mma_dot_batch
    handle = current_stream_handle(device) if stream is None else stream
    rc = fn(ctypes.byref(model), ctypes.byref(bs), ctypes.c_void_p(handle))
    nat.check(rc, "t5e_mma_dot_batch")
    return d, st

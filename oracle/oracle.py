"""TEST INFRASTRUCTURE ONLY -- ctypes wrapper of the C restatement of the
tcgen05_model arithmetic (oracle/t5e_oracle.c).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
bench.py use this module, as the parity reference and the timed CPU baseline.
The product path (tcgen05_b200) never imports it.

``mma_dot_batch`` takes the public ``mma_dot`` arguments for N cases
(logical-K words, per-case scales and metadata) and returns the result
words with the per-case status (0, or a negative code where the reference
raises ValueError).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_t5e.so"

FORMATS = {"tf32": 0, "bf16": 1, "f16": 2, "e4m3": 3, "e5m2": 4, "e2m3": 5, "e3m2": 6, "e2m1": 7, "u8": 8, "s8": 9}
ALIASES = {"fp8": "e4m3", "fp8e4m3": "e4m3", "fp8e5m2": "e5m2", "fp6e2m3": "e2m3", "fp6e3m2": "e3m2",
           "fp4": "e2m1", "fp4e2m1": "e2m1"}
D_TYPES = {"f32": 0, "f16": 1, "s32": 2}
SCALINGS = {None: 0, "ue8m0": 1, "ue4m3": 2}
KINDS = {None: 0, "mxf8f6f4": 1, "mxf4": 2, "mxf4nvf4": 3, "nvfp4": 4}

OK = 0
ERR_DESCRIPTOR = -1
ERR_RANGE = -100


class Desc(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in
                ("a_fmt", "b_fmt", "d_type", "saturate", "scaling", "scale_vec", "kind")]


_lib = None


def build() -> Path:
    """Compile the restatement with gcc (oracle/Makefile) when stale."""
    src = HERE / "t5e_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "ORACLE_CC=gcc"], check=True)
    return LIB_PATH


def load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.oracle_mma_dot_batch.restype = ctypes.c_int
        lib.oracle_mma_dot_batch.argtypes = [
            ctypes.POINTER(Desc), ctypes.c_int64, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ]
        lib.oracle_check_descriptor.restype = ctypes.c_int
        lib.oracle_check_descriptor.argtypes = [ctypes.POINTER(Desc)]
        lib.oracle_sparse_active.restype = ctypes.c_int
        lib.oracle_sparse_active.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        _lib = lib
    return _lib


def _fmt(name):
    if name is None:
        return -1
    n = name.lower().replace("_", "").replace("-", "")
    n = ALIASES.get(n, n)
    return FORMATS.get(n, 99)


def make_desc(a_format="tf32", b_format=None, d_type="f32", saturate=False, scaling=None, scale_vec=None,
              kind=None) -> Desc:
    d = Desc()
    d.a_fmt = _fmt(a_format)
    d.b_fmt = _fmt(b_format)
    d.d_type = D_TYPES.get(d_type.lower(), 99)
    d.saturate = 1 if saturate else 0
    d.scaling = SCALINGS.get(None if scaling is None else scaling.lower(), 99)
    d.scale_vec = 0 if scale_vec is None else int(scale_vec)
    d.kind = KINDS.get(None if kind is None else kind.lower(), 99)
    return d


def _u32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.uint32))


def default_threads() -> int:
    return len(os.sched_getaffinity(0))


def mma_dot_batch(a, b, c=None, *, scale_a=None, scale_b=None, sparse_metadata=None, meta_is_int=False,
                  threads=None, **desc):
    """Evaluate N public mma_dot calls on the CPU; returns (d, status)."""
    lib = load()
    a = _u32(a)
    b = _u32(b)
    n, k = a.shape
    c = np.zeros(n, dtype=np.uint32) if c is None else _u32(c).reshape(n)
    d = np.zeros(n, dtype=np.uint32)
    st = np.zeros(n, dtype=np.int32)
    sa = None if scale_a is None else _u32(scale_a).reshape(n, -1)
    sb = None if scale_b is None else _u32(scale_b).reshape(n, -1)
    meta = None if sparse_metadata is None else _u32(sparse_metadata).reshape(n, -1)
    dd = make_desc(**desc)
    rc = lib.oracle_mma_dot_batch(
        ctypes.byref(dd), n, k, a.ctypes.data, b.ctypes.data, c.ctypes.data,
        None if sa is None else sa.ctypes.data, 0 if sa is None else sa.shape[1],
        None if sb is None else sb.ctypes.data, 0 if sb is None else sb.shape[1],
        None if meta is None else meta.ctypes.data, 0 if meta is None else meta.shape[1], 1 if meta_is_int else 0,
        d.ctypes.data, st.ctypes.data, threads or default_threads())
    if rc == ERR_RANGE:
        raise RuntimeError("oracle left its exact range")
    if rc < 0:
        st[:] = rc
    return d, st


def check_descriptor(**desc) -> int:
    return load().oracle_check_descriptor(ctypes.byref(make_desc(**desc)))


def eval_cases(cases, threads=None):
    """Oracle words for a workloads.Cases batch (raises on any failing case)."""
    d, st = mma_dot_batch(cases.a, cases.b, cases.c, scale_a=cases.scale_a, scale_b=cases.scale_b,
                          sparse_metadata=cases.meta, threads=threads, **cases.desc)
    if (st != 0).any():
        i = int(np.flatnonzero(st)[0])
        raise ValueError(f"oracle status {int(st[i])} at case {i}")
    return d

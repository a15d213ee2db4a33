"""tcgen05_b200 -- a B200-native (sm_100a) batched emulator of NVIDIA
Blackwell tcgen05 MMA arithmetic, bit-exact with the tcgen05_model
reference package and a drop-in for its API.

Scalar and matrix calls (``mma_dot``, ``mma``, ``make_model(...).eval``)
keep the reference's signatures and errors; ``mma_dot_batch`` and
``mma_batch`` evaluate millions of independent dot products or tiles per
kernel launch.  Every result word is computed by hand-written integer CUDA
kernels in ``tcgen05_b200/_lib/libt5e.so``; there is no CPU fallback.
"""

from .formats import bits_to_f32, f32_to_bits
from .model import (
    DotProduct,
    ScalarModel,
    Tcgen05BlockScaledMmaModel,
    Tcgen05I8S32MmaModel,
    Tcgen05MixedRawWindowMmaModel,
    Tcgen05RawWindowNvfp4MmaModel,
    make_model,
    normalize_format,
)
from .simulator import PackedRows, PendingBatch, mma, mma_batch, mma_dot, mma_dot_batch, sparse_active_indices

__all__ = [
    "DotProduct",
    "PackedRows",
    "PendingBatch",
    "ScalarModel",
    "Tcgen05BlockScaledMmaModel",
    "Tcgen05I8S32MmaModel",
    "Tcgen05MixedRawWindowMmaModel",
    "Tcgen05RawWindowNvfp4MmaModel",
    "bits_to_f32",
    "f32_to_bits",
    "make_model",
    "mma",
    "mma_batch",
    "mma_dot",
    "mma_dot_batch",
    "normalize_format",
    "sparse_active_indices",
]

"""The ctypes binding shown in INTEGRATION.md (what tcgen05_model would add)
matches the library: struct layouts and descriptors on the CPU, results on
the GPU."""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

import numpy as np
import pytest

from tcgen05_b200 import _native as nat

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def stub():
    text = (REPO / "INTEGRATION.md").read_text()
    blocks = re.findall(r"```python\n(# tcgen05_model/_t5e\.py.*?)```", text, flags=re.S)
    assert len(blocks) == 1, "INTEGRATION.md must hold exactly one tcgen05_model/_t5e.py block"
    nat.load()
    old = os.environ.get("T5E_LIB")
    os.environ["T5E_LIB"] = str(nat.LIB_PATH)
    try:
        ns: dict = {"__name__": "tcgen05_model_t5e_stub"}
        exec(compile(blocks[0], "INTEGRATION.md:_t5e.py", "exec"), ns)
    finally:
        if old is None:
            os.environ.pop("T5E_LIB", None)
        else:
            os.environ["T5E_LIB"] = old
    return ns


def _layout(cls):
    return [(name, getattr(cls, name).offset, getattr(cls, name).size) for name, _ in cls._fields_]


def test_stub_struct_layouts_match_the_library(stub):
    assert _layout(stub["t5e_model"]) == _layout(nat.Model)
    assert _layout(stub["t5e_batch"]) == _layout(nat.Batch)
    assert ctypes.sizeof(stub["t5e_batch"]) == ctypes.sizeof(nat.Batch)


def test_stub_format_tables_match(stub):
    assert stub["FMT"] == nat.FORMAT_IDS
    assert stub["BITS"] == nat.FORMAT_BITS
    assert stub["NONE"] == nat.NONE


@pytest.mark.parametrize("a,b,d", [("tf32", "tf32", "f32"), ("bf16", "bf16", "f32"), ("f16", "f16", "f32"),
                                   ("f16", "f16", "f16"), ("e4m3", "e5m2", "f32"), ("e4m3", "e5m2", "f16"),
                                   ("e2m3", "e2m1", "f16"), ("e3m2", "e3m2", "f32")])
def test_stub_descriptor_equals_make_model(stub, a, b, d):
    import tcgen05_b200 as t5

    want = t5.make_model(a, b, d_type=d).descriptor()
    got = stub["raw_window_desc"](a, b, d)
    for name, _ in nat.Model._fields_:
        assert getattr(got, name) == getattr(want, name), (a, b, d, name)


@pytest.mark.gpu
@pytest.mark.parametrize("a,b,d,k", [("e4m3", "e5m2", "f32", 32), ("e4m3", "e5m2", "f16", 32),
                                     ("tf32", "tf32", "f32", 8), ("bf16", "bf16", "f32", 16)])
def test_stub_eval_batch_matches_oracle(stub, a, b, d, k):
    from oracle import oracle
    from tcgen05_b200 import workloads

    rng = np.random.default_rng(7)
    n = 4096
    a_w = workloads.format_words(a, rng, (n, k))
    b_w = workloads.format_words(b, rng, (n, k))
    c_w = workloads.finite_f16_c(rng, n) if d == "f16" else rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    got = stub["eval_batch"](stub["raw_window_desc"](a, b, d), a_w, b_w, c_w)
    want, status = oracle.mma_dot_batch(a_w, b_w, c_w, a_format=a, b_format=b, d_type=d)
    assert not status.any()
    assert np.array_equal(got, want)

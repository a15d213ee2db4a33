"""The C-ABI library builds for sm_100a, loads without a GPU, exports every
symbol include/t5e.h declares, and agrees with the header on struct
layouts.  Argument validation runs on the host and never reaches a launch."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from tcgen05_b200 import _native as nat

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "t5e.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(t5e_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = nat.load()
    declared = declared_functions()
    assert declared, "no declarations parsed from include/t5e.h"
    assert sorted(declared) == sorted(nat.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(nat.LIB_PATH)], capture_output=True, text=True).stdout
    for name in declared:
        assert re.search(rf"\bT {name}\b", out), name
    assert lib.t5e_abi_version() == nat.ABI_VERSION


def test_library_targets_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", str(nat.LIB_PATH)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    archs = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert archs == {"100a"}, archs


def test_struct_layouts_match_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "t5e.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu\\n\", sizeof(t5e_model), sizeof(t5e_batch),"
        " offsetof(t5e_batch, a), offsetof(t5e_batch, d), offsetof(t5e_batch, status));return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    want = [ctypes.sizeof(nat.Model), ctypes.sizeof(nat.Batch), nat.Batch.a.offset, nat.Batch.d.offset,
            nat.Batch.status.offset]
    assert [int(x) for x in got] == want


def _batch(**kw):
    b = nat.Batch()
    b.n = 4
    b.k = 8
    b.tile_m = b.tile_n = 1
    b.a = b.b = b.c = b.d = 4096  # never dereferenced: validation fails first
    b.a_stride = b.b_stride = 32
    b.c_bytes = 4
    for key, value in kw.items():
        setattr(b, key, value)
    return b


def _model(**kw):
    m = nat.Model()
    m.family = nat.FAMILY_RAW_WINDOW
    m.window_bits = 25
    m.window_floor = nat.NONE
    for key, value in kw.items():
        setattr(m, key, value)
    return m


@pytest.mark.parametrize("bad", [
    dict(k=0), dict(k=nat.MAX_K + 1), dict(a_stride=30), dict(b_stride=8), dict(tile_m=0), dict(c_bytes=3),
    dict(a=None), dict(sparse=7, metadata=4096, meta_words=1), dict(sparse=2, metadata=None, meta_words=1),
])
def test_invalid_batches_are_rejected_before_launch(bad):
    lib = nat.load()
    rc = lib.t5e_mma_dot_batch(ctypes.byref(_model()), ctypes.byref(_batch(**bad)), None)
    assert rc in (nat.ERR_INVALID, nat.ERR_K_RANGE)


@pytest.mark.parametrize("bad", [
    dict(family=9), dict(window_bits=40), dict(a_format=nat.FMT_U8),
    dict(family=nat.FAMILY_BLOCK_SCALED, a_format=nat.FMT_E2M1, b_format=nat.FMT_E2M1, scale_format=nat.SCALE_UE8M0,
         scale_block=32, c_merge_group=48, window_bits=39, c_merge_bits=35),
    dict(family=nat.FAMILY_NVFP4, a_format=nat.FMT_E2M1, b_format=nat.FMT_E2M1, scale_block=64, c_merge_group=16),
])
def test_unsupported_descriptors_are_rejected(bad):
    lib = nat.load()
    rc = lib.t5e_mma_dot_batch(ctypes.byref(_model(**bad)), ctypes.byref(_batch()), None)
    assert rc == nat.ERR_UNSUPPORTED


def test_empty_batch_is_a_no_op():
    lib = nat.load()
    assert lib.t5e_mma_dot_batch(ctypes.byref(_model()), ctypes.byref(_batch(n=0)), None) == nat.OK


def test_issue_probe_rejects_bad_arguments_without_a_device():
    lib = nat.load()
    count = ctypes.c_uint64(0)
    assert lib.t5e_issue_probe(3, 1, ctypes.byref(count), None) == nat.ERR_INVALID
    assert lib.t5e_issue_probe(-1, 1, ctypes.byref(count), None) == nat.ERR_INVALID
    assert lib.t5e_issue_probe(0, 0, ctypes.byref(count), None) == nat.ERR_INVALID
    assert lib.t5e_issue_probe(0, (1 << 20) + 1, ctypes.byref(count), None) == nat.ERR_INVALID
    assert lib.t5e_issue_probe(1, 1, None, None) == nat.ERR_INVALID
    assert count.value == 0


@pytest.mark.gpu
def test_issue_probe_counts_its_instructions():
    """Two blocks of 1024 threads per SM, 256 probe instructions per thread
    and iteration, for each pipe (ALU, FMA, FP64)."""
    import torch

    lib = nat.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for pipe in (0, 1, 2):
        count = ctypes.c_uint64(0)
        assert lib.t5e_issue_probe(pipe, 4, ctypes.byref(count), None) == nat.OK
        torch.cuda.synchronize()
        assert count.value == sms * 2 * 32 * 4 * 256


def test_staged_async_needs_an_event_without_a_device():
    lib = nat.load()
    assert lib.t5e_mma_dot_batch_staged_async(None, None, None, 0, None, None) == nat.ERR_INVALID

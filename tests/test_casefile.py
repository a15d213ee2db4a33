"""MMAPRB1 / MMAPRO1 case files of the reference hardware harness: record
layouts round-trip, every op maps to the same arithmetic as the validation
path it probes (checked with the oracle), the report fields count
mismatches and position failures, and -- on a GPU -- the emulator evaluates
input files word for word like the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from tcgen05_b200 import casefile, sweep, workloads

PATHS = {p.name: p for p in workloads.validation_paths()}

# (op, layout index, validation path)
OP_PATHS = [
    (2, 0, "dense-tf32"), (3, 0, "dense-bf16"), (4, 0, "dense-e4m3"), (5, 0, "dense-nvfp4"),
    (6, 0, "sparse-tf32"), (7, 0, "sparse-bf16"), (8, 0, "sparse-fp8"), (9, 0, "sparse-nvfp4"),
    (10, 0, "dense-f16"), (11, 0, "sparse-f16"),
    (12, 0, "dense-e5m2"), (13, 0, "dense-e2m3"), (14, 0, "dense-e3m2"), (15, 0, "dense-e2m1"),
    (16, 0, "sparse-e5m2"), (17, 0, "sparse-e2m3"), (18, 0, "sparse-e3m2"), (19, 0, "sparse-e2m1"),
    (20, 0, "dense-mx-e4m3"), (21, 0, "dense-mx-e5m2"), (22, 0, "dense-mx-e2m3"), (23, 0, "dense-mx-e3m2"),
    (24, 0, "dense-mx-e2m1"), (20, 1, "sparse-mx-e4m3"), (23, 1, "sparse-mx-e3m2"),
    (25, 0, "dense-mxf4"), (26, 0, "dense-mxf4nvf4-2x"), (27, 0, "dense-mxf4nvf4-4x"),
    (25, 1, "sparse-mxf4"), (27, 1, "sparse-mxf4nvf4-4x"),
    (37, 0, "dense-mxf4nvf4-4x-ue4m3"), (38, 0, "sparse-mxf4nvf4-4x-ue4m3"),
    (29, 0, "i8-u8-u8-wrap"), (32, 0, "i8-s8-s8-wrap"), (35, 0, "i8-u8-s8-saturate"),
]


def _fields(layout, cases):
    n = cases.n
    f = {}
    for name, width in layout.fields:
        f[name] = np.zeros((n, width), dtype=np.uint32)
    f["a"][:, :cases.k] = cases.a
    f["b"][:, :cases.k] = cases.b
    f["c"][:, 0] = cases.c
    if "scale_a" in f:
        unit = 0x38 if layout.descriptor.get("scaling") == "ue4m3" else 0x7F
        f["scale_a"][:] = unit
        f["scale_b"][:] = unit
        f["scale_a"][:, :cases.scale_a.shape[1]] = cases.scale_a
        f["scale_b"][:, :cases.scale_b.shape[1]] = cases.scale_b
    if "meta" in f:
        f["meta"][:, 0] = cases.meta[:, 0]
    if "meta_hi" in f:
        f["meta_hi"][:, 0] = cases.meta[:, 1]
    if layout.mx_formats:
        code = casefile.MX_FORMAT_CODES[cases.desc["a_format"]]
        f["fmt_a"][:] = code
        f["fmt_b"][:] = code
        f["n"][:] = 8
        f["cta_group"][:] = 1
        f["m"][:] = 128
    return f


def _expected(layout, fields):
    from oracle import oracle

    n = fields["a"].shape[0]
    d = np.zeros(n, dtype=np.uint32)
    for rows, kw, arr in casefile.case_groups(layout, fields):
        want, st = oracle.mma_dot_batch(arr["a"], arr["b"], arr["c"], scale_a=arr.get("scale_a"),
                                        scale_b=arr.get("scale_b"), sparse_metadata=arr.get("meta"), **kw)
        assert (st == 0).all()
        d[rows] = want
    return d


@pytest.mark.parametrize("op,which,path", OP_PATHS, ids=[f"op{o}-{p}" for o, _, p in OP_PATHS])
def test_records_round_trip_and_match_the_path_arithmetic(tmp_path, op, which, path):
    from oracle import oracle

    layout = casefile.OPS[op][which]
    spec = PATHS[path]
    cases = sweep.host_cases(spec, 0, 96, 96)
    fields = _fields(layout, cases)
    p = tmp_path / "cases.bin"
    casefile.write_input(p, op, layout, fields)
    op2, layout2, back = casefile.read_input(p)
    assert op2 == op and layout2 is layout
    for k in fields:
        assert np.array_equal(back[k], fields[k]), k
    # the record's op and layout reach the same model as the validation path
    assert np.array_equal(_expected(layout, back), oracle.eval_cases(cases))


def test_report_counts_mismatches_and_position_failures(tmp_path):
    layout = casefile.OPS[4][0]
    cases = sweep.host_cases(PATHS["dense-e4m3"], 0, 64, 64)
    fields = _fields(layout, cases)
    d = _expected(layout, fields)
    frag = np.broadcast_to(d[:, None, None], (64, casefile.THREADS, casefile.REGS)).copy()
    assert casefile.compare(layout, d, frag) == {"cases": 64, "mismatches": 0, "position_failures": 0}
    frag[3, 0, 0] ^= 1                       # first valid word wrong (and now disagreeing)
    frag[7, 13, 1] ^= 1                      # another valid position disagrees
    frag[9, 2, 0] ^= 1                       # thread 2 is not a valid 8-bit position: ignored
    path = tmp_path / "out.bin"
    casefile.write_output(path, 4, frag)
    op, words = casefile.read_output(path, 4)
    assert op == 4
    assert casefile.compare(layout, d, words) == {"cases": 64, "mismatches": 1, "position_failures": 2}


def test_malformed_files_are_rejected(tmp_path):
    layout = casefile.OPS[2][0]
    cases = sweep.host_cases(PATHS["dense-tf32"], 0, 4, 4)
    p = tmp_path / "c.bin"
    casefile.write_input(p, 2, layout, _fields(layout, cases))
    raw = p.read_bytes()
    (tmp_path / "magic.bin").write_bytes(b"XXXXXXX\0" + raw[8:])
    (tmp_path / "short.bin").write_bytes(raw[:-4])
    (tmp_path / "shape.bin").write_bytes(casefile.INPUT_HEADER.pack(casefile.INPUT_MAGIC, 1, 28, 0))
    with pytest.raises(ValueError, match="magic"):
        casefile.read_input(tmp_path / "magic.bin")
    with pytest.raises(ValueError, match="matches no record layout"):
        casefile.read_input(tmp_path / "short.bin")
    with pytest.raises(ValueError, match="shape probe"):
        casefile.read_input(tmp_path / "shape.bin")


@pytest.mark.gpu
@pytest.mark.parametrize("op,which,path", OP_PATHS, ids=[f"op{o}-{p}" for o, _, p in OP_PATHS])
def test_gpu_evaluates_case_files_like_the_oracle(tmp_path, op, which, path):
    layout = casefile.OPS[op][which]
    cases = sweep.host_cases(PATHS[path], 0, 2000, 2000)
    fields = _fields(layout, cases)
    src, dst = tmp_path / "in.bin", tmp_path / "out.bin"
    casefile.write_input(src, op, layout, fields)
    _, _, d = casefile.evaluate_input(src, dst)
    want = _expected(layout, fields)
    assert np.array_equal(d, want)
    _, words = casefile.read_output(dst, op)
    assert casefile.compare(layout, want, words) == {"cases": 2000, "mismatches": 0, "position_failures": 0}

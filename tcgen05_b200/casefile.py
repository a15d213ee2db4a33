"""The reference hardware harness's case files: MMAPRB1 inputs and MMAPRO1
outputs (hardware_validation/mma_probe/tcgen05.py:28-67, :187-204 for the
record layouts, :688-1276 for the writers and the output reader).

With these the emulator stands in for a tcgen05 probe runner: it reads an
input file the harness wrote, evaluates every case in one batched call, and
writes an output file in the runner's layout (the case's D word in every
register of the fragment).  It also replays a harness run: given the input
file and the hardware's output file, it reports the harness's fields --
cases, mismatches (first valid word against the emulator) and
position_failures (cases whose valid fragment words disagree).

    python -m tcgen05_b200.casefile --input cases.bin --output outputs.bin
    python -m tcgen05_b200.casefile --input cases.bin --compare hw_outputs.bin [--report r.json]
"""

from __future__ import annotations

import argparse
import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

INPUT_MAGIC = b"MMAPRB1\0"
OUTPUT_MAGIC = b"MMAPRO1\0"
VERSION = 1
INPUT_HEADER = struct.Struct("<8sIIQ")     # magic, version, op, case count
OUTPUT_HEADER = struct.Struct("<8sIIIIQ")  # magic, version, op, threads, registers per thread, case count
THREADS = 128
REGS = 4

# format codes of the block-scaled records (tcgen05.py:121-127)
MX_FORMAT_CODES = {"e4m3": 0, "e5m2": 1, "e2m3": 3, "e3m2": 4, "e2m1": 5}
MX_FORMAT_NAMES = {v: k for k, v in MX_FORMAT_CODES.items()}

# valid (thread, register) positions of a case's fragment (tcgen05.py:72-80, :1283-1308)
POS_ALL32 = tuple((t, r) for t in range(32) for r in range(REGS))
POS_16BIT = tuple([(t, r) for t in range(16) for r in range(4)] + [(t, r) for t in range(16, 32) for r in range(2)])
POS_8BIT = tuple([(t, r) for t in (0, 1, 4, 5) for r in range(4)] + [(t, r) for t in (8, 9, 12, 13) for r in range(2)])
POS_FIRST = ((0, 0),)


@dataclass(frozen=True)
class Layout:
    """One record layout: the uint32 fields in order, the words of A and B in
    the record, the logical K the model sees, the mma_dot keywords, and the
    valid fragment positions."""

    name: str
    fields: tuple            # ("a", 64), ("b", 64), ("c", 1), ("meta", 1), ...
    k: int                   # logical K passed to the model (a[:k], b[:k])
    desc: tuple              # sorted (keyword, value) pairs for mma_dot
    positions: tuple
    mx_formats: bool = False  # record carries A/B format codes (block-scaled)

    @property
    def words(self) -> int:
        return sum(n for _, n in self.fields)

    @property
    def descriptor(self) -> dict:
        return dict(self.desc)


def _L(name, fields, k, positions, mx=False, **desc):
    return Layout(name, tuple(fields), k, tuple(sorted(desc.items())), positions, mx)


def _plain(k, extra=()):
    return [("a", k), ("b", k), ("c", 1), *extra]


_META1 = (("meta", 1),)
_META2 = (("meta", 1), ("meta_hi", 1))
_SCALES = (("scale_a", 4), ("scale_b", 4))
_MX_TAIL = (("fmt_a", 1), ("fmt_b", 1), ("n", 1), ("cta_group", 1), ("m", 1))


def _mx_dense(name, k, **desc):
    return _L(name, [("a", 64), ("b", 64), ("c", 1), *_SCALES, *_MX_TAIL], k, POS_FIRST, True, **desc)


def _mx_sparse(name, k, **desc):
    return _L(name, [("a", 128), ("b", 128), ("c", 1), *_META2, *_SCALES, *_MX_TAIL], k, POS_FIRST, True, **desc)


def _layouts() -> dict:
    ops = {
        2: [_L("tf32", _plain(8), 8, POS_ALL32, a_format="tf32")],
        3: [_L("bf16", _plain(16), 16, POS_16BIT, a_format="bf16")],
        4: [_L("fp8", _plain(32), 32, POS_8BIT, a_format="e4m3")],
        5: [_L("nvfp4", [*_plain(64), *_SCALES], 64, POS_FIRST, a_format="e2m1", scaling="ue4m3", scale_vec=4)],
        6: [_L("tf32-sparse", _plain(16, _META1), 16, POS_ALL32, a_format="tf32")],
        7: [_L("bf16-sparse", _plain(32, _META1), 32, POS_16BIT, a_format="bf16")],
        8: [_L("fp8-sparse", _plain(64, _META2), 64, POS_8BIT, a_format="e4m3")],
        9: [_L("nvfp4-sparse", [*_plain(128), *_META2, *_SCALES], 128, POS_FIRST, a_format="e2m1", scaling="ue4m3",
               scale_vec=4)],
        10: [_L("f16", _plain(16), 16, POS_16BIT, a_format="f16")],
        11: [_L("f16-sparse", _plain(32, _META1), 32, POS_16BIT, a_format="f16")],
    }
    for op, fmt in ((12, "e5m2"), (13, "e2m3"), (14, "e3m2"), (15, "e2m1")):
        ops[op] = [_L(f"f8f6f4-{fmt}", _plain(32), 32, POS_8BIT, a_format=fmt)]
    for op, fmt in ((16, "e5m2"), (17, "e2m3"), (18, "e3m2"), (19, "e2m1")):
        ops[op] = [_L(f"f8f6f4-{fmt}-sparse", _plain(64, _META2), 64, POS_8BIT, a_format=fmt)]
    for op, fmt in ((20, "e4m3"), (21, "e5m2"), (22, "e2m3"), (23, "e3m2"), (24, "e2m1")):
        kw = dict(a_format=fmt, scaling="ue8m0", kind="mxf8f6f4", scale_vec=1)
        ops[op] = [_mx_dense(f"mxf8f6f4-{fmt}", 32, **kw), _mx_sparse(f"mxf8f6f4-{fmt}-sparse", 64, **kw)]
    for op, name, kw in ((25, "mxf4", dict(kind="mxf4", scale_vec=2)),
                         (26, "mxf4nvf4-2x", dict(kind="mxf4nvf4", scale_vec=2)),
                         (27, "mxf4nvf4-4x", dict(kind="mxf4nvf4", scale_vec=4))):
        full = dict(a_format="e2m1", scaling="ue8m0", **kw)
        ops[op] = [_mx_dense(name, 64, **full), _mx_sparse(name + "-sparse", 128, **full)]
    for i, (a, b, sat) in enumerate([(x, y, s) for s in (False, True) for (x, y) in
                                     (("u8", "u8"), ("s8", "u8"), ("u8", "s8"), ("s8", "s8"))]):
        ops[29 + i] = [_L(f"i8-{a}-{b}{'-sat' if sat else ''}", _plain(32), 32, POS_8BIT, a_format=a, b_format=b,
                          d_type="s32", saturate=sat)]
    ue4m3 = dict(a_format="e2m1", scaling="ue4m3", kind="mxf4nvf4", scale_vec=4)
    ops[37] = [_mx_dense("mxf4nvf4-4x-ue4m3", 64, **ue4m3)]
    ops[38] = [_mx_sparse("mxf4nvf4-4x-ue4m3-sparse", 128, **ue4m3)]
    return ops


OPS = _layouts()
SHAPE_OP = 28  # the layout probe: its records describe fragment coordinates, not a dot product


def _layout_for(op: int, payload_bytes: int, count: int) -> Layout:
    if op == SHAPE_OP:
        raise ValueError("op 28 (shape probe) records are layout probes, not dot products")
    if op not in OPS:
        raise ValueError(f"unknown case-file op {op}")
    for layout in OPS[op]:
        if payload_bytes == count * layout.words * 4:
            return layout
    sizes = ", ".join(str(count * lay.words * 4) for lay in OPS[op])
    raise ValueError(f"op {op}: payload of {payload_bytes} bytes matches no record layout ({sizes})")


def read_input(path) -> tuple[int, Layout, dict]:
    """(op, layout, fields): each field an [n, width] uint32 array."""
    raw = Path(path).read_bytes()
    if len(raw) < INPUT_HEADER.size:
        raise ValueError("short input header")
    magic, version, op, count = INPUT_HEADER.unpack_from(raw)
    if magic != INPUT_MAGIC:
        raise ValueError("bad input magic")
    if version != VERSION:
        raise ValueError(f"unsupported input version {version}")
    layout = _layout_for(op, len(raw) - INPUT_HEADER.size, count)
    words = np.frombuffer(raw, dtype="<u4", offset=INPUT_HEADER.size).reshape(count, layout.words)
    fields, col = {}, 0
    for name, width in layout.fields:
        fields[name] = words[:, col:col + width].astype(np.uint32)
        col += width
    return op, layout, fields


def write_input(path, op: int, layout: Layout, fields: dict) -> None:
    n = fields["a"].shape[0]
    cols = []
    for name, width in layout.fields:
        v = np.asarray(fields[name], dtype=np.uint32).reshape(n, width)
        cols.append(v)
    body = np.concatenate(cols, axis=1).astype("<u4")
    Path(path).write_bytes(INPUT_HEADER.pack(INPUT_MAGIC, VERSION, op, n) + body.tobytes())


def read_output(path, expected_op: int | None = None) -> tuple[int, np.ndarray]:
    """(op, words [n, threads, 4])."""
    raw = Path(path).read_bytes()
    if len(raw) < OUTPUT_HEADER.size:
        raise ValueError("short output header")
    magic, version, op, threads, regs, count = OUTPUT_HEADER.unpack_from(raw)
    if magic != OUTPUT_MAGIC:
        raise ValueError("bad output magic")
    if version != VERSION or (expected_op is not None and op != expected_op):
        raise ValueError("unsupported output file")
    if regs != REGS or threads < 1:
        raise ValueError("unexpected output shape")
    payload = len(raw) - OUTPUT_HEADER.size
    if payload != count * threads * regs * 4:
        raise ValueError(f"short output payload: got {payload}, expected {count * threads * regs * 4}")
    words = np.frombuffer(raw, dtype="<u4", offset=OUTPUT_HEADER.size).reshape(count, threads, regs)
    return op, words.astype(np.uint32)


def write_output(path, op: int, words: np.ndarray) -> None:
    count, threads, regs = words.shape
    Path(path).write_bytes(OUTPUT_HEADER.pack(OUTPUT_MAGIC, VERSION, op, threads, regs, count)
                           + np.asarray(words, dtype="<u4").tobytes())


def case_groups(layout: Layout, fields: dict):
    """Yield (row indices, mma_dot keywords, arrays) per distinct A/B format
    pair: the public-API view of the records (a[:k], b[:k], c, scales, the
    metadata pair)."""
    n = fields["a"].shape[0]
    desc = layout.descriptor
    if layout.mx_formats:
        keys = fields["fmt_a"][:, 0].astype(np.int64) * 16 + fields["fmt_b"][:, 0].astype(np.int64)
        groups = [(np.flatnonzero(keys == key), int(key)) for key in np.unique(keys)]
    else:
        groups = [(np.arange(n), None)]
    for rows, key in groups:
        kw = dict(desc)
        if key is not None:
            fa, fb = key // 16, key % 16
            if fa not in MX_FORMAT_NAMES or fb not in MX_FORMAT_NAMES:
                raise ValueError(f"unknown block-scaled format codes {fa}/{fb}")
            if desc.get("kind") == "mxf8f6f4":
                kw["a_format"], kw["b_format"] = MX_FORMAT_NAMES[fa], MX_FORMAT_NAMES[fb]
        arrays = {"a": fields["a"][rows, :layout.k], "b": fields["b"][rows, :layout.k], "c": fields["c"][rows, 0]}
        if "scale_a" in fields:
            arrays["scale_a"] = fields["scale_a"][rows].astype(np.uint8)
            arrays["scale_b"] = fields["scale_b"][rows].astype(np.uint8)
        if "meta" in fields:
            hi = fields["meta_hi"][rows, 0] if "meta_hi" in fields else fields["meta"][rows, 0]
            arrays["meta"] = np.stack([fields["meta"][rows, 0], hi], axis=1).astype(np.uint32)
        yield rows, kw, arrays


def _fragment_threads(layout: Layout, fields: dict) -> int:
    if "cta_group" in fields and fields["cta_group"].size and int(fields["cta_group"].max()) == 2:
        return 2 * THREADS
    return THREADS


def evaluate_input(path_in, path_out=None, *, device=None) -> tuple[int, Layout, np.ndarray]:
    """Evaluate every record of an input file on the GPU; optionally write the
    runner-layout output file.  Returns (op, layout, D words [n])."""
    from . import simulator

    op, layout, fields = read_input(path_in)
    n = fields["a"].shape[0]
    d = np.zeros(n, dtype=np.uint32)
    for rows, kw, arr in case_groups(layout, fields):
        d[rows] = simulator.mma_dot_batch(arr["a"], arr["b"], arr["c"], scale_a=arr.get("scale_a"),
                                          scale_b=arr.get("scale_b"), sparse_metadata=arr.get("meta"),
                                          device=device, **kw)
    if path_out is not None:
        threads = _fragment_threads(layout, fields)
        write_output(path_out, op, np.broadcast_to(d[:, None, None], (n, threads, REGS)).copy())
    return op, layout, d


def compare(layout: Layout, expected: np.ndarray, outputs: np.ndarray) -> dict:
    """The harness's report fields for observed fragments against expected D
    words: position_failures counts cases whose valid positions disagree,
    mismatches cases whose first valid word differs from the expectation."""
    t = np.array([p[0] for p in layout.positions])
    r = np.array([p[1] for p in layout.positions])
    valid = outputs[:, t, r]
    position_failures = int((valid != valid[:, :1]).any(axis=1).sum())
    mismatches = int((valid[:, 0] != expected).sum())
    return {"cases": int(expected.shape[0]), "mismatches": mismatches, "position_failures": position_failures}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--input", required=True, help="MMAPRB1 case file")
    ap.add_argument("--output", help="write the emulator's MMAPRO1 output file here")
    ap.add_argument("--compare", help="a hardware MMAPRO1 output file to check against the emulator")
    ap.add_argument("--report", help="write the JSON report here")
    args = ap.parse_args(argv)
    op, layout, d = evaluate_input(args.input, args.output)
    report = {"op": op, "layout": layout.name, "cases": int(d.shape[0])}
    if args.compare:
        _, words = read_output(args.compare, op)
        if words.shape[0] != d.shape[0]:
            raise SystemExit(f"output case count mismatch: got {words.shape[0]}, expected {d.shape[0]}")
        report.update(compare(layout, d, words))
    text = json.dumps(report, indent=2, sort_keys=True)
    if args.report:
        Path(args.report).write_text(text + "\n")
    print(text)
    return 1 if report.get("mismatches") or report.get("position_failures") else 0


if __name__ == "__main__":
    raise SystemExit(main())

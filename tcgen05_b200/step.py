"""One step of the benchmark workload, resident in HBM: the 46-path
validation sweep at 1M cases per path plus the matrix configuration (4,096
BF16 tiles of 128 x 256 x 16), sharded over the ranks of a job.

``build_step`` generates a rank's shard of every path (tcgen05_b200.sweep)
and of the tiles in the kernels' layout; ``launcher`` returns the call that
evaluates one of them through t5e_mma_dot_batch.  ``stream_groups`` and
``capture_step`` record the step as one CUDA graph whose launches run on
several streams: the paths are independent, so one launch's tail and the
next one's start overlap with other paths' launches.  bench.py times these
launches; ``python -m tcgen05_b200.step`` runs warm-up steps and one step, the
command the launch-list profiles are taken with.
"""

from __future__ import annotations

import argparse
import ctypes

CASES_PER_PATH = 1_000_000
MATRIX_TILES = 4096
TILE_M, TILE_N, TILE_K = 128, 256, 16


def kernel_of(spec) -> str:
    """The specialised kernel t5e_mma_dot_batch dispatches a path to."""
    d = spec.descriptor
    fam, fmt = spec.family, d["a_format"]
    if fam == "i8":
        return "i8_kernel"
    if d["scaling"] == "ue4m3":
        return "nvfp4_kernel"
    if fam in ("fp4block", "sparse-fp4block"):
        return "mxf4_kernel"
    if fmt in ("tf32", "bf16", "f16") or (fam == "sparse" and spec.params[0] in ("tf32", "bf16", "f16")):
        return "wide_kernel"
    if fam in ("mx", "sparse-mx") and fmt in ("e2m3", "e3m2", "e2m1"):
        return "mx_kernel"
    return "raw_window_kernel"


class Launch:
    """One launch of the step: a path's shard or the matrix tiles' shard,
    resident in HBM with its output buffer and the batch struct that
    t5e_mma_dot_batch takes."""

    def __init__(self, name, kernel, desc, db, d, macs, nbytes, first_case):
        from . import runtime

        self.name, self.kernel, self.desc = name, kernel, desc
        self.db, self.d = db, d
        self.struct = runtime.make_batch_struct(db, d, None)
        self.macs, self.bytes = macs, nbytes
        self.first_case = first_case  # global index of this shard's first case


# Microseconds per launch of each path at 1,000,000 cases on one B200 (the
# bench step's per-launch events, SM clock 1965 MHz): the weights by which
# whole paths are spread over the ranks of a job.
PATH_COST_US = {"dense-tf32": 27.1, "dense-bf16": 33.6, "dense-f16": 33.2, "dense-e4m3": 33.4,
                "dense-e5m2": 31.7, "dense-e2m3": 36.2, "dense-e3m2": 36.2, "dense-e2m1": 34.8,
                "i8-u8-u8-wrap": 18.5, "i8-s8-u8-wrap": 18.2, "i8-u8-s8-wrap": 18.7, "i8-s8-s8-wrap": 18.4,
                "i8-u8-u8-saturate": 18.4, "i8-s8-u8-saturate": 18.5, "i8-u8-s8-saturate": 18.8,
                "i8-s8-s8-saturate": 18.4, "dense-mx-e4m3": 35.9, "dense-mx-e5m2": 35.0, "dense-mx-e2m3": 36.2,
                "dense-mx-e3m2": 36.8, "dense-mx-e2m1": 36.5, "dense-mxf4": 28.7, "dense-mxf4nvf4-2x": 28.3,
                "dense-mxf4nvf4-4x": 28.7, "dense-mxf4nvf4-4x-ue4m3": 24.2, "sparse-tf32": 29.3,
                "sparse-bf16": 38.9, "sparse-f16": 39.6, "sparse-fp8": 45.4, "sparse-e5m2": 41.5,
                "sparse-e2m3": 47.2, "sparse-e3m2": 46.5, "sparse-e2m1": 43.7, "sparse-nvfp4": 31.7,
                "sparse-mx-e4m3": 47.1, "sparse-mx-e5m2": 44.4, "sparse-mx-e2m3": 46.0, "sparse-mx-e3m2": 46.1,
                "sparse-mx-e2m1": 41.3, "sparse-mxf4": 33.1, "sparse-mxf4nvf4-2x": 32.8, "sparse-mxf4nvf4-4x": 34.8,
                "sparse-mxf4nvf4-4x-ue4m3": 32.8, "mixed-e4m3-e2m1-f32": 33.1, "mixed-e2m1-e4m3-f16": 33.5,
                "dense-nvfp4": 24.6}
DEFAULT_PATH_COST_US = 40.0


def path_owners(world: int) -> dict[str, int]:
    """The rank that evaluates each whole path of the sweep: longest paths
    first, each to the least loaded rank (ties to the lower rank), so every
    rank computes the same assignment without communicating."""
    from . import workloads

    names = [s.name for s in workloads.validation_paths()]
    cost = {n: PATH_COST_US.get(n, DEFAULT_PATH_COST_US) for n in names}
    load = [0.0] * world
    owners = {}
    for n in sorted(names, key=lambda n: (-cost[n], names.index(n))):
        r = min(range(world), key=lambda x: (load[x], x))
        owners[n] = r
        load[r] += cost[n]
    return owners


def path_host_bytes(spec) -> int:
    """Host bytes per case of a path through the public API on raw words, as
    the bench's end-to-end step moves them: A and B container words (A at
    logical K for sparse paths), C, the scale bytes and metadata words the
    generator produces, and the 32-bit result word."""
    import numpy as np

    from . import sweep

    g = sweep.generate(spec, 0, 1, 2, np)
    per = 4 * (g["a"].shape[1] + g["b"].shape[1]) + (2 if spec.descriptor["d_type"] == "f16" else 4) + 4
    if g["scale_a"] is not None:
        per += g["scale_a"].shape[1] + g["scale_b"].shape[1]
    if g["meta"] is not None:
        per += 4 * g["meta"].shape[1]
    return per


def host_path_owners(world: int, rates=None, base_bytes: float = 0.0) -> dict[str, int]:
    """``path_owners`` weighted by host bytes instead of GPU time: for a step
    through the public API from host memory, which the host link bounds.

    ``rates`` (one positive figure per rank, bytes per second or any common
    unit) weights the deal by each rank's host link: a path goes to the rank
    that would finish it first, counting ``base_bytes`` the rank moves in any
    case (its share of the tiles).  Without rates every link counts the same
    and the deal is by bytes alone.  Every rank computes the same deal from
    the same rates.  A path's bytes are its per-case host bytes times
    ``CASES_PER_PATH``, the unit of ``base_bytes``."""
    from . import workloads

    if rates is None:
        rates = [1.0] * world
    rates = [float(x) for x in rates]
    if len(rates) != world or min(rates) <= 0:
        raise ValueError("rates must hold one positive figure per rank")
    specs = workloads.validation_paths()
    names = [s.name for s in specs]
    cost = {s.name: path_host_bytes(s) * CASES_PER_PATH for s in specs}
    load = [float(base_bytes)] * world
    owners = {}
    for n in sorted(names, key=lambda n: (-cost[n], names.index(n))):
        r = min(range(world), key=lambda x: ((load[x] + cost[n]) / rates[x], x))
        owners[n] = r
        load[r] += cost[n]
    return owners


def build_step(torch, dev, rank: int, world: int, *, cases_per_path: int = CASES_PER_PATH,
               tiles: int = MATRIX_TILES, shard: str = "paths") -> list[Launch]:
    """This rank's part of the step, generated in HBM in the kernels' layout
    (smaller steps for profiling keep the same distributions): the matrix
    tiles split evenly, and the sweep either as whole paths per rank
    (``shard="paths"``, ``path_owners``: every launch keeps its full size, as
    the reference's validation runner gives whole paths to devices) or as a
    contiguous share of every path's cases (``shard="cases"``)."""
    from . import sweep, workloads

    if shard not in ("paths", "cases"):
        raise ValueError(f"unknown shard mode {shard!r}")
    items = []
    owners = path_owners(world) if shard == "paths" else None
    lo, hi = (0, cases_per_path) if shard == "paths" else sweep.shard(cases_per_path, rank, world)
    for spec in workloads.validation_paths():
        if owners is not None and owners[spec.name] != rank:
            continue
        model, db = sweep.device_batch(spec, lo, hi - lo, cases_per_path, dev)
        macs, nbytes = sweep.path_work(spec, db.n, model)
        d = torch.empty(db.n, dtype=torch.int32, device=dev)
        items.append(Launch(spec.name, kernel_of(spec), model.descriptor(), db, d, macs, nbytes, lo))
    t0, t1 = sweep.shard(tiles, rank, world)
    per_tile = TILE_M * TILE_N
    model, db = sweep.matrix_tiles(t0, t1 - t0, dev, TILE_M, TILE_N, TILE_K)
    macs, nbytes = workloads.config_work("matrix-bf16", db)
    d = torch.empty(db.n, dtype=torch.int32, device=dev)
    items.append(Launch("matrix-bf16", "wide_tile_kernel", model.descriptor(), db, d, macs, nbytes, t0 * per_tile))
    torch.cuda.synchronize(dev)
    return items


def launcher(lib, stream):
    from . import _native as nat

    handle = ctypes.c_void_p(stream.cuda_stream)

    def launch(item):
        rc = lib.t5e_mma_dot_batch(ctypes.byref(item.desc), ctypes.byref(item.struct), handle)
        if rc != 0:
            nat.check(rc, "t5e_mma_dot_batch " + item.name)

    return launch


STEP_STREAMS = 4  # streams the step's graph spreads its launches over


def stream_groups(times, streams: int = STEP_STREAMS) -> list[list[int]]:
    """Indices of the step's launches split into `streams` groups of about
    equal summed time: longest first, each to the least loaded group; each
    group in launch order."""
    load = [0.0] * streams
    groups: list[list[int]] = [[] for _ in range(streams)]
    for j in sorted(range(len(times)), key=lambda j: (-times[j], j)):
        g = min(range(streams), key=lambda x: (load[x], x))
        groups[g].append(j)
        load[g] += times[j]
    return [sorted(g) for g in groups if g]


def capture_step(torch, lib, dev, items, groups):
    """The step as one CUDA graph: each group's launches in order on a stream
    of its own, forked from and joined back to the capturing stream."""
    streams = [torch.cuda.Stream(dev) for _ in groups]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        cap = torch.cuda.current_stream(dev)
        fork = torch.cuda.Event()
        fork.record(cap)
        joins = []
        for s, grp in zip(streams, groups):
            s.wait_event(fork)
            launch = launcher(lib, s)
            for j in grp:
                launch(items[j])
            done = torch.cuda.Event()
            done.record(s)
            joins.append(done)
        for done in joins:
            cap.wait_event(done)
    return graph


def whole_step_macs() -> int:
    """Element-MACs of one step of the whole job: physical products of the
    46 paths at CASES_PER_PATH cases each, plus the matrix tiles."""
    from . import sweep, workloads

    macs = sum(sweep.path_work(s, CASES_PER_PATH)[0] for s in workloads.validation_paths())
    return macs + MATRIX_TILES * TILE_M * TILE_N * TILE_K




def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--cases-per-path", type=int, default=CASES_PER_PATH)
    ap.add_argument("--tiles", type=int, default=MATRIX_TILES)
    args = ap.parse_args(argv)
    import torch

    from . import _native as nat

    dev = torch.device("cuda", 0)
    items = build_step(torch, dev, 0, 1, cases_per_path=args.cases_per_path, tiles=args.tiles)
    launch = launcher(nat.load(), torch.cuda.current_stream(dev))
    for _ in range(args.warmup + 1):
        for item in items:
            launch(item)
    torch.cuda.synchronize(dev)
    print(f"{len(items)} launches per step, {args.warmup} warm-up steps and one step", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

"""Benchmark: emulated element-MACs/s of the tcgen05 MMA emulator on B200.

Workload (one step) -- the full validation sweep: all 46 modeled paths
(every dense and sparse float, integer and block-scaled combination of the
reference harness, hardware_validation/run_full_validation.py:43-224) at
1,000,000 seeded cases each, plus the matrix configuration, 4,096
independent BF16 tiles of M=128 N=256 K=16 with F32 C/D.  That is 46M dot
products (1.68e9 element-MACs: physical products, K/2 for the sparse paths)
and 134M tile cases (2.15e9 element-MACs) per step.  The work is fixed and
sharded over the GPUs (strong scaling): rank r of N evaluates cases
[1M*r/N, 1M*(r+1)/N) of every path and its share of the tiles, on inputs
generated in its own HBM by the counter hash of tcgen05_b200.sweep (the same
words the numpy mirror produces on the host).  A step's inputs (about 4.9 GB
at N=1, 0.6 GB at N=8) exceed the 126 MB L2, and every batch is read once
per step, so no launch finds its inputs in L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank launches its shard; the timed region is
bracketed by a barrier and a device synchronisation on every rank, timed with
CUDA events, and the maximum over ranks is reported.  The only collectives
(NCCL) come after it: the maximum of the timings and the sum of the mismatch
counts.  The line also carries, per path, its kernel time and rate; the NVFP4
configuration (2^24 dense and 2^24 pairwise-sparse cases, sharded) at the
same N; end to end through the public API on raw container words in pinned
host memory; and, at N=1, the reference Python model timed on the host cores.

``--impl reference`` times the reference's own CPU implementation of the
path, the Python tcgen05_model installed in baseline/_ref, through its public
mma_dot/mma over all host cores (multiprocessing) on a bounded sample of the
same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "emulated element-MACs/s (bit-exact) at 1/2/4/8 B200 vs Python model on host"
UNIT = "element-MACs/s"
NVFP4_CASES = 1 << 24
E2E_RUNS = 3
E2E_CALIBRATIONS = 2  # untimed runs over N GPUs that measure each rank's host-link rate
REF_DIR = REPO / "baseline" / "_ref"

from tcgen05_b200.step import (CASES_PER_PATH, MATRIX_TILES, STEP_STREAMS, TILE_K, TILE_M, TILE_N,  # noqa: E402
                               build_step, capture_step, launcher, stream_groups, whole_step_macs)


def measured_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# Kernel source files behind each profiled figure: a figure in profiles/ is
# stamped with the hash of these files when it is captured, and the bench
# uses it only while the stamp still matches.
KERNEL_SOURCES = {
    "wide_tile_kernel": ["tcgen05_b200/csrc/t5e_wide.cu", "tcgen05_b200/csrc/t5e_arith.cuh"],
    "raw_window_kernel": ["tcgen05_b200/csrc/t5e_fast.cu", "tcgen05_b200/csrc/t5e_arith.cuh",
                          "tcgen05_b200/csrc/t5e_select.cuh"],
    "mx_kernel": ["tcgen05_b200/csrc/t5e_fast.cu", "tcgen05_b200/csrc/t5e_arith.cuh",
                  "tcgen05_b200/csrc/t5e_select.cuh"],
    "nvfp4_kernel": ["tcgen05_b200/csrc/t5e_nvfp4.cu", "tcgen05_b200/csrc/t5e_e2m1.cuh",
                     "tcgen05_b200/csrc/t5e_select.cuh", "tcgen05_b200/csrc/t5e_arith.cuh"],
    "mxf4_kernel": ["tcgen05_b200/csrc/t5e_mxf4.cu", "tcgen05_b200/csrc/t5e_e2m1.cuh",
                    "tcgen05_b200/csrc/t5e_select.cuh", "tcgen05_b200/csrc/t5e_arith.cuh"],
    "i8_kernel": ["tcgen05_b200/csrc/t5e_i8.cu"],
    "wide_kernel": ["tcgen05_b200/csrc/t5e_wide.cu", "tcgen05_b200/csrc/t5e_arith.cuh"],
}


def source_stamp(kernel: str) -> str:
    """First 16 hex digits of the SHA-256 of a kernel's source files."""
    h = hashlib.sha256()
    for f in KERNEL_SOURCES[kernel]:
        h.update((REPO / f).read_bytes())
    return h.hexdigest()[:16]


def profiled_figure(name: str, tag: str, kernel: str) -> tuple[float | None, str]:
    """A figure of a kernel from the committed ncu summaries: a line
    '<name>[<tag>]: <number> src=<stamp>'.  Returns (value, state), state
    'current' when the stamp matches the kernel's source today, 'stale' when
    the source changed since the capture (value None then), or 'absent'."""
    key = f"{name}[{tag}]:"
    for f in sorted((REPO / "profiles").glob("*.md")) + sorted((REPO / "profiles").glob("*.txt")):
        for line in f.read_text().splitlines():
            line = line.strip().strip("`").strip()
            if not line.startswith(key):
                continue
            fields = line[len(key):].split()
            stamp = next((x[4:] for x in fields if x.startswith("src=")), None)
            if stamp != source_stamp(kernel):
                return None, "stale"
            try:
                return float(fields[0]), "current"
            except (ValueError, IndexError):
                return None, "absent"
    return None, "absent"


def issue_peaks(torch, lib, stream, iters: int = 256, launches: int = 5) -> dict:
    """Measured issue rates (warp instructions/s) of the ALU and FMA pipes at
    the SM clock of the moment: the library's probe kernels issue a known
    number of independent LOP3/SHF (ALU) or IMAD (FMA) instructions at full
    occupancy; the best of `launches` event-timed launches per pipe."""
    from tcgen05_b200 import _native as nat

    handle = ctypes.c_void_p(stream.cuda_stream)
    out = {}
    for pipe, name in ((0, "alu"), (1, "fma"), (2, "fp64")):
        count = ctypes.c_uint64(0)
        for _ in range(2):
            nat.check(lib.t5e_issue_probe(pipe, iters, ctypes.byref(count), handle), "t5e_issue_probe")
        best = None
        for _ in range(launches):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            nat.check(lib.t5e_issue_probe(pipe, iters, ctypes.byref(count), handle), "t5e_issue_probe")
            b.record(stream)
            b.synchronize()
            ms = a.elapsed_time(b)
            best = ms if best is None else min(best, ms)
        out[name] = count.value / (best / 1e3)
    return out


# ------------------------------------------------------------------ clocks


def smi_gpu_id(local: int) -> str:
    """nvidia-smi's id (index or UUID) of this process's CUDA device `local`,
    following CUDA_VISIBLE_DEVICES when it remaps devices."""
    vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    if local < len(vis):
        return vis[local]
    return str(local)


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"t5e_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = [r.split(", ") for r in self.path.read_text().splitlines() if r.strip()]
        self.path.unlink(missing_ok=True)
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for name, flag in zip(names, r[5:9]):
                    if flag.strip().lower() == "active":
                        reasons.add(name)
            except (IndexError, ValueError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- the step


def per_launch_times(torch, stream, items, launch, steps: int = 3) -> list[float]:
    """Mean duration (ms) of each launch of the step, from an event recorded
    between consecutive launches over `steps` further steps (the events keep
    a launch from overlapping the next one's start, so these add up to a
    little more than the timed step)."""
    acc = [0.0] * len(items)
    for _ in range(steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(items) + 1)]
        ev[0].record(stream)
        for j, item in enumerate(items):
            launch(item)
            ev[j + 1].record(stream)
        ev[-1].synchronize()
        for j in range(len(items)):
            acc[j] += ev[j].elapsed_time(ev[j + 1])
    return [a / steps for a in acc]


def verify(torch, lib, stream, items) -> tuple[int, dict]:
    """Words of the timed launches against the generic kernel's on the same
    inputs (mismatch count), and per path an order-independent checksum of
    (global case index, word) pairs, which is the same at every GPU count."""
    from tcgen05_b200 import _native as nat
    from tcgen05_b200 import runtime, sweep

    handle = ctypes.c_void_p(stream.cuda_stream)
    mism = 0
    sums = {}
    for item in items:
        g = torch.empty_like(item.d)
        bs = runtime.make_batch_struct(item.db, g, None)
        nat.check(lib.t5e_mma_dot_batch_generic(ctypes.byref(item.desc), ctypes.byref(bs), handle), "generic")
        mism += int((g != item.d).sum().item())
        idx = torch.arange(item.first_case, item.first_case + item.d.numel(), dtype=torch.int64, device=item.d.device)
        sums[item.name] = sweep.result_checksum(torch, idx, item.d.to(torch.int64) & 0xFFFFFFFF)
        del g
    return mism, sums


# ------------------------------------------------------- NVFP4 configuration


def nvfp4_config(torch, dev, lib, stream, rank: int, world: int, reps: int = 8) -> dict:
    """The NVFP4 configuration, 2^24 dense (K=64) and 2^24 pairwise-sparse
    (logical K=128) cases in all, sharded like the step: the mean time of a
    launch of each form, the two forms alternating (together above the L2),
    an event pair around each launch; and the words that differ from the
    generic kernel on the first 2^18 cases of the shard."""
    from tcgen05_b200 import _native as nat
    from tcgen05_b200 import runtime, sweep, workloads

    lo, hi = sweep.shard(NVFP4_CASES, rank, world)
    n = hi - lo
    handle = ctypes.c_void_p(stream.cuda_stream)
    forms = []
    for name in ("nvfp4-k64", "nvfp4-sparse-k128"):
        model, db = workloads.device_config(name, dev, seed=900 + rank, n=n)
        d = torch.empty(n, dtype=torch.int32, device=dev)
        forms.append((name, model.descriptor(), runtime.make_batch_struct(db, d, None), db, d))

    def run(desc, bs):
        nat.check(lib.t5e_mma_dot_batch(ctypes.byref(desc), ctypes.byref(bs), handle), "t5e_mma_dot_batch")

    for _ in range(2):
        for _, desc, bs, _, _ in forms:
            run(desc, bs)
    ev = {name: [] for name, *_ in forms}
    for _ in range(reps):
        for name, desc, bs, _, _ in forms:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run(desc, bs)
            e1.record(stream)
            ev[name].append((e0, e1))
    torch.cuda.synchronize(dev)
    ms = {name: statistics.mean(a.elapsed_time(b) for a, b in pairs) for name, pairs in ev.items()}
    mism = 0
    for name, desc, bs, db, d in forms:
        m = min(n, 1 << 18)
        g = torch.empty(m, dtype=torch.int32, device=dev)
        sub = runtime.make_batch_struct(db, g, None)
        sub.n = m
        nat.check(lib.t5e_mma_dot_batch_generic(ctypes.byref(desc), ctypes.byref(sub), handle), "generic")
        torch.cuda.synchronize(dev)
        mism += int((g != d[:m]).sum().item())
    return {"ms": ms, "mismatches": mism, "cases_per_rank": n}


# ------------------------------------------------------------ end to end


def host_step(torch, dev, items) -> list[tuple]:
    """The step's inputs as a user of the public API holds them: raw container
    words (uint32 words: F32 containers for TF32/BF16, the low bits for the
    narrower formats) in pinned host memory, with pinned scales, metadata and
    output words.  Path cases are the sweep's own generated words (sparse A
    at logical K, zero off the selection); the matrix tiles are the words
    whose packed rows the timed step reads."""
    from tcgen05_b200 import sweep, workloads

    specs = {s.name: s for s in workloads.validation_paths()}
    to32 = lambda x: torch.where(x >= 1 << 31, x - (1 << 32), x).to(torch.int32)  # noqa: E731
    pin = lambda x: x.cpu().pin_memory()  # noqa: E731
    out = []
    for item in items:
        n = item.d.numel()
        res = torch.empty(item.d.shape, dtype=torch.int32, pin_memory=True)
        if item.name == "matrix-bf16":
            tiles = n // (TILE_M * TILE_N)
            a = (item.db.a.view(torch.int16).to(torch.int32) << 16).view(tiles, TILE_M, TILE_K)
            b = (item.db.b.view(torch.int16).to(torch.int32) << 16).view(tiles, TILE_N, TILE_K).transpose(1, 2)
            c = item.db.c.view(tiles, TILE_M, TILE_N)
            out.append((item, "tiles", (pin(a.contiguous()), pin(b.contiguous()), pin(c)),
                        {"a_format": "bf16"}, res.view(tiles, TILE_M, TILE_N)))
            continue
        spec = specs[item.name]
        g = sweep.generate(spec, item.first_case, n, CASES_PER_PATH, torch, dev)
        d = spec.descriptor
        kw = {k: d[k] for k in ("a_format", "b_format", "d_type", "saturate", "scaling", "scale_vec", "kind")}
        if d["d_type"] == "f16":
            c = g["c"] & 0xFFFF
            c = torch.where(c >= 1 << 15, c - (1 << 16), c).to(torch.int16)
        else:
            c = to32(g["c"])
        if g["scale_a"] is not None:
            kw["scale_a"] = pin(g["scale_a"].to(torch.uint8))
            kw["scale_b"] = pin(g["scale_b"].to(torch.uint8))
        if g["meta"] is not None:
            kw["sparse_metadata"] = pin(to32(g["meta"]))
        out.append((item, "cases", (pin(to32(g["a"])), pin(to32(g["b"])), pin(c)), kw, res))
        del g
    torch.cuda.synchronize(dev)
    return out


def e2e_items(torch, items, rank: int, world: int, shard: str, rates=None, base_bytes: float = 0.0) -> list:
    """The launches a rank evaluates end to end: its share of the tiles and,
    over N GPUs with whole-path sharding, the paths ``host_path_owners`` gives
    it (by host bytes, not GPU time, over each rank's host-link rate when
    ``rates`` holds them); otherwise its own launches' paths.  Paths it did
    not time are stood in for by their name, first case and result shape."""
    from types import SimpleNamespace

    from tcgen05_b200 import workloads
    from tcgen05_b200.step import host_path_owners

    if world == 1 or shard != "paths":
        return items
    owners = host_path_owners(world, rates=rates, base_bytes=base_bytes)
    out = [SimpleNamespace(name=s.name, first_case=0,
                           d=torch.empty(CASES_PER_PATH, dtype=torch.int32, device="meta"))
           for s in workloads.validation_paths() if owners[s.name] == rank]
    return out + [item for item in items if item.name == "matrix-bf16"]


def result_words_checksum(torch, first_case: int, res) -> int:
    """The order-independent checksum of (global case index, word) pairs of
    result words in host memory (the one ``verify`` forms on the device)."""
    from tcgen05_b200 import sweep

    words = res.view(-1).to(torch.int64) & 0xFFFFFFFF
    idx = torch.arange(first_case, first_case + words.numel(), dtype=torch.int64)
    return sweep.result_checksum(torch, idx, words)


def copy_bytes(host) -> tuple[int, int]:
    """(host-to-device, device-to-host) bytes of one end-to-end step."""
    h2d = d2h = 0
    for _item, _kind, arrays, kw, res in host:
        h2d += sum(x.numel() * x.element_size() for x in arrays)
        h2d += sum(v.numel() * v.element_size() for k, v in kw.items() if hasattr(v, "numel"))
        d2h += res.numel() * res.element_size()
    return h2d, d2h


def e2e_step(t5, host, depth: int = 4) -> None:
    """One step through the public API: every call returns once its copies
    and kernels are queued (wait=False); at most `depth` are in flight; every
    result word is in host memory when the last wait returns."""
    pending = []
    for _item, kind, (a, b, c), kw, res in host:
        if kind == "tiles":
            pending.append(t5.mma_batch(a, b, c, out=res, wait=False, **kw))
        else:
            pending.append(t5.mma_dot_batch(a, b, c, out=res, wait=False, check=False, **kw))
        if len(pending) > depth:
            pending.pop(0).wait()
    for p in pending:
        p.wait()


def host_copy_ceiling(torch, dev, stream, host) -> float:
    """Seconds that plain host-to-device copies of the step's input bytes take
    on one stream (every pinned input array once, in step order): the
    host-link ceiling of the end-to-end step on this rank."""
    arrays = []
    for _item, _kind, xs, kw, _res in host:
        arrays += list(xs) + [v for v in kw.values() if hasattr(v, "numel")]
    biggest = max(x.numel() * x.element_size() for x in arrays)
    scratch = torch.empty(biggest, dtype=torch.uint8, device=dev)

    def run():
        for x in arrays:
            nb = x.numel() * x.element_size()
            scratch[:nb].copy_(x.reshape(-1).view(torch.uint8), non_blocking=True)

    run()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / 1e3


# --------------------------------------------------------- CPU baselines
#
# The sample has the step's proportions: `c` cases of every path and
# 2.92 * 46 * c tile cases (134M tile cases against 46M path cases), the
# tile cases as row blocks of the matrix tiles (16 rows of 256 columns per
# task).  Path cases are the numpy mirror of the step's generated words.

ROW_BLOCK = 16
TILE_SHARE = (MATRIX_TILES * TILE_M * TILE_N) / (46 * CASES_PER_PATH)


def sample_tasks(c: int, tiles_host, start: int = 0) -> list[tuple]:
    """Tasks of the reference Python model: ("cases", ...) per chunk of
    path cases and ("rows", ...) per row block of a tile."""
    from tcgen05_b200 import sweep, workloads

    tasks = []
    for spec in workloads.validation_paths():
        h = sweep.host_cases(spec, start, c, CASES_PER_PATH)
        d = spec.descriptor
        for s0 in range(0, c, 512):
            sub = h.subset(slice(s0, min(c, s0 + 512)))
            tasks.append(("cases", spec.name, d, start + s0, sub))
    a, b, cm = tiles_host
    rows = max(1, round(TILE_SHARE * 46 * c / TILE_N / ROW_BLOCK)) * ROW_BLOCK
    for r0 in range(0, rows, ROW_BLOCK):
        t, r = divmod(r0, TILE_M)
        t %= a.shape[0]
        tasks.append(("rows", "matrix-bf16", t, r, (a[t, r:r + ROW_BLOCK], b[t], cm[t, r:r + ROW_BLOCK])))
    return tasks


def task_macs(task) -> int:
    from tcgen05_b200 import sweep, workloads

    if task[0] == "rows":
        return ROW_BLOCK * TILE_N * TILE_K
    spec = {s.name: s for s in workloads.validation_paths()}[task[1]]
    return task[4].n * sweep._phys_k(spec)


def _ref_worker(task):
    """One task through the reference's public API (tcgen05_model from
    baseline/_ref): mma_dot per case with the model built once per path, as
    its own mma builds it once per matrix; mma on a block of tile rows.
    Returns (words, seconds spent in the reference's calls)."""
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import tcgen05_model as ref

    if task[0] == "rows":
        a, b, c = task[4]
        A, Bm, C = a.tolist(), b.tolist(), c.tolist()
        t0 = time.perf_counter()
        out = ref.mma(A, Bm, C, a_format="bf16")
        return np.array(out, dtype=np.uint32).reshape(-1), time.perf_counter() - t0
    _, _name, d, _start, cs = task
    model = ref.make_model(d["a_format"], d["b_format"], d_type=d["d_type"], saturate=d["saturate"],
                           scaling=d["scaling"], scale_vec=d["scale_vec"], kind=d["kind"])
    rows = []
    for i in range(cs.n):
        kw = {}
        if cs.scale_a is not None:
            kw["scale_a"] = tuple(cs.scale_a[i].tolist())
            kw["scale_b"] = tuple(cs.scale_b[i].tolist())
        if cs.meta is not None:
            kw["sparse_metadata"] = tuple(cs.meta[i].tolist())
        rows.append((tuple(cs.a[i].tolist()), tuple(cs.b[i].tolist()), int(cs.c[i]), kw))
    t0 = time.perf_counter()
    out = [ref.mma_dot(a, b, c, model=model, a_format=d["a_format"], scaling=d["scaling"], kind=d["kind"], **kw)
           for a, b, c, kw in rows]
    return np.array(out, dtype=np.uint32), time.perf_counter() - t0


def _warm_worker(_):
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import tcgen05_model  # noqa: F401

    return os.getpid()


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class PythonModel:
    """The reference Python model in a pool of one process per host core
    (started with spawn: the parent may already hold a CUDA context)."""

    def __init__(self):
        import multiprocessing as mp

        if not (REF_DIR / "tcgen05_model" / "__init__.py").exists():
            raise FileNotFoundError(f"the reference is not installed in {REF_DIR}")
        self.cores = host_cores()
        self.pool = mp.get_context("spawn").Pool(self.cores)
        self.pool.map(_warm_worker, range(self.cores))

    def run(self, tasks) -> tuple[list, float, float]:
        """(results in task order, wall seconds of the map, seconds inside the
        reference's calls summed over tasks)."""
        t0 = time.perf_counter()
        res = self.pool.map(_ref_worker, tasks, chunksize=1)
        wall = time.perf_counter() - t0
        return res, wall, sum(s for _, s in res)

    def close(self):
        self.pool.terminate()
        self.pool.join()


def sized_sample(model: PythonModel, tiles_host, target_s: float, cap: int = 1 << 15) -> int:
    """Cases per path of a sample that keeps all cores busy for about
    `target_s` seconds, from a calibration run of 256 cases per path."""
    tasks = sample_tasks(256, tiles_host)
    _, wall, _ = model.run(tasks)
    c = int(256 * target_s / max(wall, 1e-3)) // 256 * 256
    return max(256, min(cap, c))


def port_rate(tasks) -> tuple[float, int]:
    """The C port of the reference arithmetic (the oracle) on the same
    sample, all host threads: (element-MACs/s, threads)."""
    from oracle import oracle

    threads = oracle.default_threads()
    cases = [t for t in tasks if t[0] == "cases"]
    rows = [t for t in tasks if t[0] == "rows"]
    t0 = time.perf_counter()
    for t in cases:
        oracle.eval_cases(t[4], threads=threads)
    for t in rows:
        a, b, c = t[4]
        aa = np.repeat(a, TILE_N, axis=0)
        bb = np.tile(b.T, (a.shape[0], 1))
        oracle.mma_dot_batch(aa, bb, c.reshape(-1), a_format="bf16", threads=threads)
    elapsed = time.perf_counter() - t0
    return sum(task_macs(t) for t in tasks) / elapsed, threads


# --------------------------------------------------------------- our arm


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    import tcgen05_b200 as t5
    from tcgen05_b200 import _native as nat
    from tcgen05_b200 import workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"bench: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    lib = nat.load()
    stream = torch.cuda.current_stream(dev)
    items = build_step(torch, dev, rank, world, shard=args.shard)
    launch = launcher(lib, stream)

    def step():
        for item in items:
            launch(item)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    # the step's launches, captured once in a CUDA graph over STEP_STREAMS
    # streams (groups of about equal time from one measured step): each
    # timed step is one graph launch, so the host's launch rate never paces
    # the GPU, and independent paths overlap one another's start and tail;
    # within a stream the launches keep their programmatic dependencies
    graph, graph_note = None, "eager launches (graph capture unavailable)"
    try:
        groups = stream_groups(per_launch_times(torch, stream, items, launch, steps=1), args.streams)
        g = capture_step(torch, lib, dev, items, groups)
        g.replay()
        torch.cuda.synchronize(dev)
        graph = g
        graph_note = f"one CUDA graph of the step's launches per step, over {len(groups)} streams"
    except RuntimeError as exc:  # capture refused: time the launches eagerly
        print(f"bench: graph capture failed ({exc}); timing eager launches", file=sys.stderr)
        torch.cuda.synchronize(dev)

    def timed_step():
        if graph is not None:
            graph.replay()
        else:
            step()

    for _ in range(2):
        timed_step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(smi_gpu_id(local))
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        timed_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    elapsed_ms = e0.elapsed_time(e1)
    graph_words = [item.d.clone() for item in items] if graph is not None else None
    launch_ms = per_launch_times(torch, stream, items, launch)
    # the timed graph's words equal those of the launches run one by one
    graph_bad = 0 if graph_words is None else sum(int((w != item.d).sum()) for w, item in zip(graph_words, items))
    del graph_words
    mismatches, sums = verify(torch, lib, stream, items)
    mismatches += graph_bad
    nv = nvfp4_config(torch, dev, lib, stream, rank, world)

    # end to end through the public API on raw words in pinned host memory;
    # over N GPUs each rank takes whole paths by host bytes (the host link
    # bounds this step) and its share of the tiles
    host = host_step(torch, dev, e2e_items(torch, items, rank, world, args.shard))
    h2d, d2h = copy_bytes(host)
    e2e_step(t5, host)  # once untimed: the allocator then holds the buffers the timed runs need
    link_gbs = []
    for _ in range(E2E_CALIBRATIONS if world > 1 and args.shard == "paths" else 0):
        # the ranks' host links differ (shared uplinks and sockets), and how
        # much depends on what the others move: an untimed run of the step on
        # every rank at once gives each rank's rate under the current deal,
        # and the paths are dealt again by bytes over rate
        dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        e2e_step(t5, host)
        torch.cuda.synchronize(dev)
        rate = torch.zeros(world, dtype=torch.float64, device=dev)
        rate[rank] = (h2d + d2h) / (time.perf_counter() - t0) / 1e9
        dist.all_reduce(rate, op=dist.ReduceOp.SUM)
        link_gbs.append(rate.tolist())
        tile_bytes = sum(sum(x.numel() * x.element_size() for x in xs) + res.numel() * res.element_size()
                         for _item, kind, xs, _kw, res in host if kind == "tiles")
        del host
        host = host_step(torch, dev, e2e_items(torch, items, rank, world, args.shard,
                                               rates=link_gbs[-1], base_bytes=tile_bytes))
        h2d, d2h = copy_bytes(host)
        e2e_step(t5, host)
    # tile words against the timed launches' directly; each path's words by
    # their checksum, compared with the timed launches' after the reduction
    e2e_bad = sum(int((res.view(-1) != item.d.cpu().view(-1)).sum())
                  for item, kind, _, _, res in host if kind == "tiles")
    e2e_sums = {item.name: result_words_checksum(torch, item.first_case, res)
                for item, kind, _, _, res in host if kind == "cases"}
    e2e_runs = []
    for _ in range(E2E_RUNS):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        e2e_step(t5, host)
        torch.cuda.synchronize(dev)
        e2e_runs.append(time.perf_counter() - t0)
    e2e_s = statistics.median(e2e_runs)
    if world > 1:
        dist.barrier()
    ceiling_s = host_copy_ceiling(torch, dev, stream, host)

    # reductions over the job's launches (every path and the tiles, whichever
    # rank evaluates them): max of times over ranks, sums of counts and
    # checksums (a rank that does not evaluate a path adds 0)
    names = [spec.name for spec in workloads.validation_paths()] + ["matrix-bf16"]
    ms_by_name = {item.name: ms for item, ms in zip(items, launch_ms)}
    launch_ms = [ms_by_name.get(nm, 0.0) for nm in names]
    launches = len(items)
    by_rank = None
    if world > 1:
        # each rank's end-to-end time, copy ceiling and host bytes, in its own slot
        slots = torch.zeros(world, 3, dtype=torch.float64, device=dev)
        slots[rank] = torch.tensor([e2e_s, ceiling_s, float(h2d)], dtype=torch.float64)
        dist.all_reduce(slots, op=dist.ReduceOp.SUM)
        by_rank = {"e2e_s": slots[:, 0].tolist(), "host_copy_ceiling_s": slots[:, 1].tolist(),
                   "h2d_bytes": [int(x) for x in slots[:, 2].tolist()]}
        if link_gbs:
            by_rank["calibration_gbs"] = link_gbs
        t = torch.tensor([elapsed_ms, e2e_s, ceiling_s, nv["ms"]["nvfp4-k64"], nv["ms"]["nvfp4-sparse-k128"],
                          *launch_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_s, ceiling_s = float(t[0]), float(t[1]), float(t[2])
        nv["ms"] = {"nvfp4-k64": float(t[3]), "nvfp4-sparse-k128": float(t[4])}
        launch_ms = [float(x) for x in t[5:]]
        cnt = torch.tensor([mismatches, e2e_bad, nv["mismatches"], h2d, d2h, launches,
                            *[sums.get(nm, 0) for nm in names], *[e2e_sums.get(nm, 0) for nm in names]],
                           dtype=torch.int64, device=dev)
        dist.all_reduce(cnt, op=dist.ReduceOp.SUM)
        mismatches, e2e_bad, nv["mismatches"], h2d, d2h, launches = (int(x) for x in cnt[:6].tolist())
        sums = {nm: int(v) for nm, v in zip(names, cnt[6:6 + len(names)].tolist())}
        e2e_sums = {nm: int(v) for nm, v in zip(names, cnt[6 + len(names):].tolist())}
    # a path whose end-to-end words differ from the timed launches' counts as one mismatch
    e2e_bad += sum(1 for nm in names if nm != "matrix-bf16" and e2e_sums.get(nm, 0) != sums.get(nm, 0))
    step_macs = whole_step_macs()  # the configuration's work, however it is split over the ranks
    value = step_macs * args.steps / (elapsed_ms / 1e3)
    e2e_value = step_macs / e2e_s

    if rank == 0:
        line = report_line(args, world, items, names, launches, elapsed_ms, launch_ms, value, step_macs,
                           mismatches + e2e_bad, sums, nv, clocks, e2e_value, e2e_runs, e2e_s, ceiling_s, h2d, d2h,
                           torch, lib, stream)
        line["timed_launches"] = graph_note
        if by_rank is not None:
            line["e2e"]["by_rank"] = by_rank
        if world == 1 and not args.no_cpu_baseline:
            line.update(cpu_baselines(items, host, args.cpu_seconds))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if mismatches + e2e_bad == 0 else 1


def launch_table(world, items, names, shard) -> dict:
    """Kernel and algorithmic bytes of each of the job's launches as one rank
    runs it: a whole path (``shard="paths"``) or a rank's share of its cases,
    and a rank's share of the tiles (all ranks' shares are equal within one
    tile, so this rank's stands for all)."""
    from tcgen05_b200 import sweep, workloads
    from tcgen05_b200.step import kernel_of

    specs = {s.name: s for s in workloads.validation_paths()}
    own = {item.name: item for item in items}
    table = {}
    for nm in names:
        if nm in own:
            table[nm] = (own[nm].kernel, own[nm].bytes)
        else:
            lo, hi = (0, CASES_PER_PATH) if shard == "paths" else sweep.shard(CASES_PER_PATH, 0, world)
            table[nm] = (kernel_of(specs[nm]), sweep.path_work(specs[nm], hi - lo)[1])
    return table


def report_line(args, world, items, names, launches, elapsed_ms, launch_ms, value, step_macs, mismatches, sums, nv,
                clocks, e2e_value, e2e_runs, e2e_s, ceiling_s, h2d, d2h, torch, lib, stream) -> dict:
    from tcgen05_b200 import sweep, workloads

    peaks, peak_kind = measured_peaks()
    hbm = peaks["hbm_gbs"]
    specs = {s.name: s for s in workloads.validation_paths()}
    table = launch_table(world, items, names, args.shard)
    paths = {}
    for nm, ms in zip(names, launch_ms):
        job_macs = (sweep.path_work(specs[nm], CASES_PER_PATH)[0] if nm in specs
                    else MATRIX_TILES * TILE_M * TILE_N * TILE_K)
        kernel, nbytes = table[nm]
        gbs = nbytes / (ms / 1e3) / 1e9  # the launch as one rank runs it
        paths[nm] = {"kernel": kernel, "ms_per_launch": ms, "element_macs_per_s": job_macs / (ms / 1e3),
                     "hbm_frac": gbs / hbm, "checksum": f"{sums[nm] & 0xFFFFFFFFFFFFFFFF:016x}"}
    dom = max(range(len(names)), key=lambda j: launch_ms[j])
    dname, dms = names[dom], launch_ms[dom]
    dkernel, dbytes = table[dname]
    achieved = dbytes / (dms / 1e3) / 1e9
    tag = f"{dkernel} {dname}"
    traffic, traffic_state = profiled_figure("traffic_bytes_per_launch", tag, dkernel)
    # the ncu figures are for the full tile configuration on one GPU; a rank's
    # share of the tiles (or of a path's cases) does 1/N of it
    per_rank = world if (dname == "matrix-bf16" or args.shard == "cases") else 1
    if traffic is not None:
        traffic /= per_rank
    peak_issue = issue_peaks(torch, lib, stream)
    int_pipe = {"alu_peak_warp_inst_per_s": peak_issue["alu"], "fma_peak_warp_inst_per_s": peak_issue["fma"],
                "fp64_peak_warp_inst_per_s": peak_issue["fp64"],
                "source": "peaks: t5e_issue_probe in this run; kernel warp instructions per launch: the committed "
                          "ncu summary, used only while its source stamp matches the kernel's source"}
    fracs = {"hbm": achieved / hbm}
    for pipe in ("alu", "fma", "fp64"):
        per_launch, state = profiled_figure(f"{pipe}_warp_inst_per_launch", tag, dkernel)
        int_pipe[f"kernel_{pipe}_warp_inst_per_launch"] = per_launch
        int_pipe[f"{pipe}_figure"] = state
        if per_launch is not None:
            fracs[pipe] = per_launch / per_rank / (dms / 1e3) / peak_issue[pipe]
            int_pipe[f"{pipe}_frac"] = fracs[pipe]
    step_bytes = sum(item.bytes for item in items)
    nv_dense = NVFP4_CASES * 64 / (nv["ms"]["nvfp4-k64"] / 1e3)
    nv_sparse = NVFP4_CASES * 64 / (nv["ms"]["nvfp4-sparse-k128"] / 1e3)
    return {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "u32",
        "data": "synthetic: seeded counter-hash words with the reference harness's distributions "
                "(tcgen05_b200.sweep; numpy mirror for the host); uniformly random 32-bit tile words by the same "
                "hash of the global row and case index",
        "config": {"workload": "46-path validation sweep, 1M cases per path (46M total, sharded), plus matrix mma "
                               "BF16 M=128 N=256 K=16 F32 D, 4096 tiles (sharded)",
                   "cases_per_path": CASES_PER_PATH, "paths": 46, "matrix_tiles": MATRIX_TILES,
                   "element_macs_per_step": step_macs,
                   "l2": f"every batch read once per step; {step_bytes / 1e6:.0f} MB of inputs and outputs per "
                         f"step on rank 0's GPU > 126 MB L2",
                   "parallelism": (("whole paths per rank by measured cost, tile shards" if args.shard == "paths"
                                    else "case shards of every path, tile shards") + f" over {world} GPUs")
                                  if world > 1 else "single GPU"},
        "dot_products_per_s": (46 * CASES_PER_PATH + MATRIX_TILES * TILE_M * TILE_N) * args.steps
                              / (elapsed_ms / 1e3),
        "mismatches": mismatches,
        "mismatch_check": "every word of every launch against the generic kernel on the same inputs, every word "
                          "of the timed graph against the launches run one by one, the end-to-end tile words "
                          "against the timed launches' words, and each path's end-to-end words by their checksum "
                          "against the timed launches' (a differing path counts one)",
        "gpu_launches": args.steps * launches,
        "paths": paths,
        "kernel_ms_method": "an event between consecutive launches over 3 further steps, max over ranks",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": traffic, "traffic_figure": traffic_state,
                     "kernel": tag, "peak_source": f"{peak_kind} hbm_gbs (burst copy)",
                     "algorithmic_bytes_per_launch": dbytes, "ms_per_launch": dms,
                     "share_of_step": dms / sum(launch_ms), "int_pipe": int_pipe,
                     "binds": max(fracs, key=fracs.get),
                     "step": {"algorithmic_bytes": step_bytes, "gbs": step_bytes / (elapsed_ms / args.steps / 1e3) / 1e9,
                              "hbm_frac": step_bytes / (elapsed_ms / args.steps / 1e3) / 1e9 / hbm}},
        "nvfp4": {"workload": "NVFP4 E2M1 UE4M3 4X, 2^24 cases dense K=64 and 2^24 pairwise-sparse logical K=128 "
                              "(sharded)",
                  "dense": {"ms_per_launch": nv["ms"]["nvfp4-k64"], "element_macs_per_s": nv_dense},
                  "sparse": {"ms_per_launch": nv["ms"]["nvfp4-sparse-k128"], "element_macs_per_s": nv_sparse},
                  "mismatches_vs_generic": nv["mismatches"]},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "runs_s": e2e_runs, "reported": "median of the runs, max over ranks",
                "host_copy_ceiling_s": ceiling_s, "frac_of_host_copy_ceiling": ceiling_s / e2e_s,
                "calls": "mma_dot_batch per path and mma_batch for the tiles, raw uint32 container words in pinned "
                         "host memory, pinned out, wait=False, at most four calls in flight",
                "assignment": (f"whole paths per rank by host bytes over each rank's host-link rate, from "
                               f"{E2E_CALIBRATIONS} calibration runs, tile shares"
                               if world > 1 and args.shard == "paths" else "the timed launches' cases")},
        "clocks": clocks,
    }


def _tiles_numpy(host):
    """The step's matrix tiles as uint32 numpy arrays (A [T,M,K], B [T,K,N], C [T,M,N])."""
    for item, kind, (a, b, c), _kw, _res in host:
        if kind == "tiles":
            return a.numpy().view(np.uint32), b.numpy().view(np.uint32), c.numpy().view(np.uint32), item
    raise RuntimeError("no matrix tiles in the step")


def _sample_words_check(res, tasks, items, tiles_item) -> int:
    """Words of the sample that differ from the GPU's words of the same cases."""
    gpu = {item.name: item.d.cpu().numpy().view(np.uint32) for item in items}
    dm = tiles_item.d.cpu().numpy().view(np.uint32).reshape(-1, TILE_M, TILE_N)
    bad = 0
    for (words, _), task in zip(res, tasks):
        if task[0] == "rows":
            want = dm[task[2], task[3]:task[3] + ROW_BLOCK].reshape(-1)
        else:
            start, n = task[3], task[4].n
            want = gpu[task[1]][start:start + n]
        bad += int((words != want).sum())
    return bad


def cpu_baselines(items, host, seconds: float) -> dict:
    """The reference Python model on this host's cores (the CPU baseline of
    the metric) and the C port beside it, on one bounded sample of the step."""
    tiles = _tiles_numpy(host)
    a, b, c, tiles_item = tiles
    out = {}
    try:
        model = PythonModel()
    except (FileNotFoundError, OSError, ImportError) as exc:
        model = None
        out["cpu_baseline_note"] = f"reference Python model unavailable ({exc}); the C port is reported instead"
    if model is not None:
        try:
            per_path = sized_sample(model, (a, b, c), seconds)
            tasks = sample_tasks(per_path, (a, b, c))
            res, wall, busy = model.run(tasks)
        finally:
            model.close()
        macs = sum(task_macs(t) for t in tasks)
        rows = sum(1 for t in tasks if t[0] == "rows") * ROW_BLOCK
        out["cpu_baseline"] = {
            "value": macs / wall, "unit": UNIT, "cores": model.cores, "kind": "reference",
            "impl": "tcgen05_model (the reference Python package, installed in baseline/_ref): public mma_dot per "
                    "case (model built once per path) and mma on tile row blocks, one process per core",
            "sample": f"{per_path} cases of each of the 46 paths and {rows} rows of 256 tile cases "
                      f"({macs:.3g} element-MACs, the step's proportions), {wall:.1f} s wall",
            "core_seconds_in_reference_calls": busy,
            "mismatches_vs_gpu": _sample_words_check(res, tasks, items, tiles_item)}
    tasks = sample_tasks(2048, (a, b, c))
    rate, threads = port_rate(tasks)
    port = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
            "impl": "oracle/ (C restatement of the reference arithmetic)",
            "sample": "2048 cases of each path and the tile rows in the step's proportions"}
    if "cpu_baseline" in out:
        out["cpu_baseline_port"] = port
    else:
        out["cpu_baseline"] = port
    return out


# --------------------------------------------------------- reference arm


def run_reference(args) -> int:
    """The reference's own implementation (the Python tcgen05_model from
    baseline/_ref, through its public mma_dot and mma) on all host cores;
    each step is a bounded sample of the workload in its proportions."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    from tcgen05_b200 import workloads

    rng = np.random.Generator(np.random.PCG64(77))
    tiles = (workloads.f32_words(rng, 8 * TILE_M * TILE_K).reshape(8, TILE_M, TILE_K),
             workloads.f32_words(rng, 8 * TILE_K * TILE_N).reshape(8, TILE_K, TILE_N),
             workloads.f32_words(rng, 8 * TILE_M * TILE_N, finite_only=True).reshape(8, TILE_M, TILE_N))
    try:
        model = PythonModel()
    except (FileNotFoundError, OSError, ImportError) as exc:
        print(json.dumps({"impl": "reference", "unavailable": f"reference Python model not importable: {exc}"}))
        return 0
    try:
        budget = max(2.0, min(8.0, 90.0 / (args.steps + args.warmup)))  # the whole run stays near two minutes
        per_path = sized_sample(model, tiles, budget)
        tasks = sample_tasks(per_path, tiles)
        macs = sum(task_macs(t) for t in tasks)
        for _ in range(args.warmup):
            model.run(tasks)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model.run(tasks)
        elapsed = time.perf_counter() - t0
    finally:
        model.close()
    value = macs * args.steps / elapsed
    rows = sum(1 for t in tasks if t[0] == "rows") * ROW_BLOCK
    sample = (f"{per_path} cases of each of the 46 paths and {rows} rows of 256 BF16 tile cases per step "
              f"({macs:.3g} element-MACs, the step's proportions)")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "u32",
        "data": "synthetic: seeded counter-hash words with the reference harness's distributions",
        "config": {"workload": "46-path validation sweep plus BF16 matrix tiles (bounded sample per step)",
                   "cases_per_path_per_step": per_path, "tile_rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": model.cores, "kind": "reference",
                         "impl": "tcgen05_model from baseline/_ref: public mma_dot per case, mma on tile row "
                                 "blocks, one process per core", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=8.0,
                    help="wall seconds of the reference Python model's sample (all cores)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--streams", type=int, default=STEP_STREAMS,
                    help="streams the step's graph spreads its launches over")
    ap.add_argument("--shard", choices=("paths", "cases"), default="paths",
                    help="over N GPUs: whole paths per rank (by measured cost) or a share of every path's cases")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())

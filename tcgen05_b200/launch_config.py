"""Time one benchmark configuration's launches on inputs generated in HBM.

    python -m tcgen05_b200.launch_config --config nvfp4-k64 [--cases N]
        [--launches L] [--warmup W] [--generic] [--no-flush]

Prints one JSON line: mean CUDA-event time of a launch of t5e_mma_dot_batch
(or of the generic kernel), element-MACs/s, algorithmic GB/s and the number
of result words that differ from the generic kernel on the first 2^18 cases.
Between timed launches a 256 MB buffer is written so that no launch finds
its inputs in the 126 MB L2.  This is the command the kernel profiles are
taken with, and bench.py times the configurations through time_config.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import statistics

from . import _native as nat
from . import runtime, workloads


# Back-to-back timing rotates input sets until they hold this many bytes, so
# that no launch finds its inputs in the 126 MB L2.
ROTATION_BYTES = 384 << 20


def time_config(name: str, device, *, n: int | None = None, launches: int = 20, warmup: int = 3, seed: int = 0,
                generic: bool = False, flush: bool = True, check: bool = True, back_to_back: bool = False) -> dict:
    """Mean time of a launch.  Default: an event pair around each launch and a
    256 MB write before it.  back_to_back: the launches follow each other on
    the stream, cycling through input sets that together exceed the L2, with
    events only before and after the run (gaps between launches included)."""
    import torch

    lib = nat.load()
    model, db = workloads.device_config(name, device, seed=seed, n=n)
    desc = model.descriptor()
    stream = torch.cuda.current_stream(device)
    handle = ctypes.c_void_p(stream.cuda_stream)
    d = torch.empty(db.n, dtype=torch.int32, device=device)
    bs = runtime.make_batch_struct(db, d, None)
    fn = lib.t5e_mma_dot_batch_generic if generic else lib.t5e_mma_dot_batch

    def run(f, s):
        nat.check(f(ctypes.byref(desc), ctypes.byref(s), handle), name)

    if back_to_back:
        nbytes0 = workloads.config_work(name, db)[1]
        sets = [bs]
        keep = [(db, d)]  # the extra input sets and outputs stay alive while their structs are in use
        for j in range(1, -(-ROTATION_BYTES // nbytes0)):
            _, dbj = workloads.device_config(name, device, seed=seed + j, n=n)
            dj = torch.empty(dbj.n, dtype=torch.int32, device=device)
            keep.append((dbj, dj))
            sets.append(runtime.make_batch_struct(dbj, dj, None))
        for i in range(max(warmup, len(sets))):
            run(fn, sets[i % len(sets)])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        e0.record(stream)
        for i in range(launches):
            run(fn, sets[i % len(sets)])
        e1.record(stream)
        torch.cuda.synchronize(device)
        us = e0.elapsed_time(e1) * 1e3 / launches
        rotation = len(sets)
    else:
        buf = torch.empty(256 << 20, dtype=torch.uint8, device=device) if flush else None
        for _ in range(warmup):
            run(fn, bs)
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(launches)]
        for e0, e1 in events:
            if buf is not None:
                buf.zero_()
            e0.record(stream)
            run(fn, bs)
            e1.record(stream)
        torch.cuda.synchronize(device)
        us = statistics.mean(e0.elapsed_time(e1) for e0, e1 in events) * 1e3
        rotation = None
    mism = checked = None
    if check:
        per = db.tile_m * db.tile_n
        checked = min(db.n, max(per, (1 << 18) // per * per))
        sub = runtime.make_batch_struct(db, d, None)
        sub.n = checked
        ref = torch.empty(checked, dtype=torch.int32, device=device)
        sub_g = runtime.make_batch_struct(db, ref, None)
        sub_g.n = checked
        run(lib.t5e_mma_dot_batch, sub)
        run(lib.t5e_mma_dot_batch_generic, sub_g)
        torch.cuda.synchronize(device)
        mism = int((d[:checked] != ref).sum().item())
    macs, nbytes = workloads.config_work(name, db)
    return {"config": name, "cases": db.n, "k": db.k, "launches": launches, "kernel_us": us,
            "value": macs / (us * 1e-6), "dot_products_per_s": db.n / (us * 1e-6),
            "algorithmic_bytes": nbytes, "algorithmic_gbs": nbytes / (us * 1e-6) / 1e9,
            "mismatches_vs_generic": mism, "checked_cases": checked, "generic": generic,
            "timing": (f"back to back over {rotation} input sets" if back_to_back
                       else "event pair per launch, 256 MB written before each" if flush else "event pair per launch")}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", required=True, choices=sorted(workloads.CONFIG_SIZES))
    ap.add_argument("--cases", type=int, default=None, help="cases (default: the configuration's size)")
    ap.add_argument("--launches", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--generic", action="store_true")
    ap.add_argument("--no-flush", action="store_true")
    ap.add_argument("--back-to-back", action="store_true",
                    help="launches back to back over input sets larger than the L2, events around the run")
    args = ap.parse_args(argv)
    import torch

    device = runtime.require_device(None)
    res = time_config(args.config, device, n=args.cases, launches=args.launches, warmup=args.warmup,
                      seed=args.seed, generic=args.generic, flush=not args.no_flush, back_to_back=args.back_to_back)
    print(json.dumps(res), flush=True)
    del torch
    return 0 if not res["mismatches_vs_generic"] else 1


if __name__ == "__main__":
    raise SystemExit(main())

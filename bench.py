"""Benchmark: emulated element-MACs/s of the tcgen05 MMA emulator on B200.

Default workload (one step): the E4M3 x E5M2 dense mma_dot configuration,
K=32, 2^20 cases with F32 D plus its F16-D variant (2^20 cases), i.e.
2 x 2^20 bit-exact dot products = 2^26 element-MACs per step per GPU.
Inputs are resident in HBM; four distinct input sets (568 MB, above the 126 MB
L2) are rotated so that no step reads inputs left in L2 by the previous one.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank evaluates its own shard of the same size
(weak scaling); the timed region is bracketed by a barrier and a device
synchronisation, timed with CUDA events, and the maximum over ranks is
reported.  The only collective is the final reduction of timings and of the
mismatch count (specialised kernel vs generic kernel on every rank's inputs).

``--impl reference`` times the CPU restatement of the reference arithmetic
(oracle/, a C port of tcgen05_model) with all host threads on bounded
samples of the same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import ctypes
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
WORKLOAD = "e4m3xe5m2-k32"
VARIANTS = ("e4m3xe5m2-k32", "e4m3xe5m2-k32-f16")
K_ELEMS = 32
INPUT_SETS = 4
E2E_RUNS = 3


def algorithmic_bytes(variant: str, n: int) -> int:
    """A 32 B + B 32 B + C + D per case (C is 2 bytes for F16 C; D is always a
    32-bit word in this library's layout)."""
    c_bytes = 2 if variant.endswith("f16") else 4
    return n * (32 + 32 + c_bytes + 4)


def measured_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def profiled_figure(name: str, kernel_tag: str):
    """A figure of the dominant kernel from the committed ncu summaries (a line
    '<name>[<tag>]: <number>'), or None.  Used for the DRAM traffic per launch
    ('traffic_bytes_per_launch') and the ALU-pipe utilisation ('alu_pipe_pct')."""
    key = f"{name}[{kernel_tag}]:"
    for f in sorted((REPO / "profiles").glob("*.md")) + sorted((REPO / "profiles").glob("*.txt")):
        for line in f.read_text().splitlines():
            if line.strip().startswith(key):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


def _pct(x):
    return None if x is None else x / 100.0


def issue_peaks(torch, lib, stream, iters: int = 256, launches: int = 5) -> dict:
    """Measured issue rates (warp instructions/s) of the ALU and FMA pipes at
    the SM clock of the moment: the library's probe kernels issue a known
    number of independent LOP3/SHF (ALU) or IMAD (FMA) instructions at
    full occupancy; the best of `launches` event-timed launches per pipe."""
    from tcgen05_b200 import _native as nat

    handle = ctypes.c_void_p(stream.cuda_stream)
    out = {}
    for pipe, name in ((0, "alu"), (1, "fma")):
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


# --------------------------------------------------------------- our arm


def build_inputs(torch, device, rank: int, n: int):
    """INPUT_SETS x VARIANTS device batches in the kernels' packed layout."""
    import tcgen05_b200 as t5
    from tcgen05_b200 import _native as nat
    from tcgen05_b200 import packing, runtime, workloads

    sets = []
    for s in range(INPUT_SETS):
        per = []
        for variant in VARIANTS:
            cases = workloads.config_cases(variant, n, seed=100_003 * rank + 17 * s + (1 if variant.endswith("f16") else 0))
            d = cases.desc
            model = t5.make_model(d["a_format"], d.get("b_format"), d_type=d.get("d_type", "f32"))
            desc = model.descriptor()
            a = runtime.to_device(packing.pack_rows(cases.a, desc.a_format), device)
            b = runtime.to_device(packing.pack_rows(cases.b, desc.b_format), device)
            if desc.d_type == nat.D_F16:
                c = runtime.to_device((cases.c & 0xFFFF).astype(np.uint16).view(np.int16), device)
            else:
                c = runtime.to_device(cases.c, device)
            db = runtime.DeviceBatch(n=n, k=K_ELEMS, a=a, b=b, c=c)
            out = torch.empty(n, dtype=torch.int32, device=device)
            bs = runtime.make_batch_struct(db, out, None)
            per.append(dict(variant=variant, model=model, desc=desc, batch=db, struct=bs, d=out, cases=cases))
        sets.append(per)
    return sets


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    import tcgen05_b200 as t5
    from tcgen05_b200 import _native as nat

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"bench: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    lib = nat.load()
    n = args.cases
    sets = build_inputs(torch, device, rank, n)
    stream = torch.cuda.current_stream(device)
    handle = ctypes.c_void_p(stream.cuda_stream)

    def launch(item):
        rc = lib.t5e_mma_dot_batch(ctypes.byref(item["desc"]), ctypes.byref(item["struct"]), handle)
        if rc != 0:
            nat.check(rc, "t5e_mma_dot_batch")

    for w in range(args.warmup):
        for item in sets[w % INPUT_SETS]:
            launch(item)
    torch.cuda.synchronize(device)

    # The timed region launches the steps' kernels variant by variant: first every step's F32-D launch, then
    # every step's F16-D launch, each over the rotating input sets.  One event before, between and after
    # the two runs gives the whole region (value) and each variant's average launch duration (roofline);
    # an event pair around every launch would add about 3 us to each launch's gap.
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(len(VARIANTS) + 1)]
    sampler = ClockSampler(smi_gpu_id(local))
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    marks[0].record(stream)
    for j in range(len(VARIANTS)):
        for s in range(args.steps):
            launch(sets[s % INPUT_SETS][j])
        marks[j + 1].record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    elapsed_ms = marks[0].elapsed_time(marks[-1])
    variant_ms = [marks[j].elapsed_time(marks[j + 1]) for j in range(len(VARIANTS))]

    # verification: specialised dispatch vs generic kernel on this rank's inputs
    mismatches = 0
    for item in sets[0]:
        gen = torch.empty_like(item["d"])
        bs = item["struct"]
        saved = bs.d
        bs.d = gen.data_ptr()
        nat.check(lib.t5e_mma_dot_batch_generic(ctypes.byref(item["desc"]), ctypes.byref(bs), handle), "generic")
        bs.d = saved
        launch(item)
        torch.cuda.synchronize(device)
        mismatches += int((gen != item["d"]).sum().item())

    # end to end through the public API: pinned host inputs in, host words out
    e2e_steps = max(3, min(args.steps, args.e2e_steps))
    host = []
    h2d = d2h = 0
    for item in sets[0]:
        db = item["batch"]
        pa = db.a.cpu().pin_memory()
        pb = db.b.cpu().pin_memory()
        pc = db.c.cpu().pin_memory()
        out = torch.empty(n, dtype=torch.int32).pin_memory()
        host.append((item, pa, pb, pc, out))
        h2d += pa.numel() + pb.numel() + pc.numel() * pc.element_size()
        d2h += out.numel() * 4  # result words (dense batches carry no per-case status bytes)
    def e2e_run(steps, depth=4):
        # every call returns once its copies and kernels are queued (wait=False), so each batch's upload
        # follows the previous one on the link; at most `depth` calls are in flight, so the device buffers
        # they stream through come back to the allocator; every result word is in host memory when the
        # last wait returns
        pending = []
        for _ in range(steps):
            for item, pa, pb, pc, out in host:
                pending.append(t5.mma_dot_batch(t5.PackedRows(pa, K_ELEMS), t5.PackedRows(pb, K_ELEMS), pc,
                                                model=item["model"], out=out, wait=False))
                if len(pending) > depth:
                    pending.pop(0).wait()
        for p in pending:
            p.wait()

    e2e_run(e2e_steps)  # the same calls once untimed: the allocator then holds every buffer the timed run needs
    e2e_runs = []
    for _ in range(E2E_RUNS):  # the host link's rate varies from run to run: the median of three is reported
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        e2e_run(e2e_steps)
        torch.cuda.synchronize(device)
        e2e_runs.append(time.perf_counter() - t0)
    e2e_s = statistics.median(e2e_runs)
    ok_e2e = all(np.array_equal(out.numpy(), item["d"].cpu().numpy()) for item, _, _, _, out in host)

    if world > 1:
        t = torch.tensor([elapsed_ms, e2e_s, *variant_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_s = float(t[0]), float(t[1])
        variant_ms = [float(x) for x in t[2:]]
        mm = torch.tensor([mismatches + (0 if ok_e2e else 1)], dtype=torch.int64, device=device)
        dist.all_reduce(mm, op=dist.ReduceOp.SUM)
        mismatches = int(mm.item())
    else:
        mismatches += 0 if ok_e2e else 1

    cases_per_step = n * len(VARIANTS)
    macs_per_step = cases_per_step * K_ELEMS
    total_macs = macs_per_step * args.steps * world
    value = total_macs / (elapsed_ms / 1e3)
    e2e_value = macs_per_step * e2e_steps * world / e2e_s

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        dom = VARIANTS[0]
        launch_ms = {v: variant_ms[j] / args.steps for j, v in enumerate(VARIANTS)}  # mean per launch
        dom_ms = launch_ms[dom]
        bytes_per_launch = algorithmic_bytes(dom, n)
        achieved = bytes_per_launch / (dom_ms / 1e3) / 1e9
        hbm_frac = achieved / peaks["hbm_gbs"]
        peak_issue = issue_peaks(torch, lib, stream)
        int_pipe = {"source": "peaks: t5e_issue_probe, measured in this run; kernel warp instructions per launch "
                              "and pipe utilisation: ncu, committed profile"}
        fracs = {"hbm": hbm_frac}
        for pipe in ("alu", "fma"):
            per_launch = profiled_figure(f"{pipe}_warp_inst_per_launch", dom)
            int_pipe[f"{pipe}_peak_warp_inst_per_s"] = peak_issue[pipe]
            int_pipe[f"kernel_{pipe}_warp_inst_per_launch"] = per_launch
            if per_launch is not None:
                fracs[pipe] = per_launch / (dom_ms / 1e3) / peak_issue[pipe]
                int_pipe[f"{pipe}_frac"] = fracs[pipe]
        int_pipe["ncu_alu_pipe_frac"] = _pct(profiled_figure("alu_pipe_pct", dom))
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u32",
            "data": "synthetic (seeded PCG64, distributions of the E4M3xE5M2 configuration)",
            "config": {"workload": "E4M3xE5M2 dense mma_dot K=32, F32 D + F16-D variant",
                       "cases_per_step_per_gpu": cases_per_step, "k": K_ELEMS, "variants": list(VARIANTS),
                       "l2": f"{INPUT_SETS} rotating input sets, "
                             f"{INPUT_SETS * sum(algorithmic_bytes(v, n) for v in VARIANTS) / 1e6:.0f} MB > 126 MB L2",
                       "parallelism": f"dp{world}" if world > 1 else "single GPU"},
            "dot_products_per_s": value / K_ELEMS,
            "mismatches": mismatches,
            "gpu_launches": args.steps * len(VARIANTS),
            "kernel_ms": launch_ms,
            "kernel_ms_method": "events before, between and after the variant runs of the timed region; "
                                "mean over the variant's launches, gaps between launches included",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": hbm_frac,
                         "traffic": profiled_figure("traffic_bytes_per_launch", dom),
                         "kernel": f"t5e raw-window kernel, {dom}", "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_launch": bytes_per_launch,
                         "int_pipe": int_pipe,
                         "binds": max(fracs, key=fracs.get)},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    "runs_s": e2e_runs, "reported": "median of the runs",
                    "calls": "mma_dot_batch(pinned PackedRows, pinned out, wait=False) per batch, every wait "
                             "inside the timed region"},
            "clocks": clocks,
        }
        if world == 1 and not args.no_configs:
            line["configs"] = measure_configs(torch, device, lib)
            line["gpu_launches_configs"] = 23 * len(OTHER_CONFIGS)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(sets, budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if mismatches == 0 else 1


OTHER_CONFIGS = ("tf32-k8", "mx-e2m3xe3m2-k32", "u8xs8-k32-sat", "u8xs8-k32-wrap", "nvfp4-k64",
                 "nvfp4-sparse-k128", "matrix-bf16")


def measure_configs(torch, device, lib, launches: int = 20, warmup: int = 3) -> dict:
    """Every other benchmark configuration at its stated size, generated in
    HBM (tcgen05_b200.launch_config.time_config): the mean time of one launch
    of t5e_mma_dot_batch, launched back to back over input sets that together
    exceed the L2 with events around the run, as in the headline's timed
    region; element-MACs/s, algorithmic GB/s and its fraction of the measured
    HBM peak, and the number of result words that differ from the generic
    kernel on the first 2^18 cases."""
    from tcgen05_b200.launch_config import time_config

    peaks, _ = measured_peaks()
    out = {}
    for idx, name in enumerate(OTHER_CONFIGS):
        r = time_config(name, device, launches=launches, warmup=warmup, seed=1000 + idx, back_to_back=True)
        r["hbm_frac"] = r["algorithmic_gbs"] / peaks["hbm_gbs"]
        out[name] = r
        torch.cuda.empty_cache()
    return out


def cpu_baseline(sets, budget_s: float) -> dict:
    """The oracle (C port of the reference arithmetic) on a bounded sample of
    the same workload, all host threads; also checks the sample's words."""
    from oracle import oracle

    threads = oracle.default_threads()
    done_cases = 0
    elapsed = 0.0
    mism = 0
    sample = 1 << 17
    while elapsed < budget_s:
        for item in sets[0]:
            cases = item["cases"].subset(slice(0, sample))
            t0 = time.perf_counter()
            want = oracle.eval_cases(cases, threads=threads)
            elapsed += time.perf_counter() - t0
            done_cases += cases.n
            got = item["d"][:sample].cpu().numpy().view(np.uint32)
            mism += int((got != want).sum())
    return {"value": done_cases * K_ELEMS / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{done_cases} cases of the same workload (first {sample} of each variant, repeated), "
                      f"{elapsed:.1f} s", "mismatches_vs_gpu": mism}


# --------------------------------------------------------- reference arm


def run_reference(args) -> int:
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    from oracle import oracle
    from tcgen05_b200 import workloads

    threads = oracle.default_threads()
    pool = {v: workloads.config_cases(v, 1 << 18, seed=5) for v in VARIANTS}
    # calibrate, then size each step so the whole run stays within ~2 minutes of CPU time
    t0 = time.perf_counter()
    oracle.eval_cases(pool[VARIANTS[0]].subset(slice(0, 1 << 15)), threads=threads)
    rate = (1 << 15) / max(time.perf_counter() - t0, 1e-6)
    per_step = int(min(1 << 18, max(512, rate * 90.0 / (len(VARIANTS) * (args.steps + args.warmup)))))
    for w in range(args.warmup):
        for v in VARIANTS:
            oracle.eval_cases(pool[v].subset(slice(0, per_step)), threads=threads)
    t0 = time.perf_counter()
    for s in range(args.steps):
        for v in VARIANTS:
            oracle.eval_cases(pool[v].subset(slice(0, per_step)), threads=threads)
    elapsed = time.perf_counter() - t0
    macs = args.steps * len(VARIANTS) * per_step * K_ELEMS
    value = macs / elapsed
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
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u32",
        "data": "synthetic (seeded PCG64, distributions of the E4M3xE5M2 configuration)",
        "config": {"workload": "E4M3xE5M2 dense mma_dot K=32, F32 D + F16-D variant", "k": K_ELEMS,
                   "variants": list(VARIANTS), "cases_per_step": per_step * len(VARIANTS)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{per_step} cases per variant per step (bounded sample of the "
                                   f"2^20-case workload)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cases", type=int, default=1 << 20, help="cases per variant per GPU (default 2^20)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip timing the other configurations (run after the timed region, 1 GPU only)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())

"""The 46-path sweep driver: its counter-hash case generator (numpy and torch
produce the same words), the distributions it draws, its sharding and
cross-rank reduction (world size 2 over gloo on the CPU), its integrity
checks, and -- on a GPU -- every path against the oracle."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from tcgen05_b200 import sweep, workloads

PATHS = workloads.validation_paths()


@pytest.mark.parametrize("spec", PATHS, ids=lambda s: s.name)
def test_generator_numpy_and_torch_agree(spec):
    total = 1000
    g_np = sweep.generate(spec, 480, 40, total, np)  # straddles the raw/finite halves
    g_t = sweep.generate(spec, 480, 40, total, torch, torch.device("cpu"))
    for key, v in g_np.items():
        if v is None:
            assert g_t[key] is None
            continue
        assert np.array_equal(np.asarray(v, dtype=np.int64), g_t[key].numpy().astype(np.int64)), key


@pytest.mark.parametrize("spec", PATHS, ids=lambda s: s.name)
def test_generated_cases_are_valid_inputs(spec):
    """Words fit their containers, finite halves hold no specials, and the
    oracle accepts every case (legal metadata, matching scale counts)."""
    from oracle import oracle

    total = 512
    cases = sweep.host_cases(spec, 0, total, total)
    assert cases.k == sweep.path_k(spec)
    _, st = oracle.mma_dot_batch(cases.a, cases.b, cases.c, scale_a=cases.scale_a, scale_b=cases.scale_b,
                                 sparse_metadata=cases.meta, **{k: v for k, v in spec.descriptor.items()})
    assert (st == 0).all()
    d = spec.descriptor
    fin = cases.a[total // 2:]
    if spec.family == "dense" and d["a_format"] in ("tf32", "bf16"):
        assert not ((fin & 0x7F800000) == 0x7F800000).any()
        assert ((cases.a[: total // 2] & 0x7F800000) == 0x7F800000).any()
    if spec.family == "dense" and d["a_format"] == "e4m3":
        assert not ((fin & 0x7F) == 0x7F).any()
    if spec.family == "i8":
        assert cases.a[0].tolist() == [0] * 32 and cases.c[3] == 0x7FFFFFF0


def test_generator_is_shard_independent():
    spec = next(p for p in PATHS if p.name == "sparse-nvfp4")
    whole = sweep.host_cases(spec, 0, 300, 300)
    parts = sweep.host_cases(spec, 0, 100, 300).concat(sweep.host_cases(spec, 100, 200, 300))
    assert whole.digest() == parts.digest()


def _fake_evaluate(spec, lo, hi, total):
    """A device-free stand-in for the GPU evaluation: folds the generated C
    words (a deterministic function of the case index) into the checksum."""
    g = sweep.generate(spec, lo, hi - lo, total, np)
    idx = np.arange(lo, hi, dtype=np.int64)
    return hi - lo, 0, sweep.result_checksum(np, idx, np.asarray(g["c"], dtype=np.int64))


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rep = sweep.run_sweep(777, paths=PATHS[:6], rank=rank, world=world, evaluate=_fake_evaluate)
        q.put((rank, [(r["path"], r["cases"], r["checksum"]) for r in rep["results"]], rep["failed_paths"]))
    finally:
        dist.destroy_process_group()


def test_two_ranks_over_gloo_match_one_rank():
    import multiprocessing as mp

    single = sweep.run_sweep(777, paths=PATHS[:6], evaluate=_fake_evaluate)
    want = [(r["path"], r["cases"], r["checksum"]) for r in single["results"]]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, rows, failed in got:
        assert rows == want, rank
        assert failed == []


def test_shards_cover_every_case_once():
    for total in (1, 7, 1000, 1_000_000):
        for world in (1, 2, 3, 4, 8):
            bounds = [sweep.shard(total, r, world) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == total
            assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))


def test_integrity_checks():
    req = ["a", "b", "c"]
    ok = [{"path": p, "failed": False} for p in req]
    assert sweep.integrity(req, ok) == ([], [])
    bad = [{"path": "a", "failed": False}, {"path": "a", "failed": False}, {"path": "x", "failed": True}]
    failed, errors = sweep.integrity(req, bad)
    assert failed == ["b", "c", "x"]
    assert errors == ["missing paths: b, c", "duplicate paths: a", "unexpected paths: x"]


@pytest.mark.gpu
def test_gpu_sweep_every_path_matches_generic_and_oracle():
    from oracle import oracle

    dev = torch.device("cuda", 0)
    total = 8192
    rep = sweep.run_sweep(total, device=dev, chunk=3000)
    assert rep["failed_paths"] == [] and rep["integrity_errors"] == []
    assert all(r["mismatches"] == 0 and r["cases"] == total for r in rep["results"])
    for spec in PATHS:
        lo, hi = 4000, 4300  # straddles the raw/finite halves
        g = sweep.generate(spec, lo, hi - lo, total, torch, dev)
        got = sweep._device_eval(spec, g, dev, generic=False).cpu().numpy().astype(np.uint32)
        want = oracle.eval_cases(sweep.host_cases(spec, lo, hi - lo, total))
        assert np.array_equal(got, want), spec.name
    # the same report from two shards evaluated separately
    halves = [sweep.run_sweep(total, rank=r, world=1, device=dev, paths=PATHS[:4],
                              evaluate=lambda s, lo, hi, t, r=r: sweep._evaluate_shard_gpu(
                                  s, *sweep.shard(t, r, 2), t, dev, 4096)) for r in range(2)]
    whole = sweep.run_sweep(total, device=dev, paths=PATHS[:4])
    for i in range(4):
        s = (int(halves[0]["results"][i]["checksum"], 16) + int(halves[1]["results"][i]["checksum"], 16))
        assert s == int(whole["results"][i]["checksum"], 16)


def _host_cases_from_device(spec, g):
    """Device-generated cases copied to host memory in the oracle's form."""
    def words(x):
        if x is None:
            return None
        return torch.where(x >= 1 << 31, x - (1 << 32), x).to(torch.int32).cpu().numpy().view(np.uint32)

    def scales(x):
        return None if x is None else x.to(torch.uint8).cpu().numpy()

    return workloads.Cases(spec.descriptor, words(g["a"]), words(g["b"]), words(g["c"]), scales(g["scale_a"]),
                           scales(g["scale_b"]), words(g["meta"]), name=spec.name)


@pytest.mark.gpu
def test_gpu_every_path_at_full_size_matches_oracle():
    """Every path of the sweep at its full size (1M cases each, 46M in all):
    each device word equals the oracle's word for the same case.  The cases
    come from the device generator (the numpy mirror is checked above) and
    are copied to the host for the oracle."""
    from oracle import oracle

    dev = torch.device("cuda", 0)
    total, chunk = 1_000_000, 1 << 18
    bad = {}
    checked = 0
    for spec in PATHS:
        for lo in range(0, total, chunk):
            count = min(chunk, total - lo)
            g = sweep.generate(spec, lo, count, total, torch, dev)
            got = sweep._device_eval(spec, g, dev, generic=False).cpu().numpy().astype(np.uint32)
            want = oracle.eval_cases(_host_cases_from_device(spec, g))
            diff = np.flatnonzero(got != want)
            if diff.size:
                bad.setdefault(spec.name, []).append((lo + int(diff[0]), int(diff.size)))
            checked += count
    assert checked == total * len(PATHS)
    assert not bad, bad


def test_step_stream_groups_cover_every_launch_once_and_balance():
    from tcgen05_b200 import step

    times = [5.0, 1.0, 1.0, 4.0, 2.0, 2.0, 3.0, 0.5]
    groups = step.stream_groups(times, 3)
    flat = sorted(j for g in groups for j in g)
    assert flat == list(range(len(times)))
    assert all(g == sorted(g) for g in groups)  # launch order kept within a stream
    loads = [sum(times[j] for j in g) for g in groups]
    assert max(loads) - min(loads) <= max(times)
    assert step.stream_groups(times, 1) == [list(range(len(times)))]
    assert len(step.stream_groups([1.0, 2.0], 4)) == 2  # no empty streams


def test_path_owners_cover_every_path_once_with_balanced_cost():
    """Whole-path sharding: every rank computes the same assignment, each
    path has one owner, and no rank carries more than the average plus one
    path's cost."""
    from tcgen05_b200 import step, workloads

    names = [s.name for s in workloads.validation_paths()]
    assert set(step.PATH_COST_US) == set(names)
    assert step.path_owners(1) == {n: 0 for n in names}
    for world in (2, 3, 4, 8):
        owners = step.path_owners(world)
        assert owners == step.path_owners(world)
        assert set(owners) == set(names) and set(owners.values()) == set(range(world))
        load = [0.0] * world
        for n, r in owners.items():
            load[r] += step.PATH_COST_US[n]
        assert max(load) <= sum(load) / world + max(step.PATH_COST_US.values())


def test_host_path_owners_balance_host_bytes():
    """The end-to-end step deals whole paths by host bytes: every path has
    one owner, and no rank carries more than the average plus one path."""
    from tcgen05_b200 import step, workloads

    specs = workloads.validation_paths()
    per = {s.name: step.path_host_bytes(s) for s in specs}
    assert per["dense-tf32"] == 4 * (8 + 8) + 4 + 4
    assert per["sparse-nvfp4"] == 4 * (128 + 128) + 4 + 4 + 4 + 4 + 8
    for world in (1, 2, 8):
        owners = step.host_path_owners(world)
        assert set(owners) == set(per)
        load = [0] * world
        for n, r in owners.items():
            load[r] += per[n]
        assert max(load) <= sum(load) / world + max(per.values())


def test_host_path_owners_follow_each_ranks_link_rate():
    """Weighted by measured host-link rates, the deal gives a slower link
    fewer bytes and keeps every rank's time (bytes over rate, its tile bytes
    included) within one path of the balanced time; equal rates give the
    bytes-only deal, and the deal rejects a rate list of the wrong length."""
    from tcgen05_b200 import step, workloads

    specs = workloads.validation_paths()
    per = {s.name: step.path_host_bytes(s) * step.CASES_PER_PATH for s in specs}
    assert step.host_path_owners(8, rates=[5.0] * 8) == step.host_path_owners(8)
    rates = [28e9] * 4 + [36e9] * 4
    base = 170e6
    owners = step.host_path_owners(8, rates=rates, base_bytes=base)
    assert set(owners) == set(per)
    load = [base] * 8
    for n, r in owners.items():
        load[r] += per[n]
    assert max(load[:4]) < min(load[4:])
    times = [b / x for b, x in zip(load, rates)]
    balanced = sum(load) / sum(rates)
    assert max(times) <= balanced + max(per.values()) / min(rates)
    with pytest.raises(ValueError, match="one positive figure per rank"):
        step.host_path_owners(2, rates=[1.0])
    with pytest.raises(ValueError, match="one positive figure per rank"):
        step.host_path_owners(2, rates=[1.0, 0.0])


def _deal_worker(rank, world, port, q):
    """One rank of the end-to-end step's calibrated deal: its own host-link
    rate goes round an all-reduce, as bench.py does it, and the rank
    computes the deal from the reduced rates."""
    import torch
    import torch.distributed as dist

    from tcgen05_b200 import step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rate = torch.zeros(world, dtype=torch.float64)
        rate[rank] = 23.2 if rank == 0 else 34.7  # GB/s, the two link classes of an 8-GPU box
        dist.all_reduce(rate, op=dist.ReduceOp.SUM)
        q.put((rank, step.host_path_owners(world, rates=rate.tolist(), base_bytes=170e6)))
    finally:
        dist.destroy_process_group()


def test_calibrated_deal_is_the_same_on_every_rank_over_gloo():
    """Both ranks reach the same deal from the all-reduced rates, every path
    has one owner, and the rank with the slower link moves fewer bytes."""
    import multiprocessing as mp

    from tcgen05_b200 import step, workloads

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30000 + os.getpid() % 1000
    procs = [ctx.Process(target=_deal_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1]
    per = {s.name: step.path_host_bytes(s) * step.CASES_PER_PATH for s in workloads.validation_paths()}
    assert set(got[0]) == set(per)
    load = [sum(per[n] for n, r in got[0].items() if r == k) for k in (0, 1)]
    assert load[0] < load[1]

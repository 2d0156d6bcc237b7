#!/usr/bin/env python
"""Benchmark of mojodgl's B200 message-passing hot path (driver contract).

Workload (the metric's multi-GPU config): a GraphSAGE-style
aggregation on a synthetic 125M-edge power-law graph, N = 2.5M nodes,
out-degrees lognormal(3.2, 1.3) capped at 20,000 and scaled to sum to exactly
125,000,000 (floor + largest remainder), src-major edge order, destinations
uniform, h = (N, 128) float32 ~ U(-1, 1); draws in that order from
numpy.random.default_rng(3).  One step = one gSpMM copy_u_mean over all edges
(``ops.copy_u_mean``), the config's first op; copy_u_max with arg-index output
and copy_u_sum are timed beside it under "ops".

Multi-GPU (torchrun, one rank per GPU): strong scaling of the same graph on
an R x C rank grid (C = --cols, by default GRID_COLS[N]): a rank aggregates
the destination rows of its row group (R ranges balanced by in-edge count)
for the feature columns of its column group (C contiguous column blocks), and
owns one block of rows of its column block.  With --halo peer (the default)
a step pulls the column group's other owner blocks straight from the peers'
memory by copy-engine copies over NVLink (CUDA IPC mappings, no SM time) and
runs one accumulating gSpMM pass per owner block -- its own block's at once,
each peer's as its copy lands -- so the halo overlaps the aggregation.  With
--halo allgather the blocks are gathered slice by slice instead (each cut
into --halo-slices row slices, one NCCL all-gather per slice within the
column group, one pass per slice).  With one row group (R = 1) a rank
already holds every row of its columns and the step is one gSpMM.
"allgather_then_compute" times the unpipelined alternative (one all-gather,
then the local gSpMM), "allgather_only" the collective alone,
"peer_pulls_only" the copy-engine pulls alone and "compute_only" the local
gSpMM alone.

After every timed region the step's result is checked on a seeded sample of
rows against the float64 oracle ("parity"; each rank its own rows).

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU
restatement of the reference's Mojo kernels (oracle/, the reference itself
cannot be built here) on the whole config-3 workload and prints its line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mojo-dgl_b200"))
sys.path.insert(0, ROOT)

CFG3 = dict(num_nodes=2_500_000, num_edges=125_000_000, dim=128, seed=3)
METRIC = "gSpMM Gedge-feat/s"
UNIT = "Gedge-feat/s"
HALO_SLICES = 2  # row slices of each owner block in the all-gather halo (--halo allgather)
# column groups of the rank grid by GPU count (R = N / C row groups).  Measured
# on config 3 (8 x B200, copy-engine halo, ms per step): N = 2: 2 x 1 3.78
# (1 x 2, no exchange: 4.22); N = 4: 2 x 2 2.09, 4 x 1 2.19 (1 x 4: 2.40);
# N = 8: 2 x 4 1.28, 4 x 2 1.38, 8 x 1 1.83 (1 x 8: 1.60).  The pulls take no
# SMs, so a grid wins while its halo (R - 1 blocks at 520-730 GB/s per rank)
# stays under the gSpMM's time; narrower column blocks cost gSpMM efficiency.
GRID_COLS = {2: 1, 4: 2, 8: 4}


# ----------------------------------------------------------------- workload
def make_cfg3(num_nodes, num_edges, dim, seed, with_h=True):
    """Config 3's graph (and features) as numpy arrays, in the draw order of
    the module docstring."""
    rng = np.random.default_rng(seed)
    w = np.minimum(rng.lognormal(3.2, 1.3, num_nodes), 20_000.0)
    x = w * (num_edges / w.sum())
    deg = np.floor(x).astype(np.int64)
    short = num_edges - int(deg.sum())
    if short > 0:
        deg[np.argsort(-(x - deg), kind="stable")[:short]] += 1
    u = np.repeat(np.arange(num_nodes, dtype=np.int64), deg)
    v = rng.integers(0, num_nodes, num_edges, dtype=np.int64)
    h = None
    if with_h:
        h = rng.random((num_nodes, dim), dtype=np.float32)
        h *= 2.0
        h -= 1.0
    return u, v, h


def algorithmic_bytes(num_rows, num_edges, dim, elem=4, arg=False):
    """Gathered model: every edge's source row counted once per edge, plus
    the int32 neighbour ids, the output rows and the int64 row pointers
    (+ int64 arg indices for max/min)."""
    b = num_edges * dim * elem + num_edges * 4 + num_rows * dim * elem + (num_rows + 1) * 8
    if arg:
        b += num_rows * dim * 8
    return b


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (read-only queries)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ CPU baselines
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_threads(world=1):
    """Host threads for the oracle: all of them (up to the reference's 32
    workers) for the timed CPU arm; a share per rank for checks at N > 1.
    torchrun exports OMP_NUM_THREADS=1 to its ranks and the oracle's OpenMP
    runtime reads the variable when it is first loaded, so this runs before
    the first import of oracle."""
    threads = max(1, min(32, cpu_threads() // max(world, 1)))
    os.environ["OMP_NUM_THREADS"] = str(threads)
    return threads


def host_csr(u, v, num_nodes):
    """The reference's in-CSR of the whole graph (heterograph.py:69-86) on the
    host, int64, through the oracle's O(E) counting sort (= stable argsort)."""
    from oracle import oracle as orc

    indptr, deg, order, indices = orc.csr_arrays(v, u, num_nodes)
    return indptr, indices, order, deg


def time_oracle(csr, h, num_nodes, dim, calls):
    """The CPU restatement of the reference kernel (fp64, its 32-worker split
    over every host thread OpenMP offers) on the WHOLE config-3 graph:
    copy_u_mean through mdgl_gspmm, once per call.  Returns the per-call
    seconds, the thread count and a description."""
    from oracle import oracle as orc

    lib = orc.lib()
    indptr, indices, eid, deg = csr
    h64 = np.ascontiguousarray(h, dtype=np.float64)  # the reference's f64() gate
    out = np.empty((num_nodes, dim), dtype=np.float64)
    secs = []
    for _ in range(calls):
        t0 = time.perf_counter()
        lib.mdgl_gspmm(indptr.ctypes.data, indices.ctypes.data, eid.ctypes.data, h64.ctypes.data,
                       h64.ctypes.data, out.ctypes.data, num_nodes, 5, dim, dim, dim, 3,
                       deg.ctypes.data)
        secs.append(time.perf_counter() - t0)
    desc = ("copy_u_mean over the whole config-3 graph ({} destination rows, {} edges), fp64, "
            "{} OpenMP threads over the reference's 32-worker split".format(
                num_nodes, int(indices.size), int(lib.oref_threads())))
    return secs, int(lib.oref_threads()), desc


def check_parity(u, v, h, indeg, out, lo, hi, num_nodes, seed, rows=20_000, top=1000):
    """Sampled oracle check of a copy_u_mean result: ``out`` holds the rows
    [lo, hi) (a device tensor or a host array).  ``rows`` random rows of the
    range plus its ``top`` highest in-degree rows are recomputed by the float64
    oracle on their own in-edges (oracle/sampled.py) and compared under the
    suite's float32 bound |got - ref| <= 1e-5 |ref| + 1e-5 S, S = mean |h| of
    the row's sources.  Runs outside every timed region."""
    from oracle import oracle as orc
    from oracle import sampled as smp

    pick = smp.sample_rows(indeg[lo:hi], rows, top, seed) + lo
    s = smp.RowSample(u, v, pick, num_nodes)
    local = s.rows - lo
    if hasattr(out, "cpu"):
        import torch

        got = out[torch.from_numpy(local).to(out.device)].cpu().numpy()
    else:
        got = np.asarray(out)[local]
    worst, max_err = -np.inf, 0.0
    for sl, lg in s.batches(1 << 20):
        hl = h[lg.nodes]
        ref = orc.gspmm(lg.graph, "copy_lhs", "mean", hl, None)[lg.rows]
        bound = orc.gspmm(lg.graph, "copy_lhs", "mean", np.abs(hl), None)[lg.rows]
        ex, me = smp.excess(got[sl], ref, bound, 1e-5)
        worst, max_err = max(worst, ex), max(max_err, me)
    return {"rows": int(s.rows.size), "edges": int(s.num_edges), "max_abs_err": max_err,
            "max_excess": worst, "ok": bool(worst <= 0.0)}


# --------------------------------------------------------------- main paths
def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), \
        int(os.environ.get("LOCAL_RANK", 0))


def run_reference(args):
    """The reference's CPU path (the C restatement of its Mojo kernel, which
    cannot be built here) on the whole config-3 graph: W warm-up calls, then
    K timed calls; ms_per_step is the best timed call (the reference's own
    best-of statistic, bench/bench.py:80-86), the median beside it."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = oracle_threads()
    c = CFG3
    n, e, d = c["num_nodes"], c["num_edges"], c["dim"]
    u, v, h = make_cfg3(**c)
    csr = host_csr(u, v, n)
    del u, v
    secs, threads, desc = time_oracle(csr, h, n, d, args.warmup + args.steps)
    secs = secs[args.warmup:]
    best, med = min(secs), statistics.median(secs)
    value = e * d / best / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": best * 1e3,
        "median_ms_per_step": med * 1e3, "statistic": "best of the timed calls",
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": "cfg3 copy_u_mean (BASELINE config 3): N=2.5M, E=125M "
                               "lognormal out-degree, D=128, whole graph, fp64 on the host",
                   "num_nodes": n, "num_edges": e, "dim": d, "seed": c["seed"],
                   "parallelism": "cpu, {} threads".format(threads)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc + " (whole workload, best of {})".format(len(secs))},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's Mojo library cannot be built in this image (no Mojo toolchain); "
                "this arm times oracle/ported_ref.c, a C restatement of src/ported.mojo",
    }
    print(json.dumps(line), flush=True)
    return 0


# DRAM bytes (read + write) of one k_spmm copy_u mean launch over the whole
# config-3 graph: ncu captures at 0.25 and 0.5 of the edges, reads fitted
# linearly in the edge count and extrapolated to 125M edges, writes (the
# N x D output) constant (profiles/gspmm_copy_u_cfg3_traffic_scales.md).
TRAFFIC_SCALED = {"cfg3_copy_u_mean_world1": 50_570_000_000}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import mojodgl as dgl
    from mojodgl import ops
    from mojodgl.partition import (DeviceShard, DstShard, PeerPipeline, SlicePipeline,
                                   column_group_ranks, column_range, edge_balanced_ranges,
                                   owner_blocks, pull_order, rank_grid)

    rank, world, local = dist_env()
    oracle_threads(world)  # the parity check (and at N=1 the CPU arm) run the oracle later
    if world > 1:
        torch.cuda.set_device(local)
        import datetime

        # NCCL's kernels on high-priority streams: the halo's all-gathers then
        # take SMs as the (HBM-bound) gSpMM's blocks retire instead of waiting
        # for the whole grid
        nccl_opts = dist.ProcessGroupNCCL.Options()
        nccl_opts.is_high_priority_stream = not args.nccl_normal_priority
        pg_timeout = datetime.timedelta(seconds=120)
        dist.init_process_group("nccl", timeout=pg_timeout,
                                device_id=torch.device("cuda", local), pg_options=nccl_opts)
    dev = torch.device("cuda", local)
    c = dict(CFG3)
    c["num_edges"] = int(round(c["num_edges"] * args.scale))
    if args.dim > 0:
        c["dim"] = args.dim
    full_size = args.scale == 1.0 and c["dim"] == CFG3["dim"]
    n, e_total, d = c["num_nodes"], c["num_edges"], c["dim"]
    u, v, h = make_cfg3(**c)

    # -------- this rank's place in the R x C grid, its graph shard (dst rows
    # balanced by in-edges within its row group) and its feature columns
    cols = args.cols if args.cols > 0 else GRID_COLS.get(world, 1)
    rows_n, rg, cg = rank_grid(rank, world, cols)
    grp = None
    if world > 1 and cols > 1:
        # every rank creates every column group, in the same order
        groups = [dist.new_group(r, timeout=pg_timeout, pg_options=nccl_opts)
                  for r in column_group_ranks(world, cols)]
        grp = groups[cg]
    indeg = np.bincount(v, minlength=n)
    bounds = edge_balanced_ranges(indeg, rows_n)
    lo, hi = int(bounds[rg]), int(bounds[rg + 1])
    c0, c1 = column_range(d, cols, cg)
    dc = c1 - c0
    shard = DeviceShard(DstShard(u, v, lo, hi))
    peer = rows_n > 1 and args.halo == "peer"
    if rows_n == 1:
        pipe = None
    elif peer:
        pipe = PeerPipeline(u, v, lo, hi, rg, rows_n, n, dc, group=grp)
    else:
        pipe = SlicePipeline(u, v, lo, hi, rg, rows_n, n, slices=args.halo_slices, group=grp)
    blk, owners = owner_blocks(n, rows_n)
    own_lo, own_hi = owners[rg]
    hc = np.ascontiguousarray(h[:, c0:c1]) if cols > 1 else h
    # this rank's feature columns for every row: with one row group that is
    # the rank's own data; otherwise it serves the kernel-only timings
    h_dev = torch.from_numpy(hc).to(dev)
    gathered = torch.empty((blk * rows_n, dc), dtype=torch.float32, device=dev)
    # this rank's owner block, padded to whole slices for the sliced gather
    my_block = torch.zeros((pipe.block_rows() if pipe and not peer else blk, dc),
                           dtype=torch.float32, device=dev)
    my_block[: own_hi - own_lo] = h_dev[own_lo:own_hi]
    if peer:
        pipe.own_block().copy_(h_dev[own_lo:own_hi])
    out = torch.empty((hi - lo, dc), dtype=torch.float32, device=dev)
    ws = None
    torch.cuda.synchronize()

    bufs = ([torch.empty((rows_n * pipe.sb, dc), dtype=torch.float32, device=dev)
             for _ in range(2)] if pipe and not peer else None)
    pws = [None]

    def step():
        # the halo overlapped with the aggregation: the peers' owner blocks
        # arrive by copy-engine pulls (or slice by slice by all-gathers) while
        # the passes over the blocks already in run; one row group needs no
        # exchange
        if peer:
            pipe.copy_u("mean", out, ws=pws)
        elif pipe:
            pipe.copy_u(my_block, "mean", out, bufs=bufs, ws=pws)
        else:
            shard.copy_u(h_dev, "mean", out=out, workspace=ws)

    def step_allgather():
        dist.all_gather_into_tensor(gathered, my_block[:blk], group=grp)
        shard.copy_u(gathered, "mean", out=out, workspace=ws)

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            fn()
        s1.record()
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # the whole step (halo + local gSpMM): the headline value
    with ClockSampler(local) as clocks:
        ms_step = timed(step, args.steps, args.warmup)
    ms_allgather = timed(step_allgather, args.steps, 1) if pipe else None
    # the all-gather alone (the collective that bounds the step when R > 1)
    ms_gather_only = (timed(lambda: dist.all_gather_into_tensor(gathered, my_block[:blk],
                                                                group=grp),
                            args.steps, 1) if pipe else None)

    # the copy-engine pulls alone (every peer block, on the timed stream)
    def pulls_only():
        for q in pull_order(rg, rows_n):
            pipe.pull(q, torch.cuda.current_stream())

    ms_pulls_only = timed(pulls_only, args.steps, 1) if peer else None
    # the gSpMM call alone (coords + main + fixup kernels) for the roofline
    feat = h_dev
    ms_kernel = timed(lambda: shard.copy_u(feat, "mean", out=out, workspace=ws), args.steps, 1)
    value = e_total * d / (ms_step * 1e-3) / 1e9

    # other ops of the config, device resident, this rank's shard
    extra = {}
    arg_u = torch.empty((hi - lo, dc), dtype=torch.int64, device=dev)
    for name, red, arg in (() if args.no_extra else
                           (("copy_u_sum", "sum", None), ("copy_u_max+arg_u", "max", arg_u))):
        ms_op = timed(lambda: shard.copy_u(feat, red, out=out, arg_u=arg), args.steps, 1)
        extra[name] = {"ms": ms_op, "Gedge_feat_s": e_total * d / (ms_op * 1e-3) / 1e9 if world == 1
                       else None,
                       "achieved_GBps": algorithmic_bytes(hi - lo, shard.shard.num_edges, dc,
                                                          arg=arg is not None) / (ms_op * 1e-3) / 1e9}
    del arg_u
    # the headline op in float64, the reference's precision (same bgl_gspmm)
    if not args.no_extra:
        h64 = h_dev.double()
        out64 = torch.empty((hi - lo, dc), dtype=torch.float64, device=dev)
        ms_op = timed(lambda: shard.copy_u(h64, "mean", out=out64), args.steps, 1)
        extra["copy_u_mean_f64"] = {
            "ms": ms_op, "Gedge_feat_s": e_total * d / (ms_op * 1e-3) / 1e9 if world == 1 else None,
            "achieved_GBps": algorithmic_bytes(hi - lo, shard.shard.num_edges, dc, elem=8)
            / (ms_op * 1e-3) / 1e9}
        del h64, out64

    # -------- parity: the timed step's result rows, sampled, against the
    # oracle (after every timed region; each rank checks its own rows)
    step()
    torch.cuda.synchronize()
    parity = check_parity(u, v, hc, indeg, out, lo, hi, n, seed=300 + rank)
    if world > 1:
        t = torch.tensor([parity["max_excess"], parity["max_abs_err"], parity["rows"],
                          parity["edges"]], dtype=torch.float64, device=dev)
        w = t.clone()
        dist.all_reduce(w, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        parity = {"rows": int(t[2]), "edges": int(t[3]), "max_abs_err": float(w[1]),
                  "max_excess": float(w[0]), "ok": bool(float(w[0]) <= 0.0),
                  "ranks": world}

    # -------- e2e through the public API with host buffers
    e2e = None
    if args.no_e2e:
        pass
    elif world == 1:
        g = dgl.graph((u, v), num_nodes=n)
        g._device()  # the graph (its device CSR) is built once, like a user's
        h_pin = torch.from_numpy(h).pin_memory()
        # warm up exactly as the timed loop runs: the previous result is still
        # held while the next is allocated, so two pinned result buffers must
        # already be in torch's pinned-memory cache when timing starts
        r = None
        for _ in range(3):
            r = ops.copy_u_mean(g, h_pin)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            r = ops.copy_u_mean(g, h_pin)
        torch.cuda.synchronize()
        dt = (time.perf_counter() - t0) / args.steps
        e2e = {"value": e_total * d / dt / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": int(h.nbytes), "d2h_bytes_per_step": int(r.numel() * 4),
               "ms_per_step": dt * 1e3, "path": "ops.copy_u_mean(g, pinned CPU tensor)",
               "parity": check_parity(u, v, h, indeg, r.numpy(), 0, n, n, seed=400,
                                      rows=5000, top=100)}
        del g, h_pin, r
    else:
        # per rank: its owned piece of h (host, pinned) in, its output piece out
        h_pin = torch.from_numpy(np.ascontiguousarray(hc[own_lo:own_hi] if pipe else hc)).pin_memory()
        out_pin = torch.empty((hi - lo, dc), dtype=torch.float32).pin_memory()

        def e2e_step():
            if peer:
                pipe.own_block().copy_(h_pin, non_blocking=True)
            elif pipe:
                my_block[: own_hi - own_lo].copy_(h_pin, non_blocking=True)
            else:
                h_dev.copy_(h_pin, non_blocking=True)
            step()
            out_pin.copy_(out, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        for _ in range(2):
            e2e_step()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        dt = time.perf_counter() - t0
        t = torch.tensor([dt / args.steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
        e2e = {"value": e_total * d / dt / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": int(h.nbytes), "d2h_bytes_per_step": int(n * d * 4),
               "ms_per_step": dt * 1e3,
               "path": "per rank: its pinned piece of h H2D, the halo within its column group "
                       "({}) overlapped with gSpMM passes (none with one row group), its output "
                       "piece D2H".format("copy-engine pulls" if peer else
                                          "sliced all-gathers")}

    # -------- roofline of the dominant kernel (this rank's gSpMM)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    alg = algorithmic_bytes(hi - lo, shard.shard.num_edges, dc)
    achieved = alg / (ms_kernel * 1e-3) / 1e9
    traffic = (TRAFFIC_SCALED.get("cfg3_copy_u_mean_world{}".format(world))
               if cols == 1 and full_size else None)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "traffic_source": "scaled" if traffic else None,
                "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                "kernel": "bgl_gspmm copy_u mean (k_spmm_coords + k_spmm + k_spmm_fixup)",
                "algorithmic_bytes": alg, "kernel_ms": ms_kernel}
    if traffic:
        # the algorithmic model counts every gathered row as a DRAM read; L2
        # serves the rows of high out-degree sources, so the measured DRAM
        # traffic is lower and its rate is the one to hold against the peak
        roofline["traffic_GBps"] = traffic / (ms_kernel * 1e-3) / 1e9
        roofline["traffic_frac"] = roofline["traffic_GBps"] / peak

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        csr = host_csr(u, v, n)
        secs, threads, desc = time_oracle(csr, h, n, d, 3)
        del csr
        cpu = {"value": e_total * d / min(secs) / 1e9, "unit": UNIT, "cores": threads,
               "kind": "port", "ms": min(secs) * 1e3,
               "sample": desc + " (whole workload, best of 3)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg3 copy_u_mean (BASELINE config 3): N=2.5M, E=125M "
                                   "lognormal out-degree, D=128 fp32" if full_size else
                                   "cfg3 copy_u_mean with edges scaled by {} and D={} (profiling "
                                   "case)".format(args.scale, d),
                       "num_nodes": n, "num_edges": e_total, "dim": d, "seed": c["seed"],
                       "parallelism": "single GPU" if world == 1 else
                       "{} x {} rank grid: dst-row shards x{} (balanced by in-edges) x feature-column "
                       "blocks x{}; {}".format(rows_n, cols, rows_n, cols,
                                               "halo by copy-engine pulls of the column group's "
                                               "owner blocks over NVLink (CUDA IPC), overlapped "
                                               "with one gSpMM pass per block" if peer else
                                               "halo by {} sliced all-gathers per step within each "
                                               "column group, overlapped with gSpMM passes".format(
                                                   args.halo_slices) if pipe else
                                               "no exchange (each rank owns its column block)"),
                       "grid": [rows_n, cols],
                       "halo": "peer" if peer else "allgather" if pipe else "none",
                       "halo_slices": args.halo_slices if pipe and not peer else 0,
                       "l2": "inputs larger than L2 (h 1.28 GB, indices 0.5 GB)"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            # per gSpMM call: coordinates, main and fixup kernels; at N > 1 one
            # call per owner block (peer halo: copy-engine copies, no kernels;
            # the fences are NCCL's) or per halo slice (NCCL's all-gathers)
            "gpu_launches": 3 * (rows_n if peer else args.halo_slices if pipe else 1) * args.steps,
            "clocks": clocks.summary(), "ops": extra, "parity": parity,
            "allgather_then_compute": None if ms_allgather is None else
            {"value": e_total * d / (ms_allgather * 1e-3) / 1e9, "unit": UNIT,
             "ms_per_step": ms_allgather,
             "what": "one NCCL all-gather of the features, then the local gSpMM (no overlap)"},
            "allgather_only": None if ms_gather_only is None else
            {"ms": ms_gather_only, "bytes_received_per_rank": blk * (rows_n - 1) * dc * 4,
             "GBps_per_rank": blk * (rows_n - 1) * dc * 4 / (ms_gather_only * 1e-3) / 1e9,
             "what": "one NCCL all_gather_into_tensor of the owner blocks (the step's halo), alone"},
            "peer_pulls_only": None if ms_pulls_only is None else
            {"ms": ms_pulls_only, "bytes_received_per_rank": blk * (rows_n - 1) * dc * 4,
             "GBps_per_rank": blk * (rows_n - 1) * dc * 4 / (ms_pulls_only * 1e-3) / 1e9,
             "what": "the copy-engine pulls of the peers' owner blocks (the step's halo), alone"},
            "compute_only": {"value": e_total * d / (ms_kernel * 1e-3) / 1e9, "unit": UNIT,
                             "ms_per_step": ms_kernel,
                             "what": "local gSpMM only (features already replicated), max over ranks"},
        }
        print(json.dumps(line), flush=True)
    if peer:
        pipe.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------- suite
def make_cfg2(seed=2, n=1_000_000, mean=16, cap=50_000):
    """Config 2: Zipf(2.1) in-degrees capped at 50,000, rescaled to mean 16
    keeping the cap, largest-remainder rounding; uniform sources; edges
    shuffled."""
    rng = np.random.default_rng(seed)
    x = np.minimum(rng.zipf(2.1, n), cap).astype(np.float64)
    total = mean * n
    for _ in range(100):
        capped = x >= cap
        free = x[~capped].sum()
        scale = (total - cap * capped.sum()) / free
        y = np.where(capped, float(cap), np.minimum(x * scale, float(cap)))
        if np.allclose(y, x):
            break
        x = y
    deg = np.floor(x).astype(np.int64)
    short = total - int(deg.sum())
    if short > 0:
        deg[np.argsort(-(x - deg), kind="stable")[:short]] += 1
    v = np.repeat(np.arange(n, dtype=np.int64), deg)
    u = rng.integers(0, n, v.size, dtype=np.int64)
    p = rng.permutation(v.size)
    return u[p], v[p]


def make_cfg5(seed=5, n=5_000_000, e=50_000_000):
    """Config 5: uniform edges; geometric(1/32) segment lengths summing to E."""
    rng = np.random.default_rng(seed)
    u = rng.integers(0, n, e, dtype=np.int64)
    v = rng.integers(0, n, e, dtype=np.int64)
    lens = rng.geometric(1 / 32, size=e // 32 + 1000)
    c = np.cumsum(lens)
    k = int(np.searchsorted(c, e)) + 1
    seglen = lens[:k].copy()
    seglen[-1] -= int(c[k - 1] - e)
    return u, v, seglen


def run_suite(args):
    """Every hot-path op at its BASELINE config's full size, inputs resident
    in HBM, CUDA-event timing (median of --steps after --warmup); one JSON
    line per op with its algorithmic bytes (gathered model) or FLOPs and the
    fraction of the measured peak."""
    import torch

    import mojodgl as dgl
    from mojodgl import ops

    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    hbm, tc_peak = float(peaks["hbm_gbs"]), float(peaks["bf16_tflops"])
    gen = torch.Generator("cuda")

    def t_ms(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    def emit(cfg, op, ms, nbytes, units=None, flops=None, extra=None):
        rec = {"suite": cfg, "op": op, "ms": round(ms, 4), "alg_bytes": nbytes,
               "GBps": round(nbytes / ms / 1e6, 1), "frac_hbm": round(nbytes / ms / 1e6 / hbm, 3)}
        if units:
            rec["Gedge_feat_s"] = round(units / ms / 1e6, 1)
        if flops:
            rec["TFLOPs"] = round(flops / ms / 1e9, 1)
        if extra:
            rec.update(extra)
        print(json.dumps(rec), flush=True)

    want = set(args.suite.split(",")) if args.suite != "all" else {"cfg2", "cfg3", "cfg4", "cfg5"}
    sc = args.suite_scale
    if "cfg2" in want:
        n = int(1_000_000 * sc)
        u, v = make_cfg2(n=n)
        e = u.size
        g = dgl.graph((u, v), num_nodes=n)
        g._device()
        gen.manual_seed(2)
        el = torch.randn((n, 8, 1), device="cuda", generator=gen)
        er = torch.randn((n, 8, 1), device="cuda", generator=gen)
        feat = torch.randn((n, 8, 64), device="cuda", generator=gen)
        s = ops.u_add_v(g, el, er)
        emit("cfg2", "gsddmm u_add_v (N,8,1)", t_ms(lambda: ops.u_add_v(g, el, er)),
             e * (2 * 32 + 8 + 32), units=e * 8)
        a = torch.nn.functional.leaky_relu(s, 0.2)
        emit("cfg2", "edge_softmax dst (E,8,1)", t_ms(lambda: ops.edge_softmax(g, a)),
             e * (32 + 32 + 4) + n * 8 + (n + 1) * 8, units=e * 8)
        att = ops.edge_softmax(g, a)
        emit("cfg2", "gspmm u_mul_e_sum (N,8,64)x(E,8,1)", t_ms(lambda: ops.u_mul_e_sum(g, feat, att)),
             e * (2048 + 32 + 4 + 4) + n * 2048 + (n + 1) * 8, units=e * 512,
             extra={"max_in_degree": int(np.bincount(v).max())})
        # the whole attention step fused (u_add_v, leaky_relu, edge_softmax,
        # u_mul_e_sum): feature row, el by source and source id per edge, er
        # and the output row per node
        unfused = {"chain": "u_add_v + leaky_relu + edge_softmax + u_mul_e_sum",
                   "chain_ms": t_ms(lambda: ops.u_mul_e_sum(g, feat, ops.edge_softmax(
                       g, torch.nn.functional.leaky_relu(ops.u_add_v(g, el, er), 0.2))))}
        emit("cfg2", "gat_aggregate fused (N,8,64)", t_ms(lambda: ops.gat_aggregate(g, feat, el, er)),
             e * (2048 + 32 + 4) + n * (2048 + 32) + (n + 1) * 8, units=e * 512, extra=unfused)
        del g, el, er, feat, s, a, att
        torch.cuda.empty_cache()
    if "cfg3" in want:
        c = CFG3
        u, v, h = make_cfg3(**c)
        n, e, d = c["num_nodes"], c["num_edges"], c["dim"]
        g = dgl.graph((u, v), num_nodes=n)
        g._device()
        hd = torch.from_numpy(h).cuda()
        for red in ("sum", "mean", "max"):
            emit("cfg3", "gspmm copy_u_" + red, t_ms(lambda: ops.gspmm(g, "copy_lhs", red, hd, None)),
                 algorithmic_bytes(n, e, d), units=e * d)
        emit("cfg3", "gspmm copy_u_max + arg_u (int64)",
             t_ms(lambda: ops.spmm._gspmm(g, "copy_lhs", "max", hd, None)),
             algorithmic_bytes(n, e, d, arg=True), units=e * d)
        gen.manual_seed(3)
        ef = torch.empty((e, d), device="cuda").uniform_(-1, 1, generator=gen)
        emit("cfg3", "gspmm u_mul_e_sum (E,128) edge feature", t_ms(lambda: ops.u_mul_e_sum(g, hd, ef)),
             algorithmic_bytes(n, e, d) + e * d * 4 + e * 4, units=e * d)
        del g, hd, ef
        torch.cuda.empty_cache()
    if "cfg4" in want:
        rng = np.random.default_rng(4)
        n, r, d = int(2_000_000 * sc), 64, 256
        gen.manual_seed(4)
        a = torch.empty((n, d), device="cuda").normal_(0, 0.05, generator=gen)
        b = torch.empty((r, d, d), device="cuda").normal_(0, 0.05, generator=gen)
        seglen = rng.multinomial(n, rng.dirichlet(0.5 * np.ones(r)))
        idx = torch.from_numpy(rng.integers(0, r, n)).cuda()
        flops = 2 * n * d * d
        for dt, name in ((torch.float32, "fp32 (TF32)"), (torch.bfloat16, "bf16")):
            aa, bb = a.to(dt), b.to(dt)
            el = 4 if dt == torch.float32 else 2
            emit("cfg4", "segment_mm " + name, t_ms(lambda: ops.segment_mm(aa, bb, seglen)),
                 n * d * el * 2 + r * d * d * el, flops=flops,
                 extra={"frac_tensor": None})
            emit("cfg4", "gather_mm " + name, t_ms(lambda: ops.gather_mm(aa, bb, idx_b=idx)),
                 n * d * el * 2 + r * d * d * el + n * 8, flops=flops)
        del a, b, aa, bb, idx
        torch.cuda.empty_cache()
    if "cfg5" in want:
        u, v, seglen = make_cfg5(n=int(5_000_000 * sc), e=int(50_000_000 * sc))
        n, e = int(5_000_000 * sc), u.size
        g = dgl.graph((u, v), num_nodes=n)
        g._device()
        gen.manual_seed(5)
        U = torch.randn((n, 256), device="cuda", generator=gen)
        V = torch.randn((n, 256), device="cuda", generator=gen)
        emit("cfg5", "gsddmm u_dot_v (N,256)", t_ms(lambda: ops.u_dot_v(g, U, V)),
             e * (2 * 1024 + 8 + 4), units=e * 256)
        del U, V, g
        torch.cuda.empty_cache()
        val = torch.randn((e, 64), device="cuda", generator=gen)
        sl = torch.from_numpy(seglen).cuda()
        ns = seglen.size
        emit("cfg5", "segment_softmax (E,64)", t_ms(lambda: ops.segment_softmax(sl, val)),
             2 * e * 256 + (ns + 1) * 8, units=e * 64, extra={"segments": ns})
        for red in ("sum", "max"):
            emit("cfg5", "segment_reduce " + red + " (E,64)",
                 t_ms(lambda: ops.segment_reduce(sl, val, red)),
                 e * 256 + ns * 256 + (ns + 1) * 8, units=e * 64)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the other ops of the config")
    ap.add_argument("--cols", type=int, default=0,
                    help="column groups of the N>1 rank grid (0: the default for N)")
    ap.add_argument("--nccl-normal-priority", action="store_true",
                    help="NCCL on normal-priority streams (default: high priority)")
    ap.add_argument("--halo", default="peer", choices=["peer", "allgather"],
                    help="N>1 halo exchange: copy-engine pulls from the peers' memory, or sliced "
                         "NCCL all-gathers")
    ap.add_argument("--halo-slices", type=int, default=HALO_SLICES,
                    help="row slices of each owner block in the all-gather halo")
    ap.add_argument("--suite", default="",
                    help="time every op of the named configs (cfg2,cfg3,cfg4,cfg5 or all) instead")
    ap.add_argument("--suite-scale", type=float, default=1.0,
                    help="scale configs 2 and 5 (nodes and edges) and config 4 (rows) in --suite "
                         "(profiling cases)")
    ap.add_argument("--scale", type=float, default=1.0,
                    help="scale the edge count (a smaller case for profiling; nodes unchanged)")
    ap.add_argument("--dim", type=int, default=0,
                    help="feature columns (0: the config's 128; a narrower case for profiling, "
                         "e.g. one rank's column block)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.suite:
        return run_suite(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

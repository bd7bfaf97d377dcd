"""Benchmark of the sparse-einsum hot path (one JSON line on rank 0).

Workload ("C2"): A = 65536^2 element COO with
4,294,967 unique entries (Zipf s=1.1 rows, uniform columns, N(0,1)), B =
dense 65536x256 N(0,1), tile 32, ``ij,jk->ik``. One step = one pass of the
hot path over it: COO->tile-COO tiling of A, dense->tile-COO of B, the
coordinate join, output grouping and the fused tile-GEMM + segment-sum
(``execute_sparse``). Metric: useful TFLOP/s = joined tile pairs x 2*32^3
per second (joined tile-pairs/s is reported beside it).

* ``value``: device-resident inputs, CUDA events around exactly K steps,
  max over ranks. Inputs (8 GB of A tiles written and read per step) are far
  larger than the 126 MB L2, so no flush is needed between steps.
* ``e2e``: the same step through the public API with host buffers: pinned
  host -> device copies of the COO arrays and B, and the result tiles copied
  back, all inside the timed region; the copies run on one stream per
  direction, so step k+1's inputs and step k-1's result move while step k
  computes (double-buffered device inputs and pinned results).
* ``--gpus N`` (torchrun, one rank per GPU): weak scaling, every rank runs its
  own C2 instance (seed = rank); the path needs no collective.
* ``--impl reference``: the CPU oracle (numpy port of the reference's path)
  on a bounded row-slice sample of the same workload, all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TILE = 32
FLOPS_PER_PAIR = 2 * TILE ** 3
# DRAM bytes (read + write) of the tile GEMM per joined pair, from the ncu
# capture of the 1/4-scale C2 case (one key block, 923,064 pairs); the lhs
# tiles dominate and are read once, so the traffic grows with the pairs.
TRAFFIC_PER_PAIR = 569.3
TRAFFIC_SOURCE = "ncu dram bytes of tc_strip_kernel at C2 scale 1/4, scaled by pairs (profiles/tc_strip_kernel_c2_scale4.md)"


def _env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms from before the
    warm-up to after the timed regions; the summary keeps the samples whose
    timestamps fall inside a timed region (``window_start``/``window_end``),
    or, for a region shorter than the sampling period, the nearest one."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.windows = []
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_bench_{gpu_index}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def window_start(self):
        self.windows.append([time.time(), None])

    def window_end(self):
        self.windows[-1][1] = time.time()

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        import datetime
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                t = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((t, float(parts[2]), float(parts[3]),
                             {n for n, v in zip(names, parts[6:10]) if v.lower() == "active"}))
            except ValueError:
                continue
        wins = [(a, b) for a, b in self.windows if b is not None]
        inside = [r for r in rows if any(a - 0.05 <= r[0] <= b + 0.05 for a, b in wins)]
        nearest = False
        if not inside and rows and wins:
            inside = [min(rows, key=lambda r: min(abs(r[0] - (a + b) / 2) for a, b in wins))]
            nearest = True
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        out = {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
               "reasons": sorted(set().union(*[r[3] for r in inside])), "samples": len(inside)}
        if nearest:
            out["nearest_sample"] = True
        return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    import einjax_b200 as E
    from einjax_b200 import _lib
    from einjax_b200 import sparse_dispatch as SD
    from einjax_b200 import workloads as W

    rank, world, local = _env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()

    t0 = time.time()
    w = W.c2_spmm(seed=args.seed + rank, scale=args.scale)
    gen_s = time.time() - t0
    shape = w.lhs.shape
    idx_h = torch.from_numpy(w.lhs.indices).pin_memory()
    val_h = torch.from_numpy(w.lhs.values).pin_memory()
    b_h = torch.from_numpy(w.rhs).pin_memory()
    idx_d, val_d, b_d = idx_h.to(dev), val_h.to(dev), b_h.to(dev)
    jk, ks, ak = w.join_keys, w.kernel_string, w.agg_keys
    ev = {}

    def step(idx, val, b, timing=False):
        A = E.tile_coo(idx, val, shape, (TILE, TILE))
        B = E.tile_dense(b, (TILE, TILE))
        plan = SD.plan_pairs(A, B, jk, ak)
        if timing:
            ev.setdefault("g", []).append(torch.cuda.Event(enable_timing=True))
            ev["g"][-1].record()
        vals = SD.tile_einsum(ks, A.values, B.values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                              precision=args.precision, seg_strip=plan.seg_strip, pair_key=plan.seg_key,
                              key_extent=plan.key_extent)
        if timing:
            ev.setdefault("h", []).append(torch.cuda.Event(enable_timing=True))
            ev["h"][-1].record()
        return A, B, plan, vals

    clk = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        A, B, plan, vals = step(idx_d, val_d, b_d)
    torch.cuda.synchronize()
    P = plan.num_pairs
    O = plan.num_segments
    T_A = A.num_tuples
    del A, B, plan, vals

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timing
    ev.clear()
    barrier()
    torch.cuda.synchronize()
    n0 = _lib.lib().es_launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.window_start()
    s.record()
    for _ in range(args.steps):
        A, B, plan, vals = step(idx_d, val_d, b_d, timing=True)
    e.record()
    torch.cuda.synchronize()
    clk.window_end()
    barrier()
    launches = _lib.lib().es_launch_count() - n0
    ms = s.elapsed_time(e)
    gemm_ms = [a.elapsed_time(b) for a, b in zip(ev["g"], ev["h"])]
    del A, B, plan, vals

    # ---- end to end through the public API with host buffers: every step
    # copies its inputs from pinned host memory and its result back, inside
    # the timed region. The copies run on their own streams (one per
    # direction) so that step k+1's inputs and step k-1's result move while
    # step k computes; input and result buffers are double-buffered.
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    hosts = (idx_h, val_h, b_h)
    slots = [tuple(torch.empty(h.shape, dtype=h.dtype, device=dev) for h in hosts) for _ in range(2)]

    def h2d(k, after):
        with torch.cuda.stream(s_in):
            if after is not None:
                s_in.wait_event(after)
            for d, h in zip(slots[k % 2], hosts):
                d.copy_(h, non_blocking=True)
            ev_h = torch.cuda.Event()
            ev_h.record(s_in)
        return ev_h

    def compute(k):
        idx, val, b = slots[k % 2]
        A = E.SparseTensor("A", (idx, val, shape)).to_relation((TILE, TILE))
        B = E.SparseTensor("B", b).to_relation((TILE, TILE))
        return E.execute_sparse(A, B, jk, ks, ak, precision=args.precision)

    def e2e_run(steps, outs, start):
        ev_in, ev_done = [None, None], [None, None]
        ev_in[0] = h2d(0, start)
        for k in range(steps):
            if k + 1 < steps:
                ev_in[(k + 1) % 2] = h2d(k + 1, ev_done[(k + 1) % 2] or start)
            comp.wait_event(ev_in[k % 2])
            res = compute(k)
            done = torch.cuda.Event()
            done.record(comp)
            ev_done[k % 2] = done
            if outs[k % 2] is None:
                outs[k % 2] = (torch.empty(res.values.shape, dtype=res.values.dtype, pin_memory=True),
                               torch.empty(res.coords.shape, dtype=res.coords.dtype, pin_memory=True))
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                outs[k % 2][0].copy_(res.values, non_blocking=True)
                outs[k % 2][1].copy_(res.coords, non_blocking=True)
                res.values.record_stream(s_out)
                res.coords.record_stream(s_out)
        comp.wait_stream(s_out)
        return outs

    outs = e2e_run(2, [None, None], None)  # untimed: allocates the pinned result buffers
    torch.cuda.synchronize()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.window_start()
    s2.record()
    outs = e2e_run(args.steps, outs, s2)
    e2.record()
    torch.cuda.synchronize()
    clk.window_end()
    clk.__exit__(None, None, None)
    barrier()
    e2e_ms = s2.elapsed_time(e2)
    out_h, oc_h = outs[0]
    h2d_bytes = idx_h.numel() * 4 + val_h.numel() * 4 + b_h.numel() * 4
    d2h_bytes = out_h.numel() * out_h.element_size() + oc_h.numel() * 4
    del slots

    # ---- per-phase split of one device-resident step (untimed for the metric)
    phases = {}
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    evs[0].record()
    A = E.tile_coo(idx_d, val_d, shape, (TILE, TILE))
    evs[1].record()
    B = E.tile_dense(b_d, (TILE, TILE))
    evs[2].record()
    plan = SD.plan_pairs(A, B, jk, ak)
    evs[3].record()
    SD.tile_einsum(ks, A.values, B.values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets, precision=args.precision,
                   seg_strip=plan.seg_strip, pair_key=plan.seg_key, key_extent=plan.key_extent)
    evs[4].record()
    torch.cuda.synchronize()
    for name, i in (("tile_coo_A", 0), ("tile_dense_B", 1), ("join_and_group", 2), ("tile_gemm", 3)):
        phases[name] = round(evs[i].elapsed_time(evs[i + 1]), 3)
    del A, B, plan

    tot = torch.tensor([ms, e2e_ms, float(P), float(P * FLOPS_PER_PAIR)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = tot[:2].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = tot[2:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms, e2e_ms = float(mx[0]), float(mx[1])
        P_all, flops_all = float(sm[0]), float(sm[1])
    else:
        P_all, flops_all = float(P), float(P * FLOPS_PER_PAIR)

    if rank == 0:
        hbm, bf16, src = _peaks()
        g_ms = statistics.mean(gemm_ms)
        # dominant kernel: the fused tile GEMM + segment-sum (one es_tile_einsum
        # call per step). Algorithmic FLOPs = P * 2*32^3 per call.
        achieved = P * FLOPS_PER_PAIR / (g_ms * 1e-3) / 1e12
        bound = "tensor"
        peak = bf16
        line = {
            "metric": "useful TFLOP/s (sparse einsum, C2 element-sparse SpMM)",
            "value": round(flops_all * args.steps / (ms * 1e-3) / 1e12, 3),
            "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded C2 generator, seed=rank)",
            "config": {"workload": "C2 ij,jk->ik: A 65536^2 COO 4,294,967 nnz Zipf(1.1) rows, B dense 65536x256, "
                                   "tile 32" + (f" (scale 1/{args.scale})" if args.scale != 1 else ""),
                       "global_batch": world, "pairs_per_rank": P, "tiles_A": T_A, "out_tiles": O,
                       "l2": "inputs >> L2 (8 GB of A tiles per step), no flush",
                       "parallelism": f"independent instance per rank x{world}", "precision": args.precision},
            "pairs_per_s": round(P_all * args.steps / (ms * 1e-3), 1),
            "e2e": {"value": round(flops_all * args.steps / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms / args.steps, 3),
                    "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": int(d2h_bytes),
                    "copies": "one stream per direction, overlapping the neighbouring steps' compute"},
            "roofline": {"kernel": "einsum (fused tile GEMM + segment-sum)", "bound": bound,
                         "achieved": round(achieved, 3), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": int(TRAFFIC_PER_PAIR * P),
                         "traffic_source": TRAFFIC_SOURCE,
                         "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
                         # fp32 runs as 3 TF32 MMAs per product at half the bf16 rate
                         "fp32_peak": round(peak / 6, 1),
                         "frac_fp32_peak": round(achieved / (peak / 6), 4),
                         "kernel_ms": round(g_ms, 3)},
            "gpu_launches": int(launches),
            "phases_ms": phases,
            "clocks": clk.summary(),
            "gen_s": round(gen_s, 1),
        }
        if world == 1:
            line["hbm_kernels"] = hbm_kernels(idx_d, val_d, b_d, shape, jk, ak, hbm)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, w)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _marks_ms(marks):
    """Launch time of one call from its plan0/plan1/fill0/fill1 marks (the
    host read of the counts between plan and fill is left out), or from its
    coalesce0/coalesce1 marks."""
    d = dict(marks)
    if "coalesce0" in d:
        return d["coalesce0"].elapsed_time(d["coalesce1"])
    ms = d["plan0"].elapsed_time(d["plan1"])
    if "fill0" in d:
        ms += d["fill0"].elapsed_time(d["fill1"])
    return ms


def hbm_kernels(idx_d, val_d, b_d, shape, jk, ak, hbm, reps=3):
    """HBM rooflines of the bandwidth-bound phases of the path on the C2
    inputs: COO->tile-COO tiling of A, coalescing A's COO (duplicates="sum"),
    join + output grouping, and the
    unfused segment_sum API on a sample of C2's (pair tile, output tile)
    rows. Each is timed by CUDA events around its own launches (median of
    ``reps``), against the algorithmic bytes of the phase."""
    import torch

    import einjax_b200 as E
    from einjax_b200 import sparse_dispatch as SD

    def entry(ms, alg, what):
        gbs = alg / (ms * 1e-3) / 1e9
        return {"kernel_ms": round(ms, 4), "alg_bytes": int(alg), "achieved_gbs": round(gbs, 1),
                "peak_gbs": hbm, "frac": round(gbs / hbm, 4), "bytes": what}

    out = {}
    t = []
    for _ in range(reps):
        m = []
        A = E.tile_coo(idx_d, val_d, shape, (TILE, TILE), marks=m)
        torch.cuda.synchronize()
        t.append(_marks_ms(m))
    nnz, T_A = int(val_d.numel()), A.num_tuples
    out["tile_coo"] = entry(statistics.median(t), nnz * (2 * 4 + 4) + T_A * (TILE * TILE * 4 + 2 * 4),
                            "nnz x 12 read + T_A x (4096 + 8) written")
    t = []
    for _ in range(reps):
        m = []
        ci, cv, _ = E.coalesce_coo(idx_d, val_d, shape, "sum", marks=m)
        torch.cuda.synchronize()
        t.append(_marks_ms(m))
    U = int(ci.shape[0])
    del ci, cv
    out["coo_coalesce"] = entry(statistics.median(t), nnz * (2 * 4 + 4) + U * (2 * 4 + 8),
                                "nnz x 12 read + U x (8 + 8) written (float64 sums); one 64-bit key sort between")
    B = E.tile_dense(b_d, (TILE, TILE))
    t = []
    for _ in range(reps):
        m = []
        plan = SD.plan_pairs(A, B, jk, ak, marks=m)
        torch.cuda.synchronize()
        t.append(_marks_ms(m))
    P, T_B = plan.num_pairs, B.num_tuples
    out["join_group"] = entry(statistics.median(t), 8 * (T_A + T_B) + 8 * P,
                              "8 x (T_A + T_B) coords read + 8 x P pair indices written")
    del A, B
    # segment_sum sample: the first output tiles of C2 up to 2^20 pair rows,
    # rows in a seeded random order, N(0,1) pair tiles
    so = plan.seg_offsets
    lim = torch.tensor([1 << 20], dtype=so.dtype, device=so.device)
    s_end = max(int(torch.searchsorted(so[1:], lim, right=True)[0]), 1)
    Ps = int(so[s_end])
    counts = so[1:s_end + 1] - so[:s_end]
    dev = so.device
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    oc = torch.repeat_interleave(plan.out_coords[:s_end], counts, dim=0)
    oc = oc[torch.randperm(Ps, device=dev, generator=g)].contiguous()
    vals = torch.randn((Ps, TILE, TILE), device=dev, generator=g)
    del plan
    t_all, t_red = [], []
    for _ in range(reps):
        m = []
        SD.segment_sum(vals, oc, marks=m)
        torch.cuda.synchronize()
        d = dict(m)
        t_all.append(_marks_ms(m))
        t_red.append(d["fill0"].elapsed_time(d["fill1"]))
    alg = (Ps + s_end) * TILE * TILE * 4
    seg = entry(statistics.median(t_red), alg, "P_s x 4096 read + O_s x 4096 written (the reduction launches)")
    seg["with_grouping"] = entry(statistics.median(t_all), alg + Ps * 8,
                                 "as above + 8 x P_s coords read; grouping (radix sort of the coordinates) included")
    seg["sample"] = f"{Ps} pair tiles into {s_end} output tiles (C2 segment sizes), fp32 32x32"
    out["segment_sum"] = seg
    del vals, oc
    return out


def cpu_baseline(args, w=None, budget_s=15.0):
    """Oracle (numpy port of the reference path) on row-slices of the C2
    workload, growing the slice until ~budget_s of CPU time."""
    import oracle as O
    from einjax_b200 import workloads as W
    if w is None:
        w = W.c2_spmm(seed=args.seed, scale=args.scale)
    n = w.lhs.shape[0]
    B = O.relation_from_dense(w.rhs.astype(np.float64), (TILE, TILE))
    frac = 1 / 1024
    best = None
    while True:
        rows = max(TILE, int(n * frac) // TILE * TILE)
        keep = w.lhs.indices[:, 0] < rows
        t0 = time.perf_counter()
        A = O.to_relation(w.lhs.indices[keep], w.lhs.values[keep].astype(np.float64), (rows, n), (TILE, TILE))
        res = O.execute_sparse(A, B, w.join_keys, w.kernel_string, w.agg_keys, compute_dtype="f32")
        dt = time.perf_counter() - t0
        li, _ = O.coordinate_join(A.coords, B.coords, w.join_keys)
        P = len(li)
        best = {"value": round(P * FLOPS_PER_PAIR / dt / 1e12, 6), "unit": "TFLOP/s",
                "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)), "kind": "port",
                "sample": f"first {rows} of {n} rows of A ({keep.sum()} nnz, {P} pairs), B full; "
                          f"to_relation+join+einsum+segment_sum in {dt:.2f}s",
                "pairs_per_s": round(P / dt, 1)}
        if dt > budget_s / 4 or frac >= 1 / 8:
            break
        frac *= 4
    return best


def run_reference(args):
    rank, world, _ = _env_rank()
    if rank != 0:
        return
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    from einjax_b200 import workloads as W
    w = W.c2_spmm(seed=args.seed, scale=args.scale)
    vals = []
    for _ in range(max(0, args.warmup)):
        cpu_baseline(args, w, budget_s=4.0)
    for _ in range(args.steps):
        vals.append(cpu_baseline(args, w, budget_s=8.0))
    v = statistics.median(x["value"] for x in vals)
    cb = dict(vals[-1])
    cb["value"] = v
    line = {"metric": "useful TFLOP/s (sparse einsum, C2 element-sparse SpMM)", "value": v, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded C2 generator)",
            "config": {"workload": "C2 ij,jk->ik: A 65536^2 COO 4,294,967 nnz Zipf(1.1) rows, B dense 65536x256, "
                                   "tile 32", "sample": cb["sample"]},
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_stats(args):
    """Sparsity statistics of every tiling scheme (planner input, tensor/stats.py)
    on C2's COO: A 65536^2 with 4,294,967 entries, all 17 x 17 = 289 factor
    tile shapes. One step = T(U) and V(l, U) of all schemes, device-resident
    COO. The reference's own per-scheme np.unique is timed beside it on a
    sample of schemes (cpu_baseline, extrapolated per scheme)."""
    import torch

    import einjax_b200 as E
    import oracle as O
    from einjax_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = W.c2_spmm(seed=args.seed, scale=args.scale)
    shape = w.lhs.shape
    idx = torch.from_numpy(w.lhs.indices).to(dev)
    val = torch.from_numpy(w.lhs.values).to(dev)
    ts = E.factor_tile_shapes(shape)
    for _ in range(args.warmup):
        got = E.compute_sparsity_stats_coo(idx, val, shape, ts, device=dev)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        got = E.compute_sparsity_stats_coo(idx, val, shape, ts, device=dev)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    nnz = int(val.numel())
    # check a sample of schemes against the oracle (integers: exact)
    sample = [ts[0], ts[len(ts) // 3], ts[len(ts) // 2], ts[-1]]
    t0 = time.time()
    ref = O.compute_sparsity_stats_coo(w.lhs.indices, w.lhs.values, shape, sample)
    cpu_s = (time.time() - t0) / len(sample)
    assert all(got[t] == ref[t] for t in sample), "sparsity statistics differ from the oracle"
    line = {
        "metric": "sparsity statistics: tiling schemes per second (C2 COO, all factor tile shapes)",
        "value": round(len(ts) / (ms * 1e-3), 1), "unit": "schemes/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic (seeded C2 generator)",
        "config": {"workload": f"STATS: A {shape[0]}x{shape[1]} COO {nnz} entries, {len(ts)} tile shapes",
                   "l2": "device-resident COO (51 MB) is re-read once per batch of schemes"},
        "entries_x_schemes_per_s": round(nnz * len(ts) / (ms * 1e-3), 1),
        "cpu_baseline": {"value": round(1.0 / cpu_s, 3), "unit": "schemes/s", "cores": 1, "kind": "port",
                         "sample": f"np.unique over {nnz} entries for {len(sample)} of the {len(ts)} schemes, "
                                   f"{cpu_s:.2f} s per scheme"},
    }
    print(json.dumps(line), flush=True)


def run_config(args):
    """The other BASELINE configurations on one GPU, for the results table
    (the headline line is C2, ``run_ours``). One step = the sparse path on
    device-resident inputs: C1/C3 ``execute_sparse`` of two tile relations;
    C4 the plan (A B) C through ``execute_sparse_plan`` (intermediate kept
    on the GPU), forward and the gradients of all three operands (loss = sum
    of the output); C5 COO -> tiles of X
    and W, then ``execute_sparse``."""
    import torch

    import einjax_b200 as E
    from einjax_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = args.workload
    t0 = time.time()
    if wl == "C4":
        w = W.c4_chain(seed=args.seed, scale=args.scale)
        c4_plan = E.plan_from_path("ij,jk,kl->il", [(0, 1), (0, 1)])  # (A B) C
        t = w["tile"]
        ops = [E.SparseTensorRelation.from_arrays(w[k].coords, w[k].values, w[k].shape, w[k].tile_shape,
                                                  device=dev, dtype=torch.float32) for k in ("A", "B", "C")]
        desc = (f"C4 ij,jk,kl->il (A B) C: 3 x {ops[0].shape[0]}^2 fp32, {t[0]}^2 tiles at 2%/5%/2% "
                f"({', '.join(str(o.num_tuples) for o in ops)} tiles), forward + gradients of A, B, C")
        dtype_s = "f32"
    elif wl in ("C1", "C3"):
        w = W.c1_block_sparse(seed=args.seed, scale=args.scale) if wl == "C1" else \
            W.c3_batched_bf16(seed=args.seed, scale=args.scale)
        tdt = torch.float32 if wl == "C1" else torch.bfloat16
        lhs = E.SparseTensorRelation.from_arrays(w.lhs.coords, w.lhs.values, w.lhs.shape, w.lhs.tile_shape,
                                                 device=dev, dtype=tdt)
        rhs = E.SparseTensorRelation.from_arrays(w.rhs.coords, w.rhs.values, w.rhs.shape, w.rhs.tile_shape,
                                                 device=dev, dtype=tdt)
        desc = (f"{wl} {w.kernel_string}: lhs {w.lhs.shape} {lhs.num_tuples} tiles of {w.lhs_tile}, "
                f"rhs {w.rhs.shape} {rhs.num_tuples} tiles of {w.rhs_tile}, {'fp32' if wl == 'C1' else 'bf16'}")
        dtype_s = "f32" if wl == "C1" else "bf16"
    else:  # C5
        w = W.c5_order3(seed=args.seed, scale=args.scale)
        idx = torch.from_numpy(w.lhs.indices).to(dev)
        val = torch.from_numpy(w.lhs.values).to(dev)
        wd = torch.from_numpy(w.rhs).to(dev)
        desc = (f"C5 ijk,kl->ijl: X {w.lhs.shape} COO {len(w.lhs.values)} nnz Zipf(1.2), W {tuple(w.rhs.shape)} "
                f"dense, tiles 16")
        dtype_s = "f32"
    gen_s = time.time() - t0

    def step():
        if wl == "C4":
            rels = [E.SparseTensorRelation(o.coords, o.values.detach().requires_grad_(True), o.shape,
                                           o.tile_shape) for o in ops]
            D = E.execute_sparse_plan(c4_plan, rels, differentiable=True)
            D.values.sum().backward()
            return D, None
        if wl in ("C1", "C3"):
            return E.execute_sparse(lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys), None
        X = E.tile_coo(idx, val, w.lhs.shape, w.lhs_tile)
        Wt = E.tile_dense(wd, w.rhs_tile)
        return E.execute_sparse(X, Wt, w.join_keys, w.kernel_string, w.agg_keys), X

    # useful flops of one step: joined pairs x flops per tile pair
    from einjax_b200 import sparse_dispatch as SD
    def pairs(lr, rr, jk, ak):
        return SD.plan_pairs(lr, rr, jk, ak).num_pairs
    for _ in range(args.warmup):
        out, aux = step()
    torch.cuda.synchronize()
    if wl == "C4":
        AB = E.execute_sparse(ops[0], ops[1], [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
        P1 = pairs(ops[0], ops[1], [(1, 0)], [(0, 0), (1, 1)])
        P2 = pairs(AB, ops[2], [(1, 0)], [(0, 0), (1, 1)])
        del AB
        flops = 3 * (P1 + P2) * 2 * t[0] ** 3  # forward + two backward products per pair
        P = P1 + P2
    elif wl in ("C1", "C3"):
        P = pairs(lhs, rhs, w.join_keys, w.agg_keys)
        te = int(np.prod(w.lhs_tile)) * w.rhs_tile[-1]
        flops = P * 2 * te
    else:
        P = pairs(aux, E.tile_dense(wd, w.rhs_tile), w.join_keys, w.agg_keys)
        flops = P * 2 * 16 ** 4
    del out, aux
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(args.steps):
        out, aux = step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    hbm, bf16, src = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    peak = bf16 if dtype_s == "bf16" else bf16 / 6
    line = {"metric": f"useful TFLOP/s (sparse einsum, {wl})", "value": round(achieved, 3), "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_s,
            "data": f"synthetic (seeded {wl} generator)",
            "config": {"workload": desc + (f" (scale 1/{args.scale})" if args.scale != 1 else ""), "pairs": P,
                       "l2": "device-resident inputs; no flush"},
            "pairs_per_s": round(P / (ms * 1e-3), 1),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 3),
                         "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{src} bf16 dense" + (" / 6 (fp32 as 3 TF32 passes)" if dtype_s == "f32"
                                                                 else "")},
            "gen_s": round(gen_s, 1)}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scale", type=int, default=1, help="shrink C2 by this factor (testing only)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--precision", default="auto", choices=["auto", "exact", "tc"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="C2", choices=["C1", "C2", "C3", "C4", "C5", "STATS"],
                    help="C2 is the headline line; the others measure one GPU for the results table")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "STATS":
        run_stats(args)
    elif args.workload != "C2":
        run_config(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

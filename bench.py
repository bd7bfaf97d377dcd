"""Benchmark of the sparse-einsum hot path (one JSON line on rank 0).

Headline workload ("C2"): A = 65536^2 element COO
with 4,294,967 unique entries (Zipf s=1.1 rows, uniform columns, N(0,1)),
B = dense 65536x256 N(0,1), tile 32, ``ij,jk->ik``. One step = one pass of the
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
  direction and are enqueued while step k's tile GEMM runs (step k+1's
  inputs, step k-1's result), so they neither wait for nor delay the step's
  reads of counts (double-buffered device inputs and pinned results).
* ``--gpus N`` (torchrun, one rank per GPU): strong scaling of the one C2
  problem through output-strip sharding (``execute_sharded_sparse``): rank r
  takes a tile-aligned range of A's rows balanced by non-empty tiles
  (``balanced_row_ranges``), tiles, joins, groups and contracts only those
  against the replicated B; output strips are disjoint, so no collective
  touches the data path.
* ``parity``: after the timed loops every rank compares its output strips
  with scipy's float64 ``A[rows] @ B`` (all elements), and with a plain fp32
  SpMM for context.
* ``configs``: the other BASELINE configurations in the same line -- C1, C3,
  C4 (forward + gradients of all three operands) and C5 on one GPU at N=1;
  at N>1, C5 sharded over its contracted (k) tile range with the partial
  output tiles summed by an NCCL reduce-scatter, as BASELINE specifies, and
  (``C5_output``) over X's i rows with no collective, for comparison.
  Each entry: ms per step, useful TFLOP/s, roofline fractions, clocks and a
  parity sample against a float64 computation.
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
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TILE = 32
FLOPS_PER_PAIR = 2 * TILE ** 3
# DRAM bytes (read + write) of the tile GEMM per joined pair, from the ncu
# capture of the 1/4-scale C2 case (one key block, 923,064 pairs); the lhs
# tiles dominate and are read once, so the traffic grows with the pairs.
TRAFFIC_PER_PAIR = 571.9
TRAFFIC_SOURCE = "ncu dram__bytes_read+write of the tile GEMM at C2 scale 1/4 per pair, times this run's pairs"


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
    warm-up to after the timed regions (into a temporary file); a summary
    keeps the samples whose timestamps fall inside the chosen timed regions
    (``window_start``/``window_end``), or, for a region shorter than the
    sampling period, the nearest one."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.windows = []
        fd, self.path = tempfile.mkstemp(prefix=f"einsparse_clocks_{gpu_index}_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def window_start(self):
        self.windows.append([time.time(), None])
        return len(self.windows) - 1

    def window_end(self):
        self.windows[-1][1] = time.time()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()
            self.f.close()
            self.proc = None

    def __exit__(self, *a):
        self.stop()
        try:
            os.unlink(self.path)
        except OSError:
            pass

    def summary(self, which=None):
        if not os.path.exists(self.path):
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
        wins = [w for i, w in enumerate(self.windows) if w[1] is not None and (which is None or i in which)]
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


# ------------------------------------------------------------------ parity
# float64 computations straight from the inputs (numpy / scipy), independent
# of the library and of the CPU oracle package.

def _err_stats(got, ref, mag, rtol):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    aref = np.abs(ref)
    nz = aref > 0
    return {
        "elements": int(ref.size),
        "max_abs_err": float(err.max()) if err.size else 0.0,
        "max_rel": float((err[nz] / aref[nz]).max()) if nz.any() else 0.0,
        "within_rtol": round(float((err <= rtol * aref).mean()), 7) if err.size else 1.0,
        "rel_fro": float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-300)),
        "bound_ok": bool(np.all(err <= rtol * (aref + mag))),
    }


def c2_parity(w, rows, coords, vals, rtol=1e-5):
    """This rank's output strips (rows [r0, r1) of the 65536 x 256 result)
    against scipy float64 ``A[rows] @ B``; a plain fp32 SpMM of the same
    inputs (scipy, float32 accumulation) is measured the same way beside it."""
    import scipy.sparse as sp
    r0, r1 = rows
    idx, val = w.lhs.indices, w.lhs.values
    keep = (idx[:, 0] >= r0) & (idx[:, 0] < r1)
    n, ncol = w.lhs.shape[1], w.rhs.shape[1]
    A = sp.csr_matrix((val[keep].astype(np.float64), (idx[keep, 0] - r0, idx[keep, 1])), shape=(r1 - r0, n))
    B = w.rhs.astype(np.float64)
    ref = A @ B
    mag = abs(A) @ np.abs(B)
    got = np.zeros((r1 - r0, ncol), dtype=np.float64)
    if len(coords):
        g4 = got.reshape((r1 - r0) // TILE, TILE, ncol // TILE, TILE)
        g4[coords[:, 0] - r0 // TILE, :, coords[:, 1], :] = vals
    out = _err_stats(got, ref, mag, rtol)
    A32 = sp.csr_matrix((val[keep].astype(np.float32), (idx[keep, 0] - r0, idx[keep, 1])), shape=(r1 - r0, n))
    f32 = _err_stats(A32 @ w.rhs.astype(np.float32), ref, mag, rtol)
    out["fp32_spmm_within_rtol"] = f32["within_rtol"]
    out["fp32_spmm_max_rel"] = f32["max_rel"]
    out["fp32_spmm_rel_fro"] = f32["rel_fro"]
    out["fp32_spmm_max_abs_err"] = f32["max_abs_err"]
    return out


def blocksparse_ref(lc, lv, rc, rv, nb, want):
    """float64 tiles of ``(batch..., i, j) x (batch..., j, k) -> (batch..., i, k)``
    at the output coordinates ``want`` (rows of (batch..., i, k)), summed over
    the contracted tile index from the host tile arrays; also the same sums
    of |a||b| (the magnitude scale of each element)."""
    from collections import defaultdict
    strips = defaultdict(list)
    for t, c in enumerate(map(tuple, lc)):
        strips[c[:-1]].append((c[-1], t))
    rmap = {c: t for t, c in enumerate(map(tuple, rc))}
    te = (lv.shape[-2], rv.shape[-1])
    ref = np.zeros((len(want), *te))
    mag = np.zeros((len(want), *te))
    for q, c in enumerate(map(tuple, want)):
        for j, li in strips.get(c[:-1], ()):
            ri = rmap.get(c[:nb] + (j, c[-1]))
            if ri is None:
                continue
            a = lv[li].reshape(te[0], -1).astype(np.float64)
            b = rv[ri].reshape(-1, te[1]).astype(np.float64)
            ref[q] += a @ b
            mag[q] += np.abs(a) @ np.abs(b)
    return ref, mag


def _sample_rows(n, k, seed=0):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(n, min(n, k), replace=False)) if n else np.zeros(0, dtype=np.int64)


# ------------------------------------------------------------------ C2 headline

def run_ours(args):
    import torch
    import torch.distributed as dist

    import einjax_b200 as E
    from einjax_b200 import _lib
    from einjax_b200 import distributed as D
    from einjax_b200 import sparse_dispatch as SD
    from einjax_b200 import workloads as W

    rank, world, local = _env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # the path runs on a high-priority stream: the tilings' deferred value
    # fills run on the library's fill stream (lowest priority), so the block
    # scheduler serves the pair grouping before the fill's remaining CTAs
    # and the two overlap
    torch.cuda.set_stream(torch.cuda.Stream(device=dev, priority=torch.cuda.Stream.priority_range()[1]))
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()

    def barrier():
        if world > 1:
            dist.barrier()

    t0 = time.time()
    w = W.c2_spmm(seed=args.seed, scale=args.scale)
    gen_s = time.time() - t0
    shape = w.lhs.shape
    # output-strip sharding: this rank's tile-aligned rows of A
    rows = D.balanced_row_ranges(w.lhs.indices, shape, (TILE, TILE), world)[rank] if world > 1 else (0, shape[0])
    keep = (w.lhs.indices[:, 0] >= rows[0]) & (w.lhs.indices[:, 0] < rows[1])
    idx_h = torch.from_numpy(np.ascontiguousarray(w.lhs.indices[keep])).pin_memory()
    val_h = torch.from_numpy(np.ascontiguousarray(w.lhs.values[keep])).pin_memory()
    b_h = torch.from_numpy(w.rhs).pin_memory()
    idx_d, val_d, b_d = idx_h.to(dev), val_h.to(dev), b_h.to(dev)
    jk, ks, ak = w.join_keys, w.kernel_string, w.agg_keys

    def step(idx, val, b, marks=None):
        E.sparse.mark(marks, "s0")
        A = E.tile_coo(idx, val, shape, (TILE, TILE))
        if marks is not None:
            A.values  # noqa: B018 -- the phase split times each tiling with its value fill
        E.sparse.mark(marks, "s1")
        B = E.tile_dense(b, (TILE, TILE))
        if marks is not None:
            B.values  # noqa: B018
        E.sparse.mark(marks, "s2")
        plan = SD.plan_pairs(A, B, jk, ak)
        E.sparse.mark(marks, "s3")
        # the tile fills launched by the plan's count read run on the fill
        # stream under the GEMM's pair grouping; the GEMM waits for them
        # right before its first launch that reads tile values
        lv, lr = A.values_and_ready()
        rv, rr = B.values_and_ready()
        vals = SD.tile_einsum(ks, lv, rv, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                              precision=args.precision, seg_strip=plan.seg_strip, pair_key=plan.seg_key,
                              key_extent=plan.key_extent, check="defer", ready=E.sparse.latest_ready(lr, rr))
        E.sparse.mark(marks, "s4")
        return A, B, plan, vals

    clk = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        A, B, plan, vals = step(idx_d, val_d, b_d)
    torch.cuda.synchronize()
    P = plan.num_pairs
    O = plan.num_segments
    T_A = A.num_tuples
    del A, B, plan, vals

    # ---- device-resident timing
    barrier()
    torch.cuda.synchronize()
    n0 = _lib.lib().es_launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w_main = clk.window_start()
    s.record()
    for _ in range(args.steps):
        A, B, plan, vals = step(idx_d, val_d, b_d)
    e.record()
    torch.cuda.synchronize()
    clk.window_end()
    barrier()
    launches = _lib.lib().es_launch_count() - n0
    ms = s.elapsed_time(e)
    del A, B, plan, vals

    # ---- end to end through the public API with host buffers: every step
    # copies its inputs from pinned host memory and its result back, inside
    # the timed region. The copies run on their own streams (one per
    # direction) so that step k+1's inputs and step k-1's result move while
    # step k computes; input and result buffers are double-buffered.
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # with N ranks each copies 1/N of B's rows from the host and NCCL
    # all-gathers the rest over NVLink inside the step, so no rank moves the
    # whole replicated operand across PCIe
    nb = b_h.shape[0] // world
    b_part_h = b_h[rank * nb:(rank + 1) * nb] if world > 1 else b_h
    hosts = (idx_h, val_h, b_part_h)
    slots = [tuple(torch.empty(h.shape, dtype=h.dtype, device=dev) for h in hosts) for _ in range(2)]
    # B's full rows, double-buffered: step k gathers into b_full[k % 2] on
    # its own stream while step k-1's deferred B fill may still read the other
    b_full = [torch.empty(b_h.shape, dtype=b_h.dtype, device=dev) for _ in range(2)] if world > 1 else None
    s_ag = torch.cuda.Stream(dev) if world > 1 else None

    def h2d(k, after, gemm=None):
        with torch.cuda.stream(s_in):
            if after is not None:
                s_in.wait_event(after)
            if gemm is not None:
                s_in.wait_event(gemm)
            for d, h in zip(slots[k % 2], hosts):
                d.copy_(h, non_blocking=True)
            ev_h = torch.cuda.Event()
            ev_h.record(s_in)
        return ev_h

    def compute(k, inputs_ready):
        idx, val, b = slots[k % 2]
        if world > 1:
            # the other ranks' rows of B come over NVLink on a stream of their
            # own as soon as this step's slice has landed, beside A's tiling,
            # which needs none of B
            bf = b_full[k % 2]
            s_ag.wait_event(inputs_ready)
            with torch.cuda.stream(s_ag):
                dist.all_gather_into_tensor(bf, b)
            gathered = torch.cuda.Event()
            gathered.record(s_ag)
        # the public device-tensor tilings (their counts resolve together at
        # the plan, their value fills overlap the GEMM's pair grouping)
        A = E.tile_coo(idx, val, shape, (TILE, TILE))
        if world > 1:
            comp.wait_event(gathered)
            b = bf
        B = E.tile_dense(b, (TILE, TILE))
        res = E.execute_sharded_sparse(A, B, jk, ks, ak, precision=args.precision, lhs_sharded=True,
                                       gather=False)
        # the event behind the step's tile fills: the tile GEMM starts when
        # it has passed, so copies issued behind it run under the GEMM
        ready = E.sparse.latest_ready(A.values_and_ready()[1], B.values_and_ready()[1])
        return res, (ready[1] if ready is not None else None)

    def d2h(k, res, done, outs, gemm=None):
        if outs[k % 2] is None:
            outs[k % 2] = (torch.empty(res.values.shape, dtype=res.values.dtype, pin_memory=True),
                           torch.empty(res.coords.shape, dtype=res.coords.dtype, pin_memory=True))
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            if gemm is not None:
                s_out.wait_event(gemm)
            outs[k % 2][0].copy_(res.values, non_blocking=True)
            outs[k % 2][1].copy_(res.coords, non_blocking=True)
            res.values.record_stream(s_out)
            res.coords.record_stream(s_out)

    def e2e_run(steps, outs, start):
        # The step reads counts back from the device before its tile GEMM and
        # none after it. The next step's inputs and the previous step's result
        # are copied while step k's GEMM runs: issued behind the event of step
        # k's tile fills, which the GEMM waits for, so they neither contend
        # with the fills and the pair grouping for HBM nor hold a count read
        # of the next step behind them on a copy engine.
        ev_in, ev_done = [None, None], [None, None]
        ev_in[0] = h2d(0, start)
        prev = None
        for k in range(steps):
            comp.wait_event(ev_in[k % 2])
            res, gemm = compute(k, ev_in[k % 2])
            done = torch.cuda.Event()
            done.record(comp)
            ev_done[k % 2] = done
            if k + 1 < steps:
                ev_in[(k + 1) % 2] = h2d(k + 1, ev_done[(k + 1) % 2] if k >= 1 else start, gemm)
            if prev is not None:
                d2h(k - 1, *prev, outs, gemm)
            prev = (res, done)
        if prev is not None:
            d2h(steps - 1, *prev, outs)
        comp.wait_stream(s_out)
        return outs

    outs = e2e_run(2, [None, None], None)  # untimed: allocates the pinned result buffers
    torch.cuda.synchronize()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w_e2e = clk.window_start()
    s2.record()
    outs = e2e_run(args.steps, outs, s2)
    e2.record()
    torch.cuda.synchronize()
    clk.window_end()
    barrier()
    e2e_ms = s2.elapsed_time(e2)
    out_h, oc_h = outs[0]
    h2d_bytes = idx_h.numel() * 4 + val_h.numel() * 4 + b_part_h.numel() * 4
    d2h_bytes = out_h.numel() * out_h.element_size() + oc_h.numel() * 4
    del slots

    E.check_device_errors()
    # ---- per-phase split of one device-resident step (untimed for the metric)
    m = []
    A, B, plan, vals = step(idx_d, val_d, b_d, marks=m)
    torch.cuda.synchronize()
    d = dict(m)
    phases = {name: round(d[a].elapsed_time(d[b]), 3) for name, a, b in
              (("tile_coo_A", "s0", "s1"), ("tile_dense_B", "s1", "s2"), ("join_and_group", "s2", "s3"),
               ("tile_gemm", "s3", "s4"))}
    # ---- the dominant kernel alone: the tile GEMM (everything es_tile_einsum
    # launches) on the step's ready operands, CUDA events on its stream
    gemm_ms = []
    for _ in range(3):
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        SD.tile_einsum(ks, A.values, B.values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                       precision=args.precision, seg_strip=plan.seg_strip, pair_key=plan.seg_key,
                       key_extent=plan.key_extent, check="defer")
        g1.record()
        torch.cuda.synchronize()
        gemm_ms.append(g0.elapsed_time(g1))
    # ---- parity of this rank's output strips (full, float64)
    par = c2_parity(w, rows, plan.out_coords.cpu().numpy(), vals.cpu().numpy())
    del A, B, plan, vals

    per_rank = torch.tensor([ms / args.steps, e2e_ms / args.steps, statistics.mean(gemm_ms),
                             *[phases[k] for k in ("tile_coo_A", "tile_dense_B", "join_and_group", "tile_gemm")],
                             float(P), float(T_A), float(O), par["max_rel"], par["max_abs_err"],
                             par["within_rtol"], 1.0 if par["bound_ok"] else 0.0, par["rel_fro"],
                             par["fp32_spmm_within_rtol"], float(launches), par["fp32_spmm_rel_fro"],
                             par["fp32_spmm_max_abs_err"]], dtype=torch.float64, device=dev)
    if world > 1:
        allr = [torch.zeros_like(per_rank) for _ in range(world)]
        dist.all_gather(allr, per_rank)
        table = torch.stack(allr).cpu().numpy()
    else:
        table = per_rank.cpu().numpy()[None, :]

    cfgs = {}
    if not args.no_configs:
        cfgs = measure_configs(args, dev, rank, world, clk, barrier)

    if rank == 0:
        hbm, bf16, src = _peaks()
        ms_step = float(table[:, 0].max())
        e2e_step = float(table[:, 1].max())
        slow = int(table[:, 0].argmax())
        P_all = float(table[:, 7].sum())
        flops_all = P_all * FLOPS_PER_PAIR
        g_ms = float(table[0, 2])
        # dominant kernel: the fused tile GEMM + segment-sum (one es_tile_einsum
        # call per step), on rank 0. Algorithmic FLOPs = P * 2*32^3 per call.
        achieved = P * FLOPS_PER_PAIR / (g_ms * 1e-3) / 1e12
        peak = bf16
        line = {
            "metric": "useful TFLOP/s (sparse einsum, C2 element-sparse SpMM)",
            "value": round(flops_all / (ms_step * 1e-3) / 1e12, 3),
            "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded C2 generator; one problem shared by all ranks)",
            "config": {"workload": "C2 ij,jk->ik: A 65536^2 COO 4,294,967 nnz Zipf(1.1) rows, B dense 65536x256, "
                                   "tile 32" + (f" (scale 1/{args.scale})" if args.scale != 1 else ""),
                       "global_batch": 1, "pairs": int(P_all), "tiles_A": int(table[:, 8].sum()),
                       "out_tiles": int(table[:, 9].sum()),
                       "l2": "inputs >> L2 (8 GB of A tiles per step), no flush",
                       "parallelism": (f"output-strip sharding x{world}: each rank tiles, joins and contracts a "
                                       "tile-row range of A balanced by non-empty tiles against the replicated B; "
                                       "no data-path collective") if world > 1 else "single GPU",
                       "precision": args.precision},
            "pairs_per_s": round(P_all / (ms_step * 1e-3), 1),
            "e2e": {"value": round(flops_all / (e2e_step * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_step, 3),
                    "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": int(d2h_bytes),
                    "copies": "one stream per direction, issued behind each step's tile fills so they run "
                              "under its tile GEMM (next inputs, previous result)" +
                              ("; each rank copies its A rows and 1/N of B's rows, B is all-gathered over "
                               "NVLink (NCCL) inside the step, on its own stream beside A's tiling"
                               if world > 1 else "")},
            "roofline": {"kernel": "einsum (fused tile GEMM + segment-sum)", "bound": "tensor",
                         "achieved": round(achieved, 3), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": int(TRAFFIC_PER_PAIR * P),
                         "traffic_source": TRAFFIC_SOURCE,
                         "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
                         # fp32 runs as 3 TF32 MMAs per product at half the bf16 rate
                         "fp32_peak": round(peak / 6, 1),
                         "frac_fp32_peak": round(achieved / (peak / 6), 4),
                         "kernel_ms": round(g_ms, 3)},
            "parity": {"reference": "scipy float64 A @ B, every output element" +
                                    (" (each rank its own strips)" if world > 1 else ""),
                       "rtol": 1e-5, "max_rel": float(table[:, 10].max()), "max_abs_err": float(table[:, 11].max()),
                       "within_rtol": float(table[:, 12].min()), "bound_ok": bool(table[:, 13].min() > 0),
                       "bound": "|got - ref| <= rtol * (|ref| + sum |a*b|)",
                       "rel_fro": float(table[:, 14].max()),
                       "fp32_spmm": {"what": "scipy float32 A @ B (row-order fp32 accumulation) against the same "
                                             "float64 reference", "within_rtol": float(table[:, 15].min()),
                                     "rel_fro": float(table[:, 17].max()),
                                     "max_abs_err": float(table[:, 18].max())}},
            "gpu_launches": int(table[0, 16]),
            "phases_ms": {k: float(table[slow, 3 + i]) for i, k in
                          enumerate(("tile_coo_A", "tile_dense_B", "join_and_group", "tile_gemm"))},
            "clocks": clk.summary([w_main, w_e2e]),
            "gen_s": round(gen_s, 1),
        }
        if world > 1:
            line["ranks"] = {"ms_per_step": [round(float(x), 3) for x in table[:, 0]],
                             "tile_gemm_ms": [round(float(x), 3) for x in table[:, 6]],
                             "pairs": [int(x) for x in table[:, 7]],
                             "slowest": slow,
                             "imbalance": round(float(table[:, 0].max() / table[:, 0].mean()), 3),
                             "limiting": "tile GEMM of the slowest rank (no collective on the data path)"}
        if world == 1 and not args.no_hbm:
            line["hbm_kernels"] = hbm_kernels(idx_d, val_d, b_d, shape, jk, ak, hbm)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, w)
        if cfgs:
            line["configs"] = cfgs
        print(json.dumps(line), flush=True)
    clk.__exit__(None, None, None)
    if world > 1:
        barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ other configs

def _timed_steps(step, steps, warmup, clk, barrier):
    import torch
    out = None
    for _ in range(warmup):
        out = step()
    torch.cuda.synchronize()
    del out
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    win = clk.window_start()
    s.record()
    for _ in range(steps):
        out = step()
    e.record()
    torch.cuda.synchronize()
    clk.window_end()
    barrier()
    return s.elapsed_time(e) / steps, out, win


def _roof(achieved, dtype_s, bf16, src):
    r = {"bound": "tensor", "achieved": round(achieved, 3), "unit": "TFLOP/s", "peak": bf16,
         "frac": round(achieved / bf16, 4), "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)"}
    if dtype_s == "f32":
        r["fp32_peak"] = round(bf16 / 6, 1)
        r["frac_fp32_peak"] = round(achieved / (bf16 / 6), 4)
    return r


def measure_configs(args, dev, rank, world, clk, barrier):
    """C1, C3, C4 and C5 (N=1) or sharded C5 (N>1); entries of ``configs``."""
    out = {}
    steps = max(3, min(args.steps, 10))
    warm = max(3, min(args.warmup, 3))
    names = ["C1", "C3", "C4", "C5"] if world == 1 else ["C5", "C5_output"]
    if args.configs:
        names = [n for n in names if n in args.configs.split(",")]
    for name in names:
        fn = {"C1": measure_c1, "C3": measure_c3, "C4": measure_c4, "C5": measure_c5,
              "C5_output": lambda *a: measure_c5(*a, shard="output")}[name]
        try:
            out[name] = fn(args, dev, rank, world, clk, barrier, steps, warm)
        except Exception as ex:  # a failed config must not hide the headline
            if world > 1:
                raise
            out[name] = {"error": f"{type(ex).__name__}: {ex}"[:300]}
        import torch
        torch.cuda.empty_cache()
    return out


def measure_c1(args, dev, rank, world, clk, barrier, steps, warm):
    import torch

    import einjax_b200 as E
    from einjax_b200 import sparse_dispatch as SD
    from einjax_b200 import workloads as W
    w = W.c1_block_sparse(seed=args.seed)
    lhs = E.SparseTensorRelation.from_arrays(w.lhs.coords, w.lhs.values, w.lhs.shape, w.lhs.tile_shape, device=dev)
    rhs = E.SparseTensorRelation.from_arrays(w.rhs.coords, w.rhs.values, w.rhs.shape, w.rhs.tile_shape, device=dev)
    ms, res, win = _timed_steps(lambda: E.execute_sparse(lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys),
                                steps, warm, clk, barrier)
    P = SD.plan_pairs(lhs, rhs, w.join_keys, w.agg_keys).num_pairs
    flops = P * 2 * 128 ** 3
    hbm, bf16, src = _peaks()
    c, v = res.to_numpy()
    ref, mag = blocksparse_ref(w.lhs.coords, w.lhs.values, w.rhs.coords, w.rhs.values, 0, c)
    return {"workload": "C1 ij,jk->ik 4096^2 fp32, 128^2 tiles at 10% (102 tiles per operand)",
            "ms_per_step": round(ms, 4), "value": round(flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "pairs": P, "roofline": _roof(flops / (ms * 1e-3) / 1e12, "f32", bf16, src),
            "clocks": clk.summary([win]),
            "parity": dict(_err_stats(v, ref, mag, 1e-5), reference="float64 per-tile products, every output tile")}


def measure_c3(args, dev, rank, world, clk, barrier, steps, warm):
    import torch

    import einjax_b200 as E
    from einjax_b200 import sparse_dispatch as SD
    from einjax_b200 import workloads as W
    w = W.c3_batched_bf16(seed=args.seed)
    kw = dict(device=dev, dtype=torch.bfloat16)
    lhs = E.SparseTensorRelation.from_arrays(w.lhs.coords, w.lhs.values, w.lhs.shape, w.lhs.tile_shape, **kw)
    rhs = E.SparseTensorRelation.from_arrays(w.rhs.coords, w.rhs.values, w.rhs.shape, w.rhs.tile_shape, **kw)
    ms, res, win = _timed_steps(lambda: E.execute_sparse(lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys),
                                steps, warm, clk, barrier)
    P = SD.plan_pairs(lhs, rhs, w.join_keys, w.agg_keys).num_pairs
    flops = P * 2 * 64 ** 3
    hbm, bf16, src = _peaks()
    c, v = res.to_numpy()
    pick = _sample_rows(len(c), 512)
    ref, mag = blocksparse_ref(w.lhs.coords, w.lhs.values, w.rhs.coords, w.rhs.values, 1, c[pick])
    return {"workload": "C3 bij,bjk->bik b=16 8192^2 bf16, 64^2 tiles at 5% (band + random)",
            "ms_per_step": round(ms, 4), "value": round(flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "pairs": P, "roofline": _roof(flops / (ms * 1e-3) / 1e12, "bf16", bf16, src),
            "clocks": clk.summary([win]),
            "parity": dict(_err_stats(v[pick].reshape(ref.shape), ref, mag, 2e-2),
                           reference=f"float64 per-tile products of the bf16 inputs, {len(pick)} random output tiles")}


def measure_c4(args, dev, rank, world, clk, barrier, steps, warm):
    import torch

    import einjax_b200 as E
    from einjax_b200 import sparse_dispatch as SD
    from einjax_b200 import workloads as W
    w = W.c4_chain(seed=args.seed)
    plan = E.plan_from_path("ij,jk,kl->il", [(0, 1), (0, 1)])  # (A B) C
    ops = [E.SparseTensorRelation.from_arrays(w[k].coords, w[k].values, w[k].shape, w[k].tile_shape, device=dev,
                                              dtype=torch.float32) for k in ("A", "B", "C")]

    def step():
        rels = [E.SparseTensorRelation(o.coords, o.values.detach().requires_grad_(True), o.shape, o.tile_shape)
                for o in ops]
        D = E.execute_sparse_plan(plan, rels, differentiable=True)
        D.values.sum().backward()
        return D
    ms, res, win = _timed_steps(step, steps, warm, clk, barrier)
    AB = E.execute_sparse(ops[0], ops[1], [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    P1 = SD.plan_pairs(ops[0], ops[1], [(1, 0)], [(0, 0), (1, 1)]).num_pairs
    P2 = SD.plan_pairs(AB, ops[2], [(1, 0)], [(0, 0), (1, 1)]).num_pairs
    flops = 3 * (P1 + P2) * 2 * 128 ** 3  # forward + two backward products per pair
    hbm, bf16, src = _peaks()
    # forward parity: (A B) C in float64 from the host tiles, sampled output tiles
    abc = AB.coords.cpu().numpy()
    ab_ref, ab_mag = blocksparse_ref(w["A"].coords, w["A"].values, w["B"].coords, w["B"].values, 0, abc)
    c, v = res.coords.cpu().numpy(), res.values.detach().float().cpu().numpy()
    pick = _sample_rows(len(c), 256)
    ref, _ = blocksparse_ref(abc, ab_ref, w["C"].coords, w["C"].values, 0, c[pick])
    mag, _ = blocksparse_ref(abc, ab_mag, w["C"].coords, np.abs(w["C"].values), 0, c[pick])
    return {"workload": "C4 ij,jk,kl->il (A B) C: 3 x 16384^2 fp32, 128^2 tiles at 2%/5%/2%, forward + "
                        "gradients of A, B, C (loss = sum of the output)",
            "ms_per_step": round(ms, 4), "value": round(flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "pairs": P1 + P2, "roofline": _roof(flops / (ms * 1e-3) / 1e12, "f32", bf16, src),
            "clocks": clk.summary([win]),
            "parity": dict(_err_stats(v[pick], ref, mag, 1e-5),
                           reference=f"float64 (A B) C from the host tiles, {len(pick)} random output tiles "
                                     "(forward; gradients are checked by the GPU tests)")}


def c5_sample_ref(idx, val, W, want_ij, tile=16):
    """float64 C5 output tiles ``Out[i, j, :] = sum_k X[i, j, k] W[k, :]`` for
    the (i_tile, j_tile) positions ``want_ij`` (rows of 2), from the element
    COO; shape (len(want_ij), 16, 16, n_out) and the |X||W| magnitudes."""
    key = (idx[:, 0].astype(np.int64) // tile) * 1_000_000 + idx[:, 1] // tile
    wk = want_ij[:, 0].astype(np.int64) * 1_000_000 + want_ij[:, 1]
    order = np.argsort(wk)
    pos = np.searchsorted(wk[order], key)
    pos = np.minimum(pos, len(wk) - 1)
    hit = wk[order][pos] == key
    q = order[pos[hit]]
    i, j, k = idx[hit, 0] % tile, idx[hit, 1] % tile, idx[hit, 2]
    x = val[hit].astype(np.float64)
    Wd = W.astype(np.float64)
    ref = np.zeros((len(want_ij), tile, tile, W.shape[1]))
    mag = np.zeros_like(ref)
    np.add.at(ref, (q, i, j), x[:, None] * Wd[k])
    np.add.at(mag, (q, i, j), np.abs(x)[:, None] * np.abs(Wd[k]))
    return ref, mag


def measure_c5(args, dev, rank, world, clk, barrier, steps, warm, shard="contracted"):
    """C5 ``ijk,kl->ijl`` at full size (X drawn on the GPU). N=1: one GPU.
    N>1, ``shard="contracted"`` (the BASELINE configuration): X's contracted
    k tile range split over the ranks (balanced by X tile count), each rank
    tiles and contracts its k slice, and the partial output tiles are summed
    by one NCCL reduce-scatter over the union of output coordinates
    (``execute_sharded_sparse(shard="contracted")``). ``shard="output"``, for
    comparison: X's i rows split (``balanced_row_ranges``), no collective."""
    import torch
    import torch.distributed as dist

    import einjax_b200 as E
    from einjax_b200 import distributed as D
    from einjax_b200 import sparse_dispatch as SD
    from einjax_b200 import workloads as W
    t0 = time.time()
    w = W.c5_order3_device(seed=args.seed, scale=args.c5_scale, device=dev)
    gen_s = time.time() - t0
    shape, lt, rt = w.lhs.shape, w.lhs_tile, w.rhs_tile
    idx, val, Wd = w.lhs.indices, w.lhs.values, w.rhs
    if world > 1 and shard == "output":
        i_np = idx[:, 0].cpu().numpy()
        r0, r1 = D.balanced_row_ranges(idx.cpu().numpy(), shape, lt, world)[rank]
        sel = (idx[:, 0] >= r0) & (idx[:, 0] < r1)
        li, lv = idx[sel].contiguous(), val[sel].contiguous()
        del sel, i_np
    elif world > 1:
        # k tile range of this rank, balanced by non-empty X tiles per k tile
        g = [s // t for s, t in zip(shape, lt)]
        tk = (idx[:, 0].long() // lt[0] * g[1] + idx[:, 1].long() // lt[1]) * g[2] + idx[:, 2].long() // lt[2]
        kt = torch.unique(tk) % g[2]
        counts = torch.bincount(kt, minlength=g[2]).cpu().numpy()
        k0, k1 = D.balanced_key_ranges(counts, world)[rank]
        sel = (idx[:, 2] >= k0 * lt[2]) & (idx[:, 2] < k1 * lt[2])
        li, lv = idx[sel].contiguous(), val[sel].contiguous()
        del tk, kt, sel
    else:
        li, lv = idx, val
    marks = []

    def step():
        X = E.tile_coo(li, lv, shape, lt)
        Wt = E.tile_dense(Wd, rt)
        if world > 1:
            del marks[:]
            return E.execute_sharded_sparse(X, Wt, w.join_keys, w.kernel_string, w.agg_keys, shard=shard,
                                            lhs_sharded=True, gather=False, timings=marks)
        return E.execute_sparse(X, Wt, w.join_keys, w.kernel_string, w.agg_keys)
    ms, res, win = _timed_steps(step, steps, warm, clk, barrier)
    coll_ms = dict(marks)["collective0"].elapsed_time(dict(marks)["collective1"]) if marks else 0.0
    X = E.tile_coo(li, lv, shape, lt)
    Wt = E.tile_dense(Wd, rt)
    plan = SD.plan_pairs(X, Wt, w.join_keys, w.agg_keys)
    P, T_X = plan.num_pairs, X.num_tuples
    xv, wv = X.values, Wt.values  # the tile fills end before the GEMM-only window
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    SD.tile_einsum(w.kernel_string, xv, wv, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                   seg_strip=plan.seg_strip, pair_key=plan.seg_key, key_extent=plan.key_extent)
    e.record()
    torch.cuda.synchronize()
    gemm_ms = s.elapsed_time(e)
    del X, Wt, plan
    # parity: random (i, j) tile positions of this rank's result, every l
    c, v = res.coords.cpu().numpy(), res.values.float().cpu().numpy()
    ij = np.unique(c[:, :2], axis=0)
    want = ij[_sample_rows(len(ij), 96, seed=rank)]
    ref, mag = c5_sample_ref(idx.cpu().numpy(), val.cpu().numpy(), Wd.cpu().numpy(), want)
    # the output tiles of the sampled positions this rank holds (a rank's
    # union chunk may start or end inside the l tiles of one (i, j))
    rowmap = {tuple(x): r for r, x in enumerate(c)}
    got_t, ref_t, mag_t = [], [], []
    for q, (a, b) in enumerate(want):
        for lt_ in range(ref.shape[-1] // rt[1]):
            r = rowmap.get((a, b, lt_))
            if r is not None:
                sl = slice(lt_ * rt[1], (lt_ + 1) * rt[1])
                got_t.append(v[r])
                ref_t.append(ref[q, :, :, sl])
                mag_t.append(mag[q, :, :, sl])
    st = _err_stats(np.stack(got_t), np.stack(ref_t), np.stack(mag_t), 1e-5)
    flops = P * 2 * 16 ** 4
    u_rows = int(res.coords.shape[0])
    vec = torch.tensor([ms, float(P), float(T_X), gemm_ms, coll_ms, st["max_rel"], st["within_rtol"],
                        1.0 if st["bound_ok"] else 0.0, float(u_rows)], dtype=torch.float64, device=dev)
    if world > 1:
        allr = [torch.zeros_like(vec) for _ in range(world)]
        dist.all_gather(allr, vec)
        tab = torch.stack(allr).cpu().numpy()
    else:
        tab = vec.cpu().numpy()[None, :]
    hbm, bf16, src = _peaks()
    ms_step = float(tab[:, 0].max())
    P_all = float(tab[:, 1].sum())
    flops_all = P_all * 2 * 16 ** 4
    tile_bytes = 16 * 16 * 16 * 4
    entry = {"workload": f"C5 ijk,kl->ijl: X {shape} COO {int(val.numel())} nnz Zipf(1.2) per mode (drawn on the "
                         f"GPU), W {tuple(Wd.shape)} dense, tiles 16" +
                         (f" (scale 1/{args.c5_scale})" if args.c5_scale != 1 else ""),
             "ms_per_step": round(ms_step, 3), "value": round(flops_all / (ms_step * 1e-3) / 1e12, 3),
             "unit": "TFLOP/s", "pairs": int(P_all), "tiles_X": int(tab[:, 2].sum()),
             "gen_s": round(gen_s, 1),
             "roofline": dict(_roof(P * 2 * 16 ** 4 / (gemm_ms * 1e-3) / 1e12, "f32", bf16, src),
                              kernel="einsum (fused tile GEMM + segment-sum), rank 0", kernel_ms=round(gemm_ms, 3),
                              lhs_gbs=round(T_X * tile_bytes / (gemm_ms * 1e-3) / 1e9, 1),
                              frac_hbm_lhs=round(T_X * tile_bytes / (gemm_ms * 1e-3) / 1e9 / hbm, 4)),
             "clocks": clk.summary([win]),
             "parity": {"reference": "float64 sum over X entries times W, random (i, j) output tile positions "
                                     "(all l), full contracted range", "rtol": 1e-5,
                        "max_rel": float(tab[:, 5].max()), "within_rtol": float(tab[:, 6].min()),
                        "bound_ok": bool(tab[:, 7].min() > 0),
                        "bound": "|got - ref| <= rtol * (|ref| + sum |x*w|)"}}
    if world > 1 and shard == "output":
        entry["parallelism"] = (f"output sharding x{world}: X's i rows split (balanced by X tiles), W replicated, "
                                "no collective (a comparison for the contracted split BASELINE specifies)")
        entry["scaling"] = "strong"
        entry["ranks"] = {"ms_per_step": [round(float(x), 3) for x in tab[:, 0]],
                          "tile_gemm_ms": [round(float(x), 3) for x in tab[:, 3]]}
    elif world > 1:
        U = int(tab[:, 8].sum())
        per_rank_send = (world - 1) * ((U + world - 1) // world) * tile_bytes
        entry["parallelism"] = (f"contracted k tile range split x{world} (balanced by X tiles); partial output tiles "
                                "written by the tile GEMM in union order, summed by one NCCL reduce-scatter")
        entry["scaling"] = "strong"
        entry["ranks"] = {"ms_per_step": [round(float(x), 3) for x in tab[:, 0]],
                          "tile_gemm_ms": [round(float(x), 3) for x in tab[:, 3]],
                          "reduce_scatter_ms": [round(float(x), 3) for x in tab[:, 4]],
                          "nvlink_bytes_sent_per_rank": int(per_rank_send),
                          "limiting": "reduce-scatter" if tab[:, 4].max() > tab[:, 3].max() else "tile GEMM"}
    return entry


# ------------------------------------------------------------------ HBM-bound phases (N=1)

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
    B = E.tile_dense(b_d, (TILE, TILE)).materialize()
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


# ------------------------------------------------------------------ CPU reference arm

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
    # each step a bounded sample: about a minute of CPU work over the run
    per = max(1.0, min(8.0, 60.0 / max(1, args.steps)))
    for _ in range(max(0, args.warmup)):
        cpu_baseline(args, w, budget_s=min(4.0, per))
    for _ in range(args.steps):
        vals.append(cpu_baseline(args, w, budget_s=per))
    v = statistics.median(x["value"] for x in vals)
    cb = dict(vals[-1])
    cb["value"] = v
    line = {"metric": "useful TFLOP/s (sparse einsum, C2 element-sparse SpMM)", "value": v, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded C2 generator)",
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
    """One other BASELINE configuration on its own line (``--workload C1`` ...);
    the same measurement as the headline line's ``configs`` entries."""
    import torch
    import torch.distributed as dist
    rank, world, local = _env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
    fn = {"C1": measure_c1, "C3": measure_c3, "C4": measure_c4, "C5": measure_c5}[args.workload]
    with ClockSampler(local) as clk:
        entry = fn(args, dev, rank, world, clk, barrier, args.steps, max(args.warmup, 3))
    if rank == 0:
        line = {"metric": f"useful TFLOP/s (sparse einsum, {args.workload})", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": entry.pop("scaling", "strong"),
                "vs_baseline": None, "dtype": "bf16" if args.workload == "C3" else "f32",
                "data": f"synthetic (seeded {args.workload} generator)"}
        line.update(entry)
        line["config"] = {"workload": entry["workload"], "l2": "device-resident inputs; no flush"}
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scale", type=int, default=1, help="shrink C2 by this factor (testing only)")
    ap.add_argument("--c5-scale", type=int, default=1, help="shrink C5 by this factor (testing only)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--precision", default="auto", choices=["auto", "exact", "tc"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-hbm", action="store_true", help="skip the HBM-bound phase breakdown")
    ap.add_argument("--no-configs", action="store_true", help="skip the other configurations")
    ap.add_argument("--configs", default="", help="comma-separated subset of C1,C3,C4,C5 for the configs entry")
    ap.add_argument("--workload", default="C2", choices=["C1", "C2", "C3", "C4", "C5", "STATS"],
                    help="C2 is the headline line (with the others under 'configs'); the others alone")
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

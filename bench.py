#!/usr/bin/env python
"""Benchmark of the hist path: boosting rounds per second at config C2.

Workload: binary logistic on 10,000,000 x 28 f32 rows,
N(0,1) with 5% NaN, max_bin 256, max_depth 8, eta 0.1, every row in every
tree; seeded synthetic data of that shape (hessboost_b200.synth). A step is
one boosting round: gradients at the device margins, one depth-8 tree grown
on the device, its leaves added to the margins, the tree read back.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With N > 1 (launched by torch.distributed.run, one process per GPU) the rows
are sharded over the ranks (strong scaling: the 10M rows stay 10M) and every
histogram is summed with NCCL; rank 0 prints one JSON line.

`--impl reference` times the reference's CPU path instead. The reference
(Rust) cannot be built in this image, so its arm runs the C++ restatement
under oracle/ on the host cores (rank 0 only).
"""

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

METRIC = "boost rounds/s at 10M×28 depth-8 on 1/2/4/8 B200; hist-build GB/s vs HBM peak"
UNIT = "rounds/s"
N_ROWS = 10_000_000
N_COLS = 28
MISSING = 0.05
PARAMS = dict(objective="binary:logistic", max_depth=8, eta=0.1, max_bin=256)
# DRAM bytes (read + write) per k_hist32 launch at C2, 10M rows on one GPU:
# the mean over one round's root and 7 level launches of an ncu capture
# (profiles/k_hist32_c2_10M_traffic.md).
HIST_TRAFFIC_C2 = 422.0e6


# The one JSON line goes to the real stdout; everything else that writes to
# file descriptor 1 (NCCL's version banner, library messages) goes to stderr.
_RESULT = None


def claim_stdout():
    global _RESULT
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def emit(line):
    out = _RESULT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def set_rows(n):
    global N_ROWS
    N_ROWS = int(n)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def config(n_gpus):
    return {
        "workload": f"C2: binary:logistic, {N_ROWS:,} x 28 f32 N(0,1) with 5% NaN, max_bin 256, "
        "max_depth 8, eta 0.1, lambda 1, every row in every tree",
        "rows": N_ROWS,
        "features": N_COLS,
        "max_depth": 8,
        "max_bin": 256,
        "parallelism": f"rows sharded over {n_gpus} GPU(s), one NCCL allreduce per level"
        if n_gpus > 1 else "1 GPU",
        "l2": _l2_note(),
        "hist_kernel": os.environ.get("HB_HIST_KERNEL", "default"),
    }


def _l2_note():
    rec, col, gp = N_ROWS * 32 / 1e6, N_ROWS * 28 / 1e6, N_ROWS * 8 / 1e6
    sizes = (f"the binned rows ({rec:,.0f} MB records + {col:,.0f} MB columns) and {gp:,.0f} MB of "
             "gradients are re-read every round")
    # 126 MB of L2 on a B200
    return ("inputs larger than L2: " if rec + gp > 126 else "inputs SMALLER than L2 at this size: ") + sizes


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    def __init__(self, gpus):
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", ",".join(str(g) for g in gpus)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self, t0=None, t1=None):
        """Median SM clock and throttle reasons of the samples taken in
        [t0 - 0.25 s, t1 + 0.05 s] (host wall clock), or of all samples when
        none fall in that window."""
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        from datetime import datetime

        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        samples = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 10:
                    continue
                try:
                    ts = datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    sm, mx = float(f[2]), float(f[3])
                except ValueError:
                    continue
                rs = {name for name, v in zip(names, f[6:10]) if v.lower().startswith("active")}
                samples.append((ts, sm, mx, rs))
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if t0 is not None and t1 is not None:
            inside = [x for x in samples if t0 - 0.25 <= x[0] <= t1 + 0.05]
            if inside:
                samples = inside
        if not samples:
            return None
        reasons = set().union(*(x[3] for x in samples))
        return {"sm_mhz": statistics.median(x[1] for x in samples),
                "sm_max_mhz": max(x[2] for x in samples), "reasons": sorted(reasons),
                "samples": len(samples)}


def make_data():
    from hessboost_b200 import synth

    return synth.logistic_c2(N_ROWS, N_COLS, seed=0, missing=MISSING)


# ------------------------------------------------------------------ reference
def oracle_trainer(x, y, fixed_point=False):
    """The oracle (the reference's CPU hist path restated in C++, OpenMP over
    the host cores) prepared on the C2 matrix: cuts, bins, intercept."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O

    O.build()
    return O.Trainer(x, y, objective=1, max_depth=8, eta=0.1, max_bin=256, fixed_point=fixed_point)


def cpu_rounds(x, y, k_max, budget_s, warm=1, keep=False):
    """The oracle's rounds: preparation untimed, `warm` untimed rounds, then
    rounds timed, at most `k_max`, stopping once `budget_s` seconds are
    spent. Returns (rounds, seconds[, trainer when `keep`])."""
    tr = oracle_trainer(x, y)
    for _ in range(warm):
        tr.rounds(1)
    done, t0 = 0, time.perf_counter()
    while done < k_max:
        tr.rounds(1)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    if keep:
        return done, dt, tr
    tr.close()
    return done, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    x, y = make_data()
    warm = args.warmup
    k, dt = cpu_rounds(x, y, max(1, args.steps), budget_s=240.0, warm=warm)
    value = k / dt
    sample = (f"{k} timed round(s) of the C2 workload ({N_ROWS:,} rows) after binning and {warm} untimed round(s) "
              f"(C++ restatement of hessboost's CPU hist path, OpenMP on {cores} threads; "
              "the Rust reference cannot be built offline)")
    emit({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": k, "warmup": warm,
        "ms_per_step": 1000.0 * dt / k, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic", "config": config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


# ------------------------------------------------------------------ C5
C5_ROWS, C5_COLS, C5_TREES, C5_DEPTH = 100_000_000, 50, 1000, 8
C5_METRIC = "prediction rows/s (C5: 1,000 complete depth-8 trees, 100M x 50 f32 rows, 1% NaN)"


def c5_rows_device(torch, n, seed, chunk=10_000_000):
    """n x 50 rows, N(0,1) with 1% NaN, generated on the device in chunks."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.empty((n, C5_COLS), dtype=torch.float32, device="cuda")
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        x[a:b].normal_(generator=g)
        x[a:b][torch.rand((b - a, C5_COLS), device="cuda", generator=g) < 0.01] = float("nan")
    return x


def run_c5(args):
    """Batch prediction of the C5 ensemble (GpuModel::predict_margin). A step
    is one pass over all rows already in HBM; e2e predicts a pinned host
    sample through hb_predict_margin."""
    import torch

    import hessboost_b200 as H
    from hessboost_b200 import synth

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    torch.cuda.set_device(0)
    n = args.rows if args.rows is not None else C5_ROWS
    nodes, tree_ptr = synth.forest_c5(C5_TREES, C5_DEPTH, C5_COLS, seed=0)
    base = np.array([0.5], np.float32)
    pred = H.Predictor(nodes, tree_ptr, base, C5_COLS)
    x = c5_rows_device(torch, n, seed=1)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()  # a real stream: NULL would select the predictor's own
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        pred.predict_margin_device(x.data_ptr(), n, out.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    sampler = ClockSampler([0])
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        pred.predict_margin_device(x.data_ptr(), n, out.data_ptr(), stream.cuda_stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop(t_wall0, t_wall1)
    value = n * args.steps / (ms / 1000.0)
    # parity on a sample: the oracle's prediction of the same rows
    import oracle_lib as O

    O.build()
    k = 4096
    xs = x[:k].cpu().numpy()
    want = O.predict(nodes, tree_ptr, 1, base, xs)[:, 0]
    got = out[:k].cpu().numpy()
    exact = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
    # end to end: pinned host rows in, host margins out
    m = min(n, 8_000_000)
    xh = x[:m].cpu().pin_memory()
    oh = torch.empty(m, dtype=torch.float32).pin_memory()
    pred.predict_margin_into(xh.numpy(), oh.numpy())
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        pred.predict_margin_into(xh.numpy(), oh.numpy())
    e2e = m * reps / (time.perf_counter() - t0)
    # CPU baseline: the oracle on a bounded sample
    kc = 20_000
    xc = x[:kc].cpu().numpy()
    t0 = time.perf_counter()
    O.predict(nodes, tree_ptr, 1, base, xc)
    cpu_rate = kc / (time.perf_counter() - t0)
    step_bytes = n * C5_COLS * 4 + n * 4
    line = {
        "metric": C5_METRIC, "value": value, "unit": "rows/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"C5: {C5_TREES} complete depth-{C5_DEPTH} trees (features U[0,50), "
                               "thresholds from N(0,1) quantiles, leaves N(0,0.01)), "
                               f"{n:,} x {C5_COLS} f32 rows N(0,1) with 1% NaN, raw margin",
                   "l2": f"rows ({n * C5_COLS * 4 / 1e9:.2f} GB) "
                         f"{'larger' if n * C5_COLS * 4 > 126e6 else 'SMALLER'} than L2; "
                         "the forest (8 MB) stays in L2",
                   "parity_sample_bit_exact": exact},
        "roofline": {"bound": "hbm", "achieved": step_bytes / (ms / args.steps / 1000.0) / 1e9,
                     "peak": peaks()[0], "unit": "GB/s",
                     "frac": step_bytes / (ms / args.steps / 1000.0) / 1e9 / peaks()[0],
                     "traffic": None, "kernel": "k_predict",
                     "note": "HBM floor only (rows in, margins out); the binding resource is "
                             "on-chip: 8e11 dependent node steps per pass"},
        "cpu_baseline": {"value": cpu_rate, "unit": "rows/s", "cores": 1, "kind": "port",
                         "sample": f"{kc} rows through the oracle's predictor, 1 thread"},
        "e2e": {"value": e2e, "unit": "rows/s", "h2d_bytes_per_step": m * C5_COLS * 4,
                "d2h_bytes_per_step": m * 4,
                "scope": f"hb_predict_margin over {m:,} pinned host rows (copies in the timed region)"},
        "gpu_launches": args.steps,  # one k_predict launch per pass
        "clocks": clocks,
    }
    emit(line)
    pred.close()


# ------------------------------------------------------------------ C3
C3_METRIC = "multiclass boost rounds/s (C3: 2M x 100, 10 classes, max_bin 128, depth 6; 10 trees a round)"


def run_c3(args):
    """multi:softmax rounds at C3 (one GPU): device softmax gradients of all
    ten classes, then one tree per class. A step is one round."""
    import torch

    import hessboost_b200 as H
    from hessboost_b200 import synth

    torch.cuda.set_device(0)
    n = args.rows if args.rows is not None else 2_000_000
    x, y = synth.multiclass_c3(n, 100, 10, seed=0)
    params = H.TrainingParams(objective="multi:softmax", num_class=10, max_depth=6, eta=0.2, max_bin=128)
    m = H.BinnedMatrix.from_dense(x, 128)
    base = H.softmax_intercepts(y, 10)
    eng = H.Engine(0)
    eng.upload(m)
    eng.train_begin_classes(y, base)
    sampler = ClockSampler([0])
    eng.train_rounds(params, args.warmup)
    eng.reset_stats(timing=1)
    t_wall0 = time.time()
    nodes, ptr = eng.train_rounds(params, args.steps)
    t_wall1 = time.time()
    st = eng.stats()
    ms = st["last_rounds_ms"]
    clocks = sampler.stop(t_wall0, t_wall1)
    value = args.steps / (ms / 1000.0)
    hist_ms = st["ms"]["hist"] + st["ms"]["root_hist"]
    hist_launches = st["timed_launches"]["hist"] + st["timed_launches"]["root_hist"]
    alg = (st["rows_built_contiguous"] * (100 + 8) + st["rows_built_gathered"] * (100 + 8 + 4))
    achieved = alg / (hist_ms / 1000.0) / 1e9 if hist_ms > 0 else 0.0
    peak = peaks()[0]
    eng.reset_stats(timing=2)  # per-family breakdown, outside the timed region
    eng.train_rounds(params, min(args.steps, 5))
    bd = eng.stats()
    per_round = {k: v / max(bd["rounds"], 1) * 10 for k, v in bd["ms"].items()}  # 10 trees a round
    # the first round's ten trees from the base margins, for the parity check
    eng.train_begin_classes(y, base)
    first_nodes, first_ptr = eng.train_rounds(params, 1)
    eng.close()
    parity = None
    if not args.no_parity:
        parity = c3_parity(x, y, base, first_nodes, first_ptr)
    cpu = None
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import oracle_lib as O

        O.build()
        tr = O.Trainer(x, y, objective=2, n_outputs=10, max_depth=6, eta=0.2, max_bin=128)
        t0 = time.perf_counter()
        k = 0
        while k < 3 and time.perf_counter() - t0 < 30.0:
            tr.rounds(1)
            k += 1
        dt = time.perf_counter() - t0
        tr.close()
        cpu = {"value": k / dt, "unit": "rounds/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{k} round(s) of the full C3 workload after binning (oracle, OpenMP)"}
    emit({
        "metric": C3_METRIC, "value": value, "unit": "rounds/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": {"workload": f"C3: multi:softmax, {n:,} x 100 f32 U(-1,1), 10 classes "
                               "(argmax of random projections + Gumbel noise), max_bin 128, "
                               "max_depth 6, eta 0.2",
                   "trees": int(len(ptr) - 1),
                   "kernel_ms_per_round": per_round,
                   "l2": f"inputs {'larger' if n * 128 > 126e6 else 'SMALLER'} than L2: "
                         f"{n:,} x 128 B records + 10 x {n * 8 / 1e6:,.0f} MB pairs per round"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "kernel": "k_hist32",
                     "launches": hist_launches},
        "cpu_baseline": cpu,
        "parity": parity,
        "e2e": None,
        "gpu_launches": int(st["kernel_launches"]),
        "clocks": clocks,
    })


def c4_parity(indptr, indices, values, n_cols, y, nodes, ptr, margins):
    """The GPU's first C4 round (one lossguide tree over the 5M x 2,000 CSR
    index) against the oracle's fixed-point CSR trainer on the same matrix:
    every node field and all training margins bit for bit."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    import parity as P

    O.build()
    t0 = time.perf_counter()
    tr = O.Trainer(None, y, csr=(indptr, indices, values, n_cols), objective=1, grow_policy=1,
                   max_depth=0, max_leaves=255, max_bin=64, fixed_point=True)
    on, op = tr.rounds(1)
    om = tr.margins()[:, 0]
    tr.close()
    exact, where = P.forest_bit_exact(nodes, ptr, on, op)
    m_exact = bool(np.array_equal(np.ascontiguousarray(margins, np.float32).view(np.uint32), om.view(np.uint32)))
    log(f"c4 parity: {time.perf_counter() - t0:.1f}s")
    return {"rows": int(len(y)), "rounds": 1, "fixed_point_bit_exact": bool(exact),
            "fixed_point_first_difference": where or None, "fixed_point_margins_bit_exact": m_exact,
            "pass": bool(exact and m_exact),
            "criteria": "oracle fixed point (CSR index, lossguide), first round: every node field and "
                        "margin bit for bit"}


def c3_parity(x, y, base, nodes, ptr):
    """The GPU's first C3 round (ten trees, one per class, from the class
    intercepts) against the oracle's fixed-point mode on the same 2M x 100
    matrix, under the north-star criteria (the device's softmax exp is CUDA's
    double exp rounded once, the oracle's glibc expf, so not bit for bit):
    trees, leaves and the margins after the round (GPU predictor on the
    training rows)."""
    import hessboost_b200 as H

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    import parity as P

    O.build()
    t0 = time.perf_counter()
    tr = O.Trainer(x, y, objective=2, n_outputs=10, max_depth=6, eta=0.2, max_bin=128, fixed_point=True)
    on, op = tr.rounds(1)
    om = tr.margins()
    tr.close()
    cmp = P.compare_forests(nodes, ptr, on, op)
    bases = np.ascontiguousarray(base, np.float32)
    pred = H.Predictor(nodes, ptr, bases, x.shape[1])
    gm = pred.predict_margin(x)
    pred.close()
    ok, rel, exact = P.margins_ok(gm, om)
    log(f"c3 parity: {time.perf_counter() - t0:.1f}s")
    return dict(cmp, rows=int(x.shape[0]), rounds=1, margins_ok=ok, margin_max_rel=rel,
                margin_bit_exact_frac=exact, pass_all=bool(cmp["pass"] and ok),
                criteria="oracle fixed point, first round: structure equal except gain ties (1e-5), "
                         "leaves rtol 1e-5 atol 1e-7, margins rtol 1e-6 atol 1e-7")


C4_METRIC = "boost rounds/s (C4: 5M x 2,000 CSR at 2%, max_bin 64, lossguide 255 leaves)"


def run_c4(args):
    """Lossguide rounds over a CSR index at C4 (one GPU): 2,000 features at
    2% density, 64 bins, up to 255 leaves a tree (no depth limit). A step is
    one round: gradients (with the last tree's walk over the CSR rows), one
    lossguide tree grown on the device, read back."""
    import torch

    import hessboost_b200 as H
    from hessboost_b200 import synth

    torch.cuda.set_device(0)
    n = args.rows if args.rows is not None else 5_000_000
    f = 2000
    t0 = time.perf_counter()
    indptr, indices, values, y = synth.sparse_c4(n, f, density=0.02, seed=0)
    t1 = time.perf_counter()
    m = H.BinnedMatrix.from_csr(indptr, indices, values, f, 64)
    t2 = time.perf_counter()
    log(f"c4: data {t1 - t0:.1f} s, host binning {t2 - t1:.1f} s, nnz {int(indptr[-1]):,}")
    nnz = int(indptr[-1])
    params = H.TrainingParams(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                              max_leaves=255, max_bin=64)
    eng = H.Engine(0)
    eng.upload(m)
    eng.train_begin(y, H.base_margin(params, y))
    sampler = ClockSampler([0])
    eng.train_rounds(params, args.warmup)
    eng.reset_stats(timing=1)
    t_wall0 = time.time()
    nodes, ptr = eng.train_rounds(params, args.steps)
    t_wall1 = time.time()
    st = eng.stats()
    ms = st["last_rounds_ms"]
    clocks = sampler.stop(t_wall0, t_wall1)
    value = args.steps / (ms / 1000.0)
    hist_ms = st["ms"]["hist"] + st["ms"]["root_hist"]
    hist_launches = st["timed_launches"]["hist"] + st["timed_launches"]["root_hist"]
    rows_built = st["rows_built_contiguous"] + st["rows_built_gathered"]
    per_row = nnz / n
    # per built row: its offsets (16 B), gradient pair (8 B), a gathered row
    # id (4 B) and its stored cells' bins (4 B each, the matrix average)
    alg = rows_built * (16 + 8 + 4 * per_row) + st["rows_built_gathered"] * 4
    achieved = alg / (hist_ms / 1000.0) / 1e9 if hist_ms > 0 else 0.0
    updates = rows_built * per_row / (hist_ms / 1000.0) if hist_ms > 0 else 0.0
    peak = peaks()[0]
    eng.reset_stats(timing=2)  # per-family breakdown, outside the timed region
    eng.train_rounds(params, min(args.steps, 3))
    bd = eng.stats()
    per_round = {k: v / max(bd["rounds"], 1) for k, v in bd["ms"].items()}
    # the first round from the base margin, for the parity check
    base = H.base_margin(params, y)
    eng.train_begin(y, base)
    first_nodes, first_ptr = eng.train_rounds(params, 1)
    first_margins = eng.read_margins()
    eng.close()
    parity = None
    if not args.no_parity:
        parity = c4_parity(indptr, indices, values, f, y, first_nodes, first_ptr, first_margins)
    cpu = None
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import oracle_lib as O

        O.build()
        rs = min(n, 250_000)
        e_s = int(indptr[rs])
        tr = O.Trainer(None, y[:rs], csr=(indptr[: rs + 1], indices[:e_s], values[:e_s], f), objective=1,
                       grow_policy=1, max_depth=0, max_leaves=255, max_bin=64)
        tr.rounds(1)
        t0 = time.perf_counter()
        k = 0
        while k < 3 and time.perf_counter() - t0 < 30.0:
            tr.rounds(1)
            k += 1
        dt = time.perf_counter() - t0
        tr.close()
        cpu = {"value": k / dt * rs / n, "unit": "rounds/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{k} round(s) on the first {rs:,} rows of the C4 matrix (oracle CSR index, OpenMP), "
                         f"scaled to {n:,} rows by the row ratio"}
    emit({
        "metric": C4_METRIC, "value": value, "unit": "rounds/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": {"workload": f"C4: binary:logistic, {n:,} x {f:,} CSR, 2% of cells stored (uniform "
                               "positions), values lognormal(0,1), absent cells missing, max_bin 64, "
                               "lossguide, max_leaves 255, no depth limit, eta 0.3",
                   "nnz": nnz, "trees": int(len(ptr) - 1), "leaves_per_tree": round(
                       float(np.mean([(int(ptr[i + 1] - ptr[i]) + 1) // 2 for i in range(len(ptr) - 1)])), 1),
                   "hist_updates_per_s": updates,
                   "kernel_ms_per_round": per_round,
                   "l2": f"inputs larger than L2: {nnz * 4 / 1e9:.2f} GB of bins"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "kernel": "k_hist_csr",
                     "launches": hist_launches},
        "cpu_baseline": cpu,
        "parity": parity,
        "e2e": None,
        "gpu_launches": int(st["kernel_launches"]),
        "clocks": clocks,
    })


# ------------------------------------------------------------------ probe
PROBE_KINDS = {
    0: "red.shared.add.u32, conflict-free",
    1: "red.shared.add.u64, conflict-free",
    2: "atom.shared.add.u32, result used",
    3: "ld.shared.u32 + st.shared.u32",
    4: "k_hist32 update: 4 x red.u32 at a random row, diagonal column",
    5: "64-bit update: 2 x red.u64 at a random row, diagonal column",
    6: "red.shared.add.u32, 32 lanes on one word",
}


def run_probe(args):
    """Shared-memory throughput of the histogram update patterns
    (hb_probe_smem): lane operations per SM clock, one CTA per SM."""
    import ctypes

    import hessboost_b200 as H

    out = {}
    for threads in (512, 1024):
        for kind, what in PROBE_KINDS.items():
            v = ctypes.c_double()
            st = H.lib().hb_probe_smem(0, kind, threads, 4096, ctypes.byref(v))
            if st != H.HB_OK:
                raise SystemExit(f"hb_probe_smem kind {kind}: status {st}")
            out.setdefault(str(threads), {})[f"{kind}: {what}"] = round(v.value, 2)
    emit({"probe": "smem", "unit": "lane operations per SM clock (slowest SM)",
          "iters": 4096, "results_by_threads_per_cta": out})


# ------------------------------------------------------------------ ours
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the comparison of the first trees with the oracle (N=1)")
    ap.add_argument("--parity-rounds", type=int, default=3)
    ap.add_argument("--no-row-engine", action="store_true",
                    help="skip timing the RowEngine host loop (device_round over the trait calls)")
    ap.add_argument("--rows", type=int, default=None,
                    help="rows of the synthetic matrix (default: the workload's own, 10M for "
                         "C2 and 100M for C5; smaller values are for profiling captures)")
    ap.add_argument("--workload", default="c2", choices=["c2", "c3", "c4", "c5"],
                    help="c2: boosting rounds (the headline); c3: multiclass rounds; "
                         "c4: lossguide rounds over a CSR index; c5: batch prediction")
    ap.add_argument("--probe", choices=["smem"], default=None,
                    help="smem: measure the shared-memory atomic throughput the histogram "
                         "kernels are bound by (hb_probe_smem), instead of a workload")
    args = ap.parse_args()
    if args.probe:
        claim_stdout()
        run_probe(args)
        return
    if args.rows is not None and args.workload == "c2":
        set_rows(args.rows)
    claim_stdout()
    if args.workload == "c5":
        run_c5(args)
        return
    if args.workload == "c3":
        run_c3(args)
        return
    if args.workload == "c4":
        run_c4(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    import hessboost_b200 as H
    from hessboost_b200 import dist as hdist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def allreduce_max(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def allreduce_sum(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    t_data = time.perf_counter()
    x, y = make_data()
    params = H.TrainingParams(**PARAMS)
    # cut table over the whole matrix (rank 0), shared so every rank bins
    # against the same cuts; the index-level dense flag is the whole matrix's
    prep = None
    if world > 1:
        shard, begin, end = hdist.shard_matrix(dist, x, 256, device=local)
    else:
        # sketch + binning of the whole matrix on the GPU (hb_sketch_dense:
        # the f32 matrix up, cuts and binned columns back), then the same on
        # the host's threads (hb_cuts_dense + hb_bin_dense), for the record
        begin, end = 0, N_ROWS
        H.sketch_dense(x[:4096], 256, local)  # context and module load
        t0 = time.perf_counter()
        off, cuts, cols, miss, dense = H.sketch_dense(x, 256, local)
        t_dev = time.perf_counter() - t0
        t0 = time.perf_counter()
        hoff, hcuts = H.cuts_dense(x, 256)
        hcols, _, _ = H.bin_dense(x, hoff, hcuts)
        t_host = time.perf_counter() - t0
        if not (np.array_equal(hcuts.view(np.uint32), cuts.view(np.uint32)) and np.array_equal(hcols, cols)):
            raise SystemExit("device sketch and host sketch disagree")
        del hcols
        shard = H.BinnedMatrix(off, cuts, cols, miss, dense)
        prep = {"device_sketch_and_bins_s": t_dev, "host_sketch_and_bins_s": t_host,
                "host_threads": os.cpu_count() or 1,
                "scope": "HistCuts + GHistIndex of the 10M x 28 f32 matrix from host memory "
                         "(device: hb_sketch_dense, upload and download included; host: "
                         "hb_cuts_dense + hb_bin_dense); same cuts and bins, checked"}
    off, cuts, cols, miss, dense = (shard.feature_offset, shard.cut_values, shard.columns,
                                    shard.missing, shard.dense)
    base = H.base_margin(params, y)
    log(f"[rank {rank}] data + binning {time.perf_counter() - t_data:.1f}s rows [{begin}, {end})")

    eng = H.Engine(local)
    eng.set_shard(begin, N_ROWS)
    if world > 1:
        uid = hdist.broadcast_unique_id(dist, hdist.unique_id)
        eng.comm_init(world, rank, uid, N_ROWS)
    eng.upload(shard)
    y_shard = np.ascontiguousarray(y[begin:end])
    eng.train_begin(y_shard, base)
    # clocks sampled from before the warm-up to the end of the timed region
    # (nvidia-smi needs a moment to start)
    sampler = ClockSampler([local]) if rank == 0 else None
    eng.train_rounds(params, args.warmup)

    # ---- timed region: K rounds, device time, max over ranks. No event
    # nodes inside the rounds: events around the histogram launches cost
    # about 0.08 ms a round (they break the launches' programmatic
    # overlap), so the histogram kernel's own times come from a second pass
    eng.reset_stats(timing=0)
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    ev0.record(stream)
    nodes, tree_ptr = eng.train_rounds(params, args.steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    barrier()
    st = eng.stats()
    # the K rounds' device time: CUDA events the engine records on its
    # stream around the rounds (the bracketing events above also hold the
    # host-side graph capture); max over ranks
    ms = allreduce_max(st["last_rounds_ms"] if st["last_rounds_ms"] > 0 else ev0.elapsed_time(ev1))
    clocks = sampler.stop(t_wall0, t_wall1) if sampler else None
    launches = int(allreduce_sum(st["kernel_launches"]))
    value = args.steps / (ms / 1000.0)

    # roofline of the histogram kernel (root + level launches of k_hist32):
    # a second pass of K rounds with CUDA events around every histogram
    # launch, on the engine's stream
    eng.reset_stats(timing=1)
    barrier()
    eng.train_rounds(params, args.steps)
    torch.cuda.synchronize()
    sth = eng.stats()
    hist_ms = sth["ms"]["hist"] + sth["ms"]["root_hist"]
    hist_launches = sth["timed_launches"]["hist"] + sth["timed_launches"]["root_hist"]
    bitmap = N_COLS / 8.0 if not dense else 0.0
    alg_bytes = (sth["rows_built_contiguous"] * (N_COLS + 8 + bitmap)
                 + sth["rows_built_gathered"] * (N_COLS + 8 + 4 + bitmap))
    achieved = alg_bytes / (hist_ms / 1000.0) / 1e9 if hist_ms > 0 else 0.0
    peak, peak_kind = peaks()
    log(f"[rank {rank}] {args.steps} rounds {ms:.1f} ms; kernel ms {json.dumps(st['ms'])}")
    # per-family breakdown (events around every kernel family), outside the
    # timed region
    eng.reset_stats(timing=2)
    eng.train_rounds(params, min(args.steps, 20))
    breakdown = eng.stats()
    per_round = {k: v / max(breakdown["rounds"], 1) for k, v in breakdown["ms"].items()}

    # ---- the reference's unchanged device round over the RowEngine calls
    # (device_round + build_on_device: a host level loop, one C-ABI call per
    # trait method), one GPU
    row_engine = None
    if world == 1 and not args.no_row_engine:
        from hessboost_b200.device_builder import RowEngineTrainer

        eng.load_margins(np.full(end - begin, base, np.float32))
        rt = RowEngineTrainer(eng, params, y_shard)
        rt.round()  # warm-up: slot reservation, first allocations
        k_re = max(1, min(args.steps, 10))
        c0 = rt.calls
        rt.seconds = {}
        t0 = time.perf_counter()
        for _ in range(k_re):
            rt.round()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        row_engine = {"value": k_re / dt, "unit": UNIT, "rounds": k_re,
                      "ms_per_round": 1000.0 * dt / k_re,
                      "calls_per_round": (rt.calls - c0) / k_re,
                      "ms_per_round_by_call": {k: 1000.0 * v / k_re for k, v in rt.seconds.items()},
                      "whole_round_ms_per_round": ms / args.steps,
                      "scope": "hessboost_b200.device_builder.RowEngineTrainer: gradients, begin_tree, "
                               "root_total, reserve_hists, build_resident, scan_resident per level, "
                               "partition, add_leaf_values through the C ABI, host wall clock"}
        log(f"row engine: {1000.0 * dt / k_re:.2f} ms/round ({row_engine['calls_per_round']:.0f} calls)")

    # ---- end to end through the C ABI from pinned host buffers
    barrier()
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()  # noqa: E731
    pcols, plab = pin(cols), pin(y_shard)
    pmiss = pin(miss) if not dense else None
    e2e_shard = H.BinnedMatrix(off, cuts, pcols, pmiss, dense)
    # the same engine (its device context and, for N > 1, its NCCL
    # communicator with connections already set up, as in a training service
    # that trains again on new data); upload, training start and the K rounds
    # from host buffers are all inside the timed region
    eng.reset_stats(timing=0)  # no event nodes in the end-to-end rounds
    barrier()
    t0 = time.perf_counter()
    eng.upload(e2e_shard)
    eng.train_begin(plab, base)
    nodes2, ptr2 = eng.train_rounds(params, args.steps)
    torch.cuda.synchronize()
    e2e_s = allreduce_max(time.perf_counter() - t0)
    barrier()
    h2d = (pcols.nbytes + (pmiss.nbytes if pmiss is not None else 0) + plab.nbytes
           + off.nbytes + cuts.nbytes)
    h2d_total = allreduce_sum(h2d)
    d2h_total = allreduce_sum(len(nodes2) * H.NODE_DTYPE.itemsize)
    e2e = {"value": args.steps / e2e_s, "unit": UNIT,
           "h2d_bytes_per_step": h2d_total / args.steps, "d2h_bytes_per_step": d2h_total / args.steps,
           "scope": "hb_engine_upload of the binned shard + hb_train_begin + hb_train_rounds(K) from "
                    "pinned host buffers on an engine already created (and, for N > 1, already "
                    "connected); trees read back"}
    # the forest of the end-to-end run (K trees from the base margin): the
    # same bytes at every GPU count when the sums are exact
    from hessboost_b200 import model_io

    forest = {"xxh64": f"{model_io.xxh64(np.ascontiguousarray(nodes2).tobytes()):016x}",
              "trees": int(len(ptr2) - 1), "nodes": int(len(nodes2)),
              "scope": "hb_tree_node records of the end-to-end run's K trees, grown from the base margin"}

    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        k, dt, tr64 = cpu_rounds(x, y, 3, budget_s=25.0, warm=1, keep=True)
        cpu = {"value": k / dt, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{k} round(s) of the C2 workload ({N_ROWS:,} rows) after binning and 1 untimed round (C++ restatement of "
                         f"hessboost's CPU hist path, OpenMP, {cores} threads)"}
        if not args.no_parity:
            parity = c2_parity(eng, params, x, y_shard, base, nodes2, ptr2, tr64, args.parity_rounds)
        tr64.close()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": config(world),
            "details": {"rows_per_s": value * N_ROWS, "trees_nodes": int(len(nodes)),
                        "kernel_ms_per_round": per_round, "prep": prep,
                        "timing": "device time of the K rounds from CUDA events the engine records "
                                  "on its stream around them (rounds replayed as a CUDA graph, no "
                                  "event nodes inside); histogram kernel times for the roofline "
                                  "from a second pass of K rounds with events around each "
                                  "histogram launch; per-family breakdown from a third, "
                                  "instrumented run"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": HIST_TRAFFIC_C2 if (N_ROWS == 10_000_000 and world == 1) else None,
                         "kernel": "k_hist32", "launches": hist_launches,
                         "avg_launch_ms": hist_ms / max(hist_launches, 1),
                         "timing": "CUDA events on the engine's stream around each histogram "
                                   "launch of a second pass of K rounds (the timed pass has none)",
                         "alg_bytes_per_launch": alg_bytes / max(hist_launches, 1),
                         "alg_bytes_rule": f"per built row: {N_COLS} B of bins + 8 B (g, h) pair + "
                                           f"{bitmap} B missing bitmap + 4 B row id when gathered",
                         "traffic_note": "DRAM bytes read + written per launch, averaged over one "
                                         "round's 8 launches at 10M rows, from the ncu capture in "
                                         "profiles/k_hist32_c2_10M_traffic.md (not from this run; "
                                         "null at other sizes)",
                         "peak_kind": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)"},
            "cpu_baseline": cpu,
            "parity": parity,
            "forest": forest,
            "row_engine": row_engine,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        emit(line)
    eng.close()
    if world > 1:
        dist.destroy_process_group()


def c2_parity(eng, params, x, y, base, nodes, ptr, tr64, rounds):
    """The GPU's first trees at C2 against the oracle on the same 10M-row
    matrix: (1) the oracle's fixed-point mode, every node field and the
    training margins bit for bit; (2) the oracle's f64 mode (the reference's
    summation), round by round from the same margins, under the north-star
    criteria (tests/parity.py)."""
    import parity as P

    t0 = time.perf_counter()
    rounds = min(rounds, len(ptr) - 1)
    trq = oracle_trainer(x, y, fixed_point=True)
    on, op = trq.rounds(rounds)
    om = trq.margins()[:, 0]
    trq.close()
    gn = nodes[: int(ptr[rounds])]
    exact, where = P.forest_bit_exact(gn, ptr[: rounds + 1], on, op)
    eng.train_begin(y, base)
    eng.train_rounds(params, rounds)
    gm = eng.read_margins()
    m_exact = bool(np.array_equal(gm.view(np.uint32), om.view(np.uint32)))
    t1 = time.perf_counter()
    eng.train_begin(y, base)
    f64 = P.forced_f64_rounds(eng, params, tr64, rounds)
    t2 = time.perf_counter()
    log(f"parity: fixed {t1 - t0:.1f}s f64 {t2 - t1:.1f}s")
    return {"rows": int(len(y)), "fixed_point_rounds": rounds,
            "fixed_point_bit_exact": bool(exact), "fixed_point_first_difference": where or None,
            "fixed_point_margins_bit_exact": m_exact,
            "f64": f64,
            "pass": bool(exact and m_exact and f64["pass"]),
            "criteria": "fixed point: every node field and margin bit for bit; f64 mode, each round "
                        "from the same margins: structure equal except gain ties (1e-5), leaves "
                        "rtol 1e-5 atol 1e-7, margins rtol 1e-6 atol 1e-7"}


if __name__ == "__main__":
    main()

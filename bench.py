#!/usr/bin/env python3
"""Benchmark of the decode-fused DOT library (libautdot, sm_100a).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload e8-sweep|e2m3|lns|raw|gemv] [--accum fp32|fp64]

Default workload (the one the headline metric is quoted on): the E8
truncated-float bit-width sweep -- e8m0 (9 bits; the 8-bit width has no room
for 8 exponent bits), e8m1 (10), e8m3 (12), e8m5 (14), bf16_e8m7 (16) and
e8m15 (24) -- stored as dense LSB-first 32-bit-word bitstreams with fields
crossing word boundaries, N = 2^27 values per GPU, x, y uniform[-1, 1)
(seeded, counter based), contiguous shards over GPUs, one FP64 all-reduce.
A step is one fused DOT per format (six launches) plus, on more than one GPU,
one NCCL all-reduce of the six FP64 partials.

value       packed HBM GB/s of the whole job (2 N bits / 8 per DOT, all GPUs),
            inputs resident in HBM; each pair is larger than the 126 MB L2 and
            consecutive DOTs read different buffers, so no L2 flush is needed.
e2e         the same metric through the C ABI from pinned HOST buffers: every
            step copies the packed vectors host->device, runs the DOTs and
            reads the FP64 results back.
roofline    the dominant kernel's packed bytes per launch / its CUDA-event
            launch time, against the measured HBM copy bandwidth.
per_config  (one GPU) every other storage format of the benchmark's
            configurations at its stated size -- raw FP32/FP64 (with the
            N = 2^10 ... 2^27 sweep), e2m3 dense and padded, the E8 sweep with
            the FP64 accumulator, lns8_r3 / lns16_r11 on the cancellation
            pair -- each accumulator and decoder: CUDA-event GB/s of packed
            bits (the reference's metric: 2 N bits / 8), GB/s of the bytes the
            layout moves (padded: whole 8/16/32-bit containers) and its
            fraction of the measured peak, and the normalised error against
            the reference's compensated long-double CPU DOT.  Also the GEMV (1024 x 2^17,
            vector in the same format) of the E8 sweep formats (FP32, FP64),
            e2m3 (dense, padded) and lns8_r3, error over three sampled rows.

The gemv workload runs aut_gemv instead: a 1024-row matrix of the E8 sweep
formats with N / 1024 columns per GPU (rows sharded over GPUs, no
collective), packed bytes = (rows * columns + columns) * bits / 8.
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

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

N_DEFAULT = 1 << 27
SEED = 0x243F6A8885A308D3
HBM_FALLBACK_GBS = 6650.0
DENSE, PADDED = 0, 1

# (family, total bits, exponent bits / LNS fraction bits, finite) of the
# formats the benchmark uses -- the registry entries of storage_formats.hpp
# and lns_benchmark_core.hpp, kept here so that the reference arm needs no
# product library.
FORMAT_DESC = {
    "fp32": (3, 32, 8, 0), "fp64": (4, 64, 11, 0), "e2m3": (0, 6, 2, 1),
    "e8m0": (0, 9, 8, 0), "e8m1": (0, 10, 8, 0), "e8m3": (0, 12, 8, 0),
    "e8m5": (0, 14, 8, 0), "bf16_e8m7": (0, 16, 8, 0), "e8m15": (0, 24, 8, 0),
    "lns8_r3": (2, 8, 3, 0), "lns16_r11": (2, 16, 11, 0),
}
E8_SWEEP = [("e8m0", 0), ("e8m1", 0), ("e8m3", 0), ("e8m5", 0), ("bf16_e8m7", 0),
            ("e8m15", 0)]

WORKLOADS = {
    # name: (description, [(format, generator kind)], layout, n per GPU)
    "e8-sweep": ("E8 truncated-float bit-width sweep e8m0/e8m1/e8m3/e8m5/bf16_e8m7/e8m15 "
                 "(9/10/12/14/16/24 bits), dense LSB-first u32 bitstream, x,y uniform[-1,1)",
                 E8_SWEEP, DENSE, N_DEFAULT),
    "e2m3": ("FP6 E2M3 dense (4 values per 24 bits), x,y ~ N(0,1) (Irwin-Hall), RNE encoded",
             [("e2m3", 2)], DENSE, N_DEFAULT),
    "lns": ("LNS lns8_r3 and lns16_r11, N=2^28, cancellation pair y_i = s_i x_i (1+1e-6 u_i)",
            [("lns8_r3", 3), ("lns16_r11", 3)], DENSE, 1 << 28),
    "raw": ("raw FP32 and FP64 storage DOT, x,y uniform[-1,1)",
            [("fp32", 1), ("fp64", 0)], DENSE, N_DEFAULT),
    "gemv": ("GEMV over the E8 sweep formats: 1024 x N/1024 matrix per GPU times a dense "
             "vector of the same format, uniform[-1,1)", E8_SWEEP, DENSE, N_DEFAULT),
}
GEMV_ROWS = 1024
METRIC = "decoded elems/s & HBM GB/s (% of 8 TB/s) at N=2^27/GPU, 1-8 GPUs; normalized err"

DECODERS = {"auto": 0, "direct": 1, "full_lut": 2, "fraction_lut": 3,
            "fraction_lut_fused": 4, "fused_sum_lut": 5, "ex2_approx": 6}

# The other configurations, timed on one GPU after the headline:
# (group, format, generator kind, layout, n, accumulators, decoders)
PER_CONFIG = [
    ("raw", "fp32", 1, DENSE, 1 << 27, ("fp32", "fp64"), ("auto",)),
    ("raw", "fp64", 0, DENSE, 1 << 27, ("fp64",), ("auto",)),
    ("e2m3", "e2m3", 2, DENSE, 1 << 27, ("fp32", "fp64"), ("auto", "full_lut")),
    ("e2m3", "e2m3", 2, PADDED, 1 << 27, ("fp32", "fp64"), ("auto",)),
] + [("e8-sweep", f, k, DENSE, 1 << 27, ("fp64",), ("auto",)) for f, k in E8_SWEEP] + [
    ("lns", "lns8_r3", 3, DENSE, 1 << 28, ("fp32", "fp64"),
     ("auto", "full_lut", "fused_sum_lut", "ex2_approx")),
    ("lns", "lns16_r11", 3, DENSE, 1 << 28, ("fp32", "fp64"),
     ("auto", "fraction_lut_fused", "fraction_lut", "full_lut", "ex2_approx")),
]
RAW_SWEEP = [10, 16, 20, 23, 26, 27]
# GEMV rows of per_config: (format, generator kind, layout, accumulators)
GEMV_CONFIG = [(f, k, DENSE, ("fp32", "fp64")) for f, k in E8_SWEEP] + [
    ("e2m3", 2, DENSE, ("fp32",)), ("e2m3", 2, PADDED, ("fp32",)),
    ("lns8_r3", 3, DENSE, ("fp32", "fp64")),
]


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="e8-sweep")
    p.add_argument("--accum", choices=["fp32", "fp64"], default="fp32")
    p.add_argument("--strategy", choices=["auto", "ldg", "tma"], default="auto")
    p.add_argument("--layout", choices=["dense", "padded"], default="dense",
                   help="storage layout of the DOT workloads")
    p.add_argument("--n", type=int, default=0, help="values per GPU (default: workload's)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-per-config", action="store_true",
                   help="skip the other configurations (one GPU only)")
    p.add_argument("--e2e-steps", type=int, default=6)
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peak():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return HBM_FALLBACK_GBS, "fallback"


def committed_traffic():
    path = os.path.join(HERE, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# ---- clocks during the timed region ---------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.first = 0  # samples before this index precede the timed region

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # wait for the first sample (nvidia-smi needs ~0.1 s to start)
            # before the ranks meet at the barrier that opens the timed region
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def mark(self):
        """Called as the timed region starts."""
        self.first = len(self.lines)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        timed = self.lines[self.first:] or self.lines[-1:]
        for line in timed:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


# ---- CPU baseline (the reference's CPU path on the host cores) -------------------
def _pyoracle():
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import pyoracle
    return pyoracle


def cpu_reference_dot(fmt_name, stride, xw, yw, n, threads):
    """The reference's host decode + compensated long-double DOT; oracle/_ref
    when the reference was compiled here, else the oracle's restatement."""
    pyoracle = _pyoracle()
    ref = pyoracle.reference()
    if ref is not None and fmt_name in ref.formats:
        d, s = ref.dot_dense(fmt_name, stride, xw, yw, n, threads)
        return d, s, "reference"
    if ref is not None and fmt_name in ("fp32", "fp64"):
        import numpy as np
        dt = np.float32 if fmt_name == "fp32" else np.float64
        d, s = ref.dot_raw(xw.view(dt)[:n], yw.view(dt)[:n], threads)
        return d, s, "reference"
    orc = pyoracle.oracle()
    d, s = orc.dot_dense(FORMAT_DESC[fmt_name], stride, xw, yw, n, threads)
    return d, s, "port"


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def normalized_error(got, d, s):
    import numpy as np
    ref = np.longdouble(d[0]) + np.longdouble(d[1])
    sabs = np.longdouble(s[0]) + np.longdouble(s[1])
    if got != got:
        return float("nan")
    return float(abs(np.longdouble(got) - ref) / sabs) if sabs else 0.0


def condition_number(d, s):
    import numpy as np
    ref = abs(np.longdouble(d[0]) + np.longdouble(d[1]))
    sabs = np.longdouble(s[0]) + np.longdouble(s[1])
    return float(sabs / ref) if ref else float("inf")


# ---- the reference arm ---------------------------------------------------------
def run_reference_arm(args, rank, world):
    """The reference's own CPU implementation of the path (host decode +
    compensated long-double DOT, compiled from its headers into
    oracle/_ref/libautref.so), on rank 0 with every host thread.  Inputs are
    generated by the oracle's generators and encoded and packed by the
    reference's own host codec; nothing here loads the product library."""
    if rank != 0:
        return 0
    import numpy as np
    desc, fmts, layout, n_full = WORKLOADS[args.workload]
    threads = host_threads()
    pyoracle = _pyoracle()
    orc = pyoracle.oracle()
    ref = pyoracle.reference()
    kind_used = "reference" if ref is not None else "port"
    pool_n = 1 << 22  # values generated per format; every step reads a prefix
    streams = []
    for name, kind in fmts:
        fam, bits, _, _ = FORMAT_DESC[name]
        x = orc.synthetic(kind, SEED, 0, pool_n)
        y = orc.synthetic(kind, SEED, 1, pool_n)
        if fam == 4:  # raw FP64
            streams.append((name, 64, x.view(np.uint32), y.view(np.uint32), bits))
            continue
        if fam == 3:  # raw FP32
            streams.append((name, 32, x.astype(np.float32).view(np.uint32),
                            y.astype(np.float32).view(np.uint32), bits))
            continue
        out = []
        for v in (x, y):
            if ref is not None:
                out.append(ref.pack_dense(bits, ref.encode(name, v)))
            else:
                out.append(orc.pack_dense(bits, orc.encode(FORMAT_DESC[name], v)))
        streams.append((name, bits, out[0], out[1], bits))

    def one_step(m):
        for name, stride, xw, yw, _ in streams:
            cpu_reference_dot(name, stride, xw, yw, m, threads)

    # A fixed per-step sample (the largest power of two up to 2^22 values per
    # format for which the whole run stays within about two minutes), so that
    # the figure is a property of the host, not of the step count.
    t0 = time.perf_counter()
    one_step(1 << 18)
    per_value = (time.perf_counter() - t0) / (1 << 18)
    budget = 120.0 / max(1, args.steps + args.warmup)
    m = pool_n
    while m > (1 << 14) and m * per_value > budget:
        m //= 2
    for _ in range(args.warmup):
        one_step(m)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step(m)
    elapsed = time.perf_counter() - t0
    bytes_step = sum(2 * m * b / 8 for (_, _, _, _, b) in streams)
    gbs = bytes_step * args.steps / elapsed / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f80 (long double)",
        "data": "synthetic (seeded splitmix64; encoded by the reference's host codec)",
        "config": dict(config_of(args, world, desc, n_full), sample_values_per_format=m),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind_used,
                         "sample": f"{m} values per format per step ({len(streams)} formats), "
                                   f"host decode + compensated long-double DOT"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_of(args, world, desc, n_full):
    n = args.n or n_full
    if args.workload == "gemv":
        return {"workload": f"{desc}; {GEMV_ROWS} x {n // GEMV_ROWS} per GPU", "n_per_gpu": n,
                "rows": GEMV_ROWS, "columns": n // GEMV_ROWS,
                "formats": [f for f, _ in WORKLOADS[args.workload][1]],
                "layout": "dense", "accumulator": args.accum,
                "l2": "matrices larger than L2 (each > 126 MB); the vector is re-read from "
                      "L2 by every row",
                "parallelism": f"rows sharded x{world}, no collective"}
    return {"workload": f"{desc}; N={n} per GPU", "n_per_gpu": n,
            "formats": [f for f, _ in WORKLOADS[args.workload][1]],
            "layout": args.layout, "accumulator": args.accum,
            "l2": "inputs larger than L2 (every pair > 126 MB; consecutive DOTs read different buffers)",
            "parallelism": f"contiguous shards x{world}, one FP64 all-reduce per step"}


# ---- the other configurations (one GPU) -----------------------------------------
def run_per_config(ws, stream, threads, peak, reuse_refs):
    """Each configuration's DOT at its stated size with every accumulator and
    decoder: CUDA-event GB/s (inputs larger than L2 unless marked) and the
    normalised error against the reference's CPU DOT of the same codes."""
    import numpy as np
    import torch
    from accessor_universal_test_b200 import _lib, vectors

    def timed(fn, reps):
        """Mean launch time over back-to-back launches; at least `reps`
        launches and at least ~10 ms of device time, so that short DOTs are
        not timed over a few hundred microseconds."""
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(3):
            fn()
        b.record()
        torch.cuda.synchronize()
        reps = max(reps, min(1000, int(10.0 / max(a.elapsed_time(b) / 3, 1e-3))))
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    entries = []
    res = torch.zeros(1, dtype=torch.float64, device="cuda")
    for group, name, kind, layout, n, accums, decoders in PER_CONFIG:
        fid = _lib.format_id(name)
        ws.prepare(fid)
        fam, bits, _, _ = _lib.format_info(fid)
        x = vectors.encoded(ws, fid, layout, kind, SEED, 0, n)
        y = vectors.encoded(ws, fid, layout, kind, SEED, 1, n)
        torch.cuda.synchronize()
        stride = 64 if name == "fp64" else (bits if layout == DENSE else
                                            (8 if bits <= 8 else 16 if bits <= 16 else 32))
        key = (name, layout, kind, n)
        if key in reuse_refs:
            d, s = reuse_refs[key]
        else:
            d, s, _ = cpu_reference_dot(name, stride, x.cpu().numpy().view(np.uint32),
                                        y.cpu().numpy().view(np.uint32), n, threads)
        packed = 2 * n * bits / 8   # the reference's GB/s counts packed bits
        moved = 2 * n * stride / 8  # padded layouts move whole containers
        for acc in accums:
            acc_id = _lib.ACC_FP32 if acc == "fp32" else _lib.ACC_FP64
            for dec in decoders:
                def launch():
                    ws.dot(fid, layout, acc_id, x.data_ptr(), y.data_ptr(), n, res.data_ptr(),
                           stream, 0, DECODERS[dec])
                try:
                    t_ms = timed(launch, 20)
                except _lib.AutError:
                    continue  # no kernel for this decoder / accumulator
                got = float(res.cpu()[0])
                e = {"group": group, "format": name, "layout": "dense" if layout == DENSE
                     else "padded", "accumulator": acc, "decoder": dec, "n": n, "ms": t_ms,
                     "gbs": packed / (t_ms / 1e3) / 1e9,
                     "gbs_moved": moved / (t_ms / 1e3) / 1e9,
                     "frac_of_peak": moved / (t_ms / 1e3) / 1e9 / peak,
                     "normalized_error": normalized_error(got, d, s)}
                if group == "lns":
                    e["condition_number"] = condition_number(d, s)
                entries.append(e)
        del x, y
        torch.cuda.empty_cache()
    # GEMV over the same storage (1024 rows x 2^17 columns, the vector in the
    # same format): packed bytes = (rows * columns + columns) * bits / 8; the
    # error is the largest normalised error of three sampled rows
    rows, cols = GEMV_ROWS, 1 << 17
    for name, kind, layout, accs in GEMV_CONFIG:
        fid = _lib.format_id(name)
        ws.prepare(fid)
        fam, bits, _, _ = _lib.format_info(fid)
        m = vectors.encoded(ws, fid, layout, kind, SEED, 0, rows * cols)
        v = vectors.encoded(ws, fid, layout, kind, SEED, 1, cols)
        out = torch.zeros(rows, dtype=torch.float64, device="cuda")
        torch.cuda.synchronize()
        stride = bits if layout == DENSE else (8 if bits <= 8 else 16 if bits <= 16 else 32)
        row_bytes = cols * stride // 8
        mh = m.cpu().numpy()
        vw = v.cpu().numpy().view(np.uint32)
        refs = []
        for r in (0, rows // 2, rows - 1):
            seg = np.zeros(row_bytes + 16, dtype=np.uint8)
            avail = mh[r * row_bytes: r * row_bytes + row_bytes + 16]
            seg[:avail.size] = avail
            refs.append((r, cpu_reference_dot(name, stride, seg.view(np.uint32), vw, cols,
                                              threads)[:2]))
        packed = (rows * cols + cols) * bits / 8
        moved = (rows * cols + cols) * stride / 8
        for acc in accs:
            acc_id = _lib.ACC_FP32 if acc == "fp32" else _lib.ACC_FP64

            def launch():
                ws.gemv(fid, layout, acc_id, m.data_ptr(), v.data_ptr(), rows, cols,
                        out.data_ptr(), stream)
            t_ms = timed(launch, 20)
            got = out.cpu().numpy()
            err = max(normalized_error(got[r], d, s_) for r, (d, s_) in refs)
            entries.append({"group": "gemv", "format": name, "layout": "dense" if layout == DENSE
                            else "padded", "accumulator": acc, "decoder": "auto",
                            "n": rows * cols, "rows": rows, "columns": cols, "ms": t_ms,
                            "gbs": packed / (t_ms / 1e3) / 1e9,
                            "gbs_moved": moved / (t_ms / 1e3) / 1e9,
                            "frac_of_peak": moved / (t_ms / 1e3) / 1e9 / peak,
                            "normalized_error": err})
        del m, v, out
        torch.cuda.empty_cache()
    if ws.status() != 0:
        raise RuntimeError("a bounded device wait timed out during the configurations")

    # the raw FP32/FP64 size sweep, 2^10 to 2^27: launch-bound to HBM-bound (small sizes stay in L2)
    sweep = []
    for name, kind, acc in (("fp32", 1, _lib.ACC_FP32), ("fp64", 0, _lib.ACC_FP64)):
        fid = _lib.format_id(name)
        bits = 64 if name == "fp64" else 32
        for p in RAW_SWEEP:
            n = 1 << p
            x = vectors.encoded(ws, fid, DENSE, kind, SEED, 0, n)
            y = vectors.encoded(ws, fid, DENSE, kind, SEED, 1, n)

            def launch():
                ws.dot(fid, DENSE, acc, x.data_ptr(), y.data_ptr(), n, res.data_ptr(), stream)
            t_ms = timed(launch, 200 if p <= 23 else 20)
            sweep.append({"format": name, "n": n, "ms": t_ms,
                          "gbs": 2 * n * bits / 8 / (t_ms / 1e3) / 1e9,
                          "l2_resident": 2 * n * bits / 8 < 126e6})
            del x, y
    torch.cuda.empty_cache()
    return entries, sweep


# ---- our arm ---------------------------------------------------------------------
def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import numpy as np
    import torch
    import torch.distributed as dist
    from accessor_universal_test_b200 import _lib, vectors
    from accessor_universal_test_b200.sharded import allreduce_partials, allreduce_partials_async

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    desc, fmts, layout, n_full = WORKLOADS[args.workload]
    if args.layout == "padded" and args.workload != "gemv":
        layout = PADDED
    n = args.n or n_full
    accum = _lib.ACC_FP32 if args.accum == "fp32" else _lib.ACC_FP64
    if any(f == "fp64" for f, _ in fmts):
        accum = _lib.ACC_FP64
    ws = _lib.Workspace(local)
    strategy = {"auto": 0, "ldg": 1, "tma": 2}[args.strategy]
    stream = torch.cuda.current_stream().cuda_stream
    gemv = args.workload == "gemv"
    rows = GEMV_ROWS if gemv else 1      # results per format
    cols = n // rows                     # values per DOT
    fids, inputs, packed_bytes = [], [], []
    for name, kind in fmts:
        fid = _lib.format_id(name)
        ws.prepare(fid)
        x = vectors.encoded(ws, fid, layout, kind, SEED, 0, rows * cols, first=rank * rows * cols)
        if gemv:  # the same vector on every GPU
            y = vectors.encoded(ws, fid, layout, kind, SEED, 1, cols)
        else:
            y = vectors.encoded(ws, fid, layout, kind, SEED, 1, n, first=rank * n)
        fids.append(fid)
        inputs.append((x, y))
        values = (rows * cols + cols) if gemv else 2 * n
        packed_bytes.append(values * _lib.format_info(fid)[1] / 8)
    # two result buffers: a timed step's all-reduce overlaps the next step
    results2 = torch.zeros(2, len(fmts) * rows, dtype=torch.float64, device="cuda")
    results = results2[0]
    res_ptr = results.data_ptr()
    torch.cuda.synchronize()

    def launch(k, strat, dec=0, out=None):
        x, y = inputs[k]
        base = res_ptr if out is None else out
        if gemv:
            ws.gemv(fids[k], layout, accum, x.data_ptr(), y.data_ptr(), rows, cols,
                    base + 8 * rows * k, stream, strat, dec)
        else:
            ws.dot(fids[k], layout, accum, x.data_ptr(), y.data_ptr(), n, base + 8 * k,
                   stream, strat, dec)

    # On N > 1 GPUs each step's all-reduce of its partials runs on NCCL's
    # stream while the next step's DOTs run; a step reusing a result buffer
    # first makes the stream wait for the all-reduce that last used it, and
    # drain() makes it wait for all of them, so every timed step is complete
    # (kernels and collective) before the stop event.
    pending = [None, None]
    steps_run = [0]

    def step():
        b = steps_run[0] & 1
        steps_run[0] += 1
        if pending[b] is not None:
            pending[b].wait()
            pending[b] = None
        out = results2[b]
        for k in range(len(fids)):
            launch(k, strategy, out=out.data_ptr())
        if world > 1 and not gemv:
            pending[b] = allreduce_partials_async(out)

    def drain():
        for b in (0, 1):
            if pending[b] is not None:
                pending[b].wait()
                pending[b] = None

    for _ in range(args.warmup):
        step()
    drain()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The clock sampler is running before the ranks meet; the ranks then
    # leave a barrier together, and on N > 1 GPUs the start event is recorded
    # behind one more all-reduce, so that every GPU's timed region opens when
    # that collective completes (within microseconds on all ranks) instead of
    # whenever its host gets there.
    sync = torch.zeros(1, dtype=torch.float64, device="cuda")
    with ClockSampler(physical_gpu(local)) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if world > 1:
            dist.all_reduce(sync)
        clocks.mark()
        start.record()
        for _ in range(args.steps):
            step()
        drain()
        stop.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    rank_ms = [ms]
    allreduce_us = None
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        rank_ms = [float(g.item()) for g in gathered]
        ms = max(rank_ms)
        # the collective alone: one all-reduce of one step's partials
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(5):
            allreduce_partials(results2[0])
        torch.cuda.synchronize()
        dist.barrier()
        a.record()
        for _ in range(50):
            allreduce_partials(results2[0])
        b.record()
        torch.cuda.synchronize()
        allreduce_us = a.elapsed_time(b) / 50 * 1e3
    step_bytes = sum(packed_bytes) * world
    value = step_bytes * args.steps / (ms / 1e3) / 1e9
    elems = 2 * n * len(fmts) * world * args.steps / (ms / 1e3)

    # per-kernel CUDA-event timing (same stream) for the roofline, for the
    # strategy in use and for each explicit access strategy
    reps = 50

    def time_kernel(k, strat, dec=0):
        launch(k, strat, dec)  # untimed: first-use set-up of this variant
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            launch(k, strat, dec)
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    per_kernel, by_strategy, by_decoder = [], {}, {}
    for k, fid in enumerate(fids):
        t_ms = time_kernel(k, strategy)
        per_kernel.append((fmts[k][0], t_ms, packed_bytes[k] / (t_ms / 1e3) / 1e9))
        by_strategy[fmts[k][0]] = {name: packed_bytes[k] / (time_kernel(k, s) / 1e3) / 1e9
                                   for name, s in (("ldg", 1), ("tma", 2))}
        # every decoder this format/accumulator has, each with both strategies
        table = {}
        for dname, dec in DECODERS.items():
            if dname == "auto":
                continue
            for sname, s in (("ldg", 1), ("tma", 2)):
                try:
                    table[f"{dname}/{sname}"] = packed_bytes[k] / (time_kernel(k, s, dec) / 1e3) / 1e9
                except _lib.AutError:
                    pass
        by_decoder[fmts[k][0]] = table
    if ws.status() != 0:
        raise RuntimeError("a bounded device wait timed out during the benchmark")
    peak, peak_kind = measured_peak()
    dom = max(per_kernel, key=lambda r: r[1])
    # an FP32 GEMV of these formats whose columns are whole 16384-value
    # segments runs two kernels (the streaming kernel and the row sums)
    launches_per_call = (2 if gemv and accum == _lib.ACC_FP32 and args.strategy != "ldg"
                         and cols % 16384 == 0 else 1)
    traffic = committed_traffic().get(f"gemv:{dom[0]}" if gemv else dom[0])
    if traffic is not None and "bytes_per_value_pair" in traffic:
        traffic = traffic["bytes_per_value_pair"] * n
    elif traffic is not None and "captured_columns" in traffic:  # GEMV, scaled to this shape
        cr, cc = traffic["captured_rows"], traffic["captured_columns"]
        traffic = traffic["bytes_per_launch"] * (rows * cols + cols) / (cr * cc + cc)
    elif traffic is not None:
        traffic = traffic.get("bytes_per_launch")

    # e2e through the C ABI from pinned host buffers
    host_in = [(x.cpu().pin_memory(), y.cpu().pin_memory()) for x, y in inputs]
    host_out = torch.zeros(len(fmts) * rows, dtype=torch.float64).pin_memory()
    h2d = sum(hx.numel() + hy.numel() for hx, hy in host_in)

    def e2e_step():
        for k in range(len(fids)):
            x, y = inputs[k]
            x.copy_(host_in[k][0], non_blocking=True)
            y.copy_(host_in[k][1], non_blocking=True)
            launch(k, strategy)
        if world > 1 and not gemv:
            allreduce_partials(results)
        host_out.copy_(results, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.all_reduce(sync)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    b.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = step_bytes / (e2e_ms / 1e3) / 1e9

    # CPU baseline + normalised error (rank 0 at N=1): the reference's CPU path
    # over the full workload on all host cores.
    cpu_baseline, errors, refs = None, {}, {}
    gpu_results = host_out.numpy().copy()
    threads = host_threads()
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        tot_bytes, tot_s, kinds = 0.0, 0.0, set()
        sample_rows = 16 if gemv else 1
        for k, (name, gen_kind) in enumerate(fmts):
            x, y = inputs[k]
            xw = x.cpu().numpy().view(np.uint32)
            yw = y.cpu().numpy().view(np.uint32)
            bits = _lib.format_info(fids[k])[1]
            stride = 64 if name == "fp64" else (
                bits if layout == DENSE else (8 if bits <= 8 else 16 if bits <= 16 else 32))
            row_words = cols * stride // 32
            worst = 0.0
            for r in range(sample_rows):
                t0 = time.perf_counter()
                d, s, kind = cpu_reference_dot(name, stride, xw[r * row_words:], yw, cols,
                                               threads)
                tot_s += time.perf_counter() - t0
                tot_bytes += (2 * cols if not gemv else cols + cols / sample_rows) * bits / 8
                kinds.add(kind)
                if not gemv:
                    refs[(name, layout, gen_kind, n)] = (d, s)
                worst = max(worst, normalized_error(gpu_results[k * rows + r], d, s))
            errors[name] = worst
        what = (f"{sample_rows} rows of each of the {len(fmts)} matrices ({cols} columns)"
                if gemv else f"the full workload ({len(fmts)} DOTs x {n} values)")
        cpu_baseline = {"value": tot_bytes / tot_s / 1e9, "unit": "GB/s", "cores": threads,
                        "kind": "reference" if kinds == {"reference"} else "port",
                        "sample": what + ", host decode + compensated long-double DOT"}

    per_config, raw_sweep = None, None
    if world == 1 and not args.no_per_config and args.n == 0:
        per_config, raw_sweep = run_per_config(ws, stream, threads, peak, refs)

    clk = clocks.summary()
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": ("fp32 FMA chains of <= 32 products with fp64 carries (e8m15: fp64)"
                  if accum == _lib.ACC_FP32 else "fp64"),
        "data": "synthetic (seeded splitmix64, generated and encoded on the GPU)",
        "config": config_of(args, world, desc, n_full),
        "decoded_elems_per_s": elems,
        "pct_of_8tbs": value / world / 8000.0 * 100.0,
        "per_format": [{"format": f, "ms": t, "gbs": g, "frac_of_peak": g / peak,
                        "gbs_by_strategy": by_strategy[f],
                        "gbs_by_decoder": by_decoder[f]}
                       for f, t, g in per_kernel],
        "strategy": args.strategy,
        "normalized_error": errors or None,
        "roofline": {"bound": "hbm", "kernel": f"{'gemv' if gemv else 'dot'}_kernel[{dom[0]}]",
                     "achieved": dom[2],
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                     "frac": dom[2] / peak, "traffic": traffic},
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 8 * len(fmts) * rows},
        "gpu_launches": len(fmts) * args.steps * launches_per_call,
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                   "reasons": clk["reasons"]},
    }
    if world > 1:
        line["multi_gpu"] = {"rank_ms": rank_ms, "allreduce_us": allreduce_us,
                             "allreduce_share_of_step": (allreduce_us / 1e3) / (ms / args.steps),
                             "collectives_per_step": 0 if gemv else 1}
    if per_config is not None:
        line["per_config"] = per_config
        line["raw_sweep"] = raw_sweep
    if rank == 0:
        print(json.dumps(line), flush=True)
    ws.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

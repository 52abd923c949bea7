"""The command-line tools keep the reference's flags and CSV schemas.

strategy_bench output is checked with the acceptance rule of the reference's
smoke validators (tools/validate_bitwidth_strategy_smoke.py:43-69,
tools/validate_lns_strategy_smoke.py:40-60): every strategy of a (format,
arithmetic, distribution, kernel, N) group agrees with the scalar baseline
row within 5e-3 (FP32) / 1e-9 (FP64; 2e-4 for LNS) relative to
max(|baseline|, 1).  dot_bench output carries the reference's header and
the accuracy columns.
"""
import csv
import math
import os
import subprocess
from collections import defaultdict

import pytest

from conftest import ROOT

LIB = os.path.join(ROOT, "accessor_universal_test_b200", "lib")

BITWIDTH_HEADER = (
    "timestamp,gpu,mode,distribution,kernel,format,bits,exponent_bits,mantissa_bits,"
    "arithmetic_type,storage_layout,access_method,packet_values,load_word_bits,"
    "loader_threads,consumer_threads,values_per_consumer,redistribution,decoder,"
    "strategy_id,N,M,rows,logical_input_bytes,physical_input_bytes,table_bytes,blocks,"
    "threads,warmup,sample,iterations,total_ms,mean_ms,result,valid")
LNS_HEADER = (
    "timestamp,gpu,mode,distribution,kernel,number_family,format,bits,log_integer_bits,"
    "log_fraction_bits,arithmetic_type,multiply_method,storage_layout,access_method,"
    "packet_values,load_word_bits,loader_threads,consumer_threads,values_per_consumer,"
    "redistribution,decoder,strategy_id,N,M,rows,logical_input_bytes,physical_input_bytes,"
    "table_bytes,blocks,threads,warmup,sample,iterations,total_ms,mean_ms,result,valid")
DOT_BENCH_HEADER = (
    "gpu,compute_capability,cuda_runtime,cuda_driver,cublas_version,mode,dataset,operation,"
    "input_type,n,algorithmic_bytes,algorithmic_flops,arithmetic_intensity_flop_per_byte,"
    "iterations,samples,min_ms,median_ms,p10_ms,p90_ms,coefficient_of_variation,"
    "giga_elements_per_s,algorithmic_gb_per_s,gflop_per_s,result,reference,absolute_error,"
    "relative_error,normalized_error,dot_condition_number")


def test_tools_are_built_and_answer_help(autlib):
    from accessor_universal_test_b200 import build
    build.build_tools()
    for tool in ("strategy_bench", "dot_bench", "accessor_dot_bench"):
        r = subprocess.run([os.path.join(LIB, tool), "--help"], capture_output=True, text=True)
        assert r.returncode == 0 and "--output" in r.stdout


def _validate(rows, lns):
    groups = defaultdict(dict)
    for row in rows:
        assert row["valid"] == "1", row
        key = (row["format"], row["arithmetic_type"], row["distribution"], row["kernel"], row["N"])
        groups[key][(row["strategy_id"], row["decoder"], row["storage_layout"])] = float(row["result"])
    assert groups
    for key, strategies in groups.items():
        if lns:
            base = [v for (sid, dec, lay), v in strategies.items()
                    if dec == "reference_exp2" and lay == "padded"]
            tol = 5e-3 if key[1] == "fp32" else 2e-4
        else:
            base = [v for (sid, dec, lay), v in strategies.items()
                    if sid == "padded/scalar/x1/generic"]
            tol = 5e-3 if key[1] == "fp32" else 1e-9
        assert base, key
        scale = max(abs(base[0]), 1.0)
        for (sid, _, _), v in strategies.items():
            assert math.isfinite(v) and abs(v - base[0]) / scale <= tol, (key, sid, v, base[0])


@pytest.mark.gpu
@pytest.mark.parametrize("family", ["bitwidth", "lns"])
def test_strategy_bench_smoke_passes_the_reference_validator_rule(tmp_path, autlib, family):
    from accessor_universal_test_b200 import build
    build.build_tools()
    out = tmp_path / f"{family}.csv"
    r = subprocess.run([os.path.join(LIB, "strategy_bench"), "--family", family, "--mode",
                        "smoke", "--output", str(out)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    lines = out.read_text().splitlines()
    assert lines[0] == (LNS_HEADER if family == "lns" else BITWIDTH_HEADER)
    rows = list(csv.DictReader(lines))
    strategies = {row["access_method"] for row in rows}
    expected = {"scalar", "thread_packet", "tma_bulk"}
    if family == "bitwidth":  # dense E8 / e2m3 streams also take the shuffle loader
        expected.add("cooperative_shuffle")
    assert strategies == expected
    _validate(rows, family == "lns")


@pytest.mark.gpu
def test_dot_bench_accuracy_rows(tmp_path, autlib):
    from accessor_universal_test_b200 import build
    build.build_tools()
    out = tmp_path / "dot.csv"
    r = subprocess.run([os.path.join(LIB, "dot_bench"), "--mode", "accuracy", "--powers",
                        "10,16,20", "--output", str(out)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    lines = out.read_text().splitlines()
    assert lines[0] == DOT_BENCH_HEADER
    rows = list(csv.DictReader(lines))
    ops = {(row["operation"], row["input_type"]) for row in rows}
    assert {("cublasSdot", "float32"), ("cublasDdot", "float64"), ("aut_dot_acc32", "float32"),
            ("aut_dot_acc64", "float32"), ("aut_dot_acc64", "float64")} <= ops
    for row in rows:
        err = float(row["normalized_error"])
        if row["operation"] == "aut_dot_acc64":
            assert err <= 1e-14, row
        if row["operation"] == "aut_dot_acc32":
            assert err <= 2e-6, row


ACCESSOR_ACCURACY_HEADER = (
    "gpu,compute_capability,multiprocessors,cuda_runtime,cuda_driver,"
    "dataset,variant,storage_type,arithmetic_type,access_kind,n,blocks,"
    "threads,result,result_bits,reference,absolute_error,relative_error,"
    "normalized_error,dot_condition_number,x_fingerprint,"
    "y_fingerprint,finite")


@pytest.mark.gpu
def test_accessor_dot_bench_accuracy_rows_match_the_golden_dataset(autlib, tmp_path):
    """accessor_dot_bench --mode accuracy: the reference's schema, the dot_v1
    fingerprints and reference DOTs of the reference's inspector (golden CSV),
    and errors no worse than those the reference's own kernels published."""
    from conftest import GOLDEN
    out = tmp_path / "accuracy.csv"
    r = subprocess.run([os.path.join(LIB, "accessor_dot_bench"), "--mode", "accuracy",
                        "--warmup", "1", "--output", str(out)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    text = out.read_text().splitlines()
    assert text[0] == ACCESSOR_ACCURACY_HEADER
    rows = list(csv.DictReader(text))
    assert len(rows) == 9 * 3 * 4
    with open(os.path.join(GOLDEN, "dot_v1_inspect.csv")) as f:
        golden = {(g["dataset"], g["n"]): g for g in csv.DictReader(f)}
    with open(os.path.join(GOLDEN, "accessor_dot_accuracy.csv")) as f:
        published = {(g["dataset"], g["n"]): g for g in csv.DictReader(f)}
    for row in rows:
        g = golden[(row["dataset"], row["n"])]
        assert row["x_fingerprint"] == g["x_fingerprint"]
        assert row["y_fingerprint"] == g["y_fingerprint"]
        assert abs(float(row["reference"]) - float(g["dot_reference"])) <= \
            1e-15 * max(1.0, abs(float(g["dot_reference"])))
        assert row["finite"] == "true"
        theirs = float(published[(row["dataset"], row["n"])][
            f"{row['variant']}_normalized_error"])
        assert float(row["normalized_error"]) <= theirs * (1 + 1e-9) + 1e-300, row


@pytest.mark.gpu
def test_device_dot_v1_generator_matches_the_golden_fingerprints(autlib):
    import numpy as np
    import torch
    from conftest import GOLDEN
    from accessor_universal_test_b200 import _lib
    cases = {"positive_uniform": (0, 0x123456789ABCDEF0, 0),
             "signed_uniform_seed0": (1, 0x123456789ABCDEF0, 0),
             "cancellation_1e6": (2, 0x123456789ABCDEF0, 19),
             "dynamic_range_40": (3, 0xA4093822299F31D0, 20)}
    with open(os.path.join(GOLDEN, "dot_v1_inspect.csv")) as f:
        golden = list(csv.DictReader(f))

    def fnv(a):
        h = 1469598103934665603
        for w in a.view(np.uint32).tolist():
            h = ((h ^ w) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        return f"0x{h:x}"
    for g in golden:
        if g["dataset"] not in cases or int(g["n"]) > 65536:
            continue
        fam, seed, param = cases[g["dataset"]]
        n = int(g["n"])
        for vid, key in ((0, "x_fingerprint"), (1, "y_fingerprint")):
            out = torch.empty(n, dtype=torch.float32, device="cuda")
            # two halves generated separately: `first` indexes into the case
            _lib.generate_dot_v1(fam, seed, param, vid, n, out.data_ptr(), 0, n // 2)
            _lib.generate_dot_v1(fam, seed, param, vid, n, out.data_ptr() + 4 * (n // 2),
                                 n // 2, n - n // 2)
            torch.cuda.synchronize()
            assert fnv(out.cpu().numpy()) == g[key], (g["dataset"], n, vid)

"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Run here, where the reference tree exists (it is compiled into
oracle/_ref/ by oracle/Makefile):

    python tests/golden/make_golden.py

Fixtures written (all small, all produced by the reference's own code):
  dot_v1_inspect.csv  -- tools/inspect_dot_dataset.cpp's CSV for
                         N = 1024, 65536, 1048576 (fingerprints, reference
                         DOT, condition numbers of the dot_v1 cases).
  codec_vectors.json  -- for the DOT formats: sampled codes with the
                         reference's FP64/FP32 decode bits, and doubles with
                         the reference's encode (storage::encode/lns::encode).
  dot_vectors.json    -- reference CPU DOTs (host decode + compensated long
                         double sum) of the synthetic workloads at small N,
                         with an FNV-1a fingerprint of each packed stream.
  accessor_dot_accuracy.csv
                      -- the normalised errors the reference's own GPU
                         kernels reached on the dot_v1 cases (FP32 storage,
                         FP32 / FP64 accumulation; raw and accessor DOT),
                         copied from its published run
                         results/003_accessor_dot/run_20260723T150439Z/
                         accuracy_comparison.csv (H200, sm_90).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle  # noqa: E402

DOT_FORMATS = ["e2m3", "e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7", "e8m15",
               "lns8_r3", "lns16_r11"]
# (generator kind, vector ids) of each workload: kind 0 = signed uniform
# double, 2 = Irwin-Hall normal, 3 = LNS cancellation pair.
WORKLOAD = {"e2m3": 2, "lns8_r3": 3, "lns16_r11": 3}
SEED = 0x243F6A8885A308D3
SIZES = [1, 7, 4099, 65536 + 13]


def fnv_words(words: np.ndarray) -> str:
    h = 1469598103934665603
    for w in words.astype(np.uint64).tolist():
        h ^= w
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"0x{h:016x}"


def main() -> None:
    if not pyoracle.build_reference():
        raise SystemExit("reference tree not found; fixtures need the reference")
    ref = pyoracle.reference()
    orc = pyoracle.oracle()

    # 1. dot_v1 statistics from the reference's own inspector.
    exe = os.path.join(ROOT, "oracle", "_ref", "dataset_inspect")
    csv = subprocess.run([exe, "1024", "65536", "1048576"], check=True,
                         capture_output=True, text=True).stdout
    with open(os.path.join(HERE, "dot_v1_inspect.csv"), "w") as f:
        f.write(csv)

    # 2. codec vectors.
    rng = np.random.default_rng(20260801)
    codec = {}
    for name in DOT_FORMATS:
        fam, bits, ebits, fin = ref.desc(name)
        allc = np.arange(1 << bits, dtype=np.uint32)
        special = allc[[0, 1, (1 << bits) - 1, 1 << (bits - 1), (1 << (bits - 1)) - 1,
                        (1 << (bits - 2)), (1 << (bits - 2)) | (1 << (bits - 1))]]
        sample = allc if allc.size <= 256 else rng.choice(allc, 200, replace=False)
        codes = np.unique(np.concatenate([special, sample]))
        d64 = ref.decode_f64(name, codes)
        d32 = ref.decode_f32(name, codes)
        finite = np.sort(d64[np.isfinite(d64)])
        mids = (finite[:-1] + finite[1:]) / 2
        vals = np.concatenate([
            mids[rng.choice(mids.size, min(64, mids.size), replace=False)],
            rng.standard_normal(64) * 3.0, rng.uniform(-1, 1, 64),
            np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e300, -1e300, 1e-300]),
        ])
        enc = ref.encode(name, vals)
        codec[name] = {
            "family": fam, "total_bits": bits, "exponent_bits": ebits, "finite": fin,
            "codes": codes.tolist(),
            "decode_f64_bits": [f"0x{b:016x}" for b in d64.view(np.uint64).tolist()],
            "decode_f32_bits": [f"0x{b:08x}" for b in d32.view(np.uint32).tolist()],
            "encode_inputs_bits": [f"0x{b:016x}" for b in vals.view(np.uint64).tolist()],
            "encode_codes": enc.tolist(),
        }
    with open(os.path.join(HERE, "codec_vectors.json"), "w") as f:
        json.dump(codec, f, indent=0)

    # 3. reference CPU DOTs of the synthetic workloads.
    dots = {"seed": SEED, "cases": []}
    for name in DOT_FORMATS:
        fam, bits, ebits, fin = ref.desc(name)
        kind = WORKLOAD.get(name, 0)
        for n in SIZES:
            x = orc.synthetic(kind, SEED, 0, n)
            y = orc.synthetic(kind, SEED, 1, n)
            xw = ref.pack_dense(bits, ref.encode(name, x))
            yw = ref.pack_dense(bits, ref.encode(name, y))
            d, s = ref.dot_dense(name, bits, xw, yw, n, threads=1)
            dots["cases"].append({
                "format": name, "kind": kind, "n": n,
                "x_words_fnv": fnv_words(xw), "y_words_fnv": fnv_words(yw),
                "dot_hi": d[0], "dot_lo": d[1], "sum_abs_hi": s[0], "sum_abs_lo": s[1],
            })
    for n in SIZES:  # raw FP32 storage, dot_v1-style signed floats
        x = orc.synthetic(1, SEED, 0, n).astype(np.float32)
        y = orc.synthetic(1, SEED, 1, n).astype(np.float32)
        d, s = ref.dot_raw(x, y)
        dots["cases"].append({"format": "fp32", "kind": 1, "n": n,
                              "dot_hi": d[0], "dot_lo": d[1],
                              "sum_abs_hi": s[0], "sum_abs_lo": s[1]})
        xd = orc.synthetic(0, SEED, 0, n)
        yd = orc.synthetic(0, SEED, 1, n)
        d, s = ref.dot_raw(xd, yd)
        dots["cases"].append({"format": "fp64", "kind": 0, "n": n,
                              "dot_hi": d[0], "dot_lo": d[1],
                              "sum_abs_hi": s[0], "sum_abs_lo": s[1]})
    with open(os.path.join(HERE, "dot_vectors.json"), "w") as f:
        json.dump(dots, f, indent=1)

    # 4. the reference GPU kernels' published normalised errors on dot_v1.
    import csv as _csv
    src = os.path.join(pyoracle.REF_TREE, "results", "003_accessor_dot",
                       "run_20260723T150439Z", "accuracy_comparison.csv")
    keep = ["dataset", "n", "dot_condition_number", "raw_f32_normalized_error",
            "accessor_f32_f32_normalized_error", "raw_f64_normalized_error",
            "accessor_f64_f32_normalized_error"]
    with open(src) as f:
        rows = list(_csv.DictReader(f))
    with open(os.path.join(HERE, "accessor_dot_accuracy.csv"), "w") as f:
        f.write(",".join(keep) + "\n")
        for r in rows:
            f.write(",".join(r[k] for k in keep) + "\n")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()

"""ctypes access to the oracle libraries.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's cpu_baseline / reference legs.  The product
never imports this module.

* ``Oracle``   -- oracle/_build/liboracle.so, the C restatement (oracle.c).
* ``Reference``-- oracle/_ref/libautref.so, the reference's own headers
  behind ref_shim.cpp.  Built here only when the reference tree is present;
  on a machine without it, ``reference()`` returns None.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libautref.so")
REFGPU_SO = os.path.join(HERE, "_ref", "librefgpu.so")
REF_TREE = os.environ.get("AUT_REFERENCE_TREE", "/root/reference")

FAMILY_BINARY, FAMILY_PREFIX, FAMILY_LNS, FAMILY_RAW_FP32, FAMILY_RAW_FP64 = range(5)

_lock = threading.Lock()
_oracle = None
_reference = None
_reference_tried = False

_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_d2 = C.c_double * 2


def build_oracle() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)


def build_reference() -> bool:
    """Compile oracle/_ref from the reference tree; False when it is absent."""
    if not os.path.isdir(os.path.join(REF_TREE, "include")):
        return False
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF_TREE}"], check=True)
    return True


def _ld_pair(p) -> float:
    return (float(p[0]), float(p[1]))


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build_oracle()
        lib = C.CDLL(path)
        self.lib = lib
        i, u32, u64, d, f = C.c_int, C.c_uint32, C.c_uint64, C.c_double, C.c_float
        lib.orc_encode.restype = u32
        lib.orc_encode.argtypes = [i, i, i, i, d]
        lib.orc_decode_f64.restype = d
        lib.orc_decode_f64.argtypes = [i, i, i, i, u32]
        lib.orc_decode_f32.restype = f
        lib.orc_decode_f32.argtypes = [i, i, i, i, u32]
        lib.orc_encode_array.argtypes = [i, i, i, i, _f64p, u64, _u32p]
        lib.orc_decode_array_f64.argtypes = [i, i, i, i, _u32p, u64, _f64p]
        lib.orc_decode_array_f32.argtypes = [i, i, i, i, _u32p, u64, _f32p]
        lib.orc_dense_word_count.restype = u64
        lib.orc_dense_word_count.argtypes = [i, u64]
        lib.orc_dense_data_bytes.restype = u64
        lib.orc_dense_data_bytes.argtypes = [i, u64]
        lib.orc_load_dense.restype = u32
        lib.orc_load_dense.argtypes = [i, _u32p, u64]
        lib.orc_pack_dense.argtypes = [i, _u32p, u64, _u32p]
        lib.orc_unpack_dense.argtypes = [i, _u32p, u64, _u32p]
        lib.orc_splitmix64.restype = u64
        lib.orc_splitmix64.argtypes = [u64]
        lib.orc_dot_v1_value.restype = f
        lib.orc_dot_v1_value.argtypes = [i, u64, i, i, u64, u64]
        lib.orc_dot_v1_fill.argtypes = [i, u64, i, i, u64, _f32p]
        lib.orc_fnv1a_f32.restype = u64
        lib.orc_fnv1a_f32.argtypes = [_f32p, u64]
        lib.orc_synthetic_value.restype = d
        lib.orc_synthetic_value.argtypes = [i, u64, i, u64]
        lib.orc_synthetic_fill.argtypes = [i, u64, i, u64, u64, _f64p]
        lib.orc_dot_reference_f64.argtypes = [_f64p, _f64p, u64, _d2, _d2]
        lib.orc_dot_reference_f32.argtypes = [_f32p, _f32p, u64, _d2, _d2]
        lib.orc_dot_codes.argtypes = [i, i, i, i, _u32p, _u32p, u64, i, _d2, _d2]
        lib.orc_dot_dense.argtypes = [i, i, i, i, i, _u32p, _u32p, u64, i, _d2, _d2]

    # -- codecs -------------------------------------------------------------
    def encode(self, fmt, values) -> np.ndarray:
        v = np.ascontiguousarray(values, dtype=np.float64)
        out = np.empty(v.size, np.uint32)
        self.lib.orc_encode_array(*fmt, v, v.size, out)
        return out

    def decode_f64(self, fmt, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        out = np.empty(c.size, np.float64)
        self.lib.orc_decode_array_f64(*fmt, c, c.size, out)
        return out

    def decode_f32(self, fmt, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        out = np.empty(c.size, np.float32)
        self.lib.orc_decode_array_f32(*fmt, c, c.size, out)
        return out

    # -- dense bitstream ----------------------------------------------------
    def dense_word_count(self, bits: int, n: int) -> int:
        return int(self.lib.orc_dense_word_count(bits, n))

    def pack_dense(self, bits: int, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        out = np.empty(self.dense_word_count(bits, c.size), np.uint32)
        self.lib.orc_pack_dense(bits, c, c.size, out)
        return out

    def unpack_dense(self, bits: int, words, n: int) -> np.ndarray:
        w = np.ascontiguousarray(words, dtype=np.uint32)
        out = np.empty(n, np.uint32)
        self.lib.orc_unpack_dense(bits, w, n, out)
        return out

    # -- datasets -----------------------------------------------------------
    def dot_v1(self, kind: int, seed: int, parameter: int, vector_id: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.orc_dot_v1_fill(kind, seed, parameter, vector_id, n, out)
        return out

    def fnv1a(self, values) -> int:
        v = np.ascontiguousarray(values, dtype=np.float32)
        return int(self.lib.orc_fnv1a_f32(v, v.size))

    def synthetic(self, kind: int, seed: int, vector_id: int, n: int, first: int = 0) -> np.ndarray:
        out = np.empty(n, np.float64)
        self.lib.orc_synthetic_fill(kind, seed, vector_id, first, n, out)
        return out

    # -- compensated reference ---------------------------------------------
    def dot_reference(self, x, y):
        """(dot, sum_abs) as (hi, lo) pairs of the long-double results."""
        d, s = _d2(), _d2()
        if np.asarray(x).dtype == np.float32:
            xs = np.ascontiguousarray(x, np.float32)
            ys = np.ascontiguousarray(y, np.float32)
            self.lib.orc_dot_reference_f32(xs, ys, xs.size, d, s)
        else:
            xs = np.ascontiguousarray(x, np.float64)
            ys = np.ascontiguousarray(y, np.float64)
            self.lib.orc_dot_reference_f64(xs, ys, xs.size, d, s)
        return _ld_pair(d), _ld_pair(s)

    def dot_codes(self, fmt, x_codes, y_codes, threads: int = 1):
        x = np.ascontiguousarray(x_codes, np.uint32)
        y = np.ascontiguousarray(y_codes, np.uint32)
        d, s = _d2(), _d2()
        self.lib.orc_dot_codes(*fmt, x, y, x.size, threads, d, s)
        return _ld_pair(d), _ld_pair(s)

    def dot_dense(self, fmt, stride_bits: int, x_words, y_words, n: int, threads: int = 1):
        x = np.ascontiguousarray(x_words).view(np.uint32)
        y = np.ascontiguousarray(y_words).view(np.uint32)
        d, s = _d2(), _d2()
        self.lib.orc_dot_dense(*fmt, stride_bits, x, y, n, threads, d, s)
        return _ld_pair(d), _ld_pair(s)


class Reference:
    """The reference's own host code (oracle/_ref/libautref.so)."""

    def __init__(self, path: str = REF_SO):
        lib = C.CDLL(path)
        self.lib = lib
        i, u32, u64, d, f = C.c_int, C.c_uint32, C.c_uint64, C.c_double, C.c_float
        lib.autref_format_count.restype = i
        lib.autref_format_name.restype = C.c_char_p
        lib.autref_format_name.argtypes = [i]
        ip = C.POINTER(C.c_int)
        lib.autref_format_desc.argtypes = [i, ip, ip, ip, ip]
        lib.autref_encode_array.argtypes = [i, _f64p, u64, _u32p]
        lib.autref_decode_array_f64.argtypes = [i, _u32p, u64, _f64p]
        lib.autref_decode_array_f32.argtypes = [i, _u32p, u64, _f32p]
        lib.autref_dense_word_count.restype = u64
        lib.autref_dense_word_count.argtypes = [i, u64]
        lib.autref_pack_dense.argtypes = [i, _u32p, u64, _u32p, u64]
        lib.autref_load_dense.restype = u32
        lib.autref_load_dense.argtypes = [i, _u32p, u64]
        lib.autref_dot_v1_case_count.restype = i
        lib.autref_dot_v1_case_id.restype = C.c_char_p
        lib.autref_dot_v1_case_id.argtypes = [i]
        lib.autref_dot_v1_fill.argtypes = [i, i, u64, _f32p]
        lib.autref_dot_dense.argtypes = [i, i, _u32p, _u32p, u64, i, _d2, _d2]
        lib.autref_dot_raw.argtypes = [i, C.c_void_p, C.c_void_p, u64, i, _d2, _d2]
        self.formats = {}
        for k in range(lib.autref_format_count()):
            fam, t, e, fin = C.c_int(), C.c_int(), C.c_int(), C.c_int()
            lib.autref_format_desc(k, C.byref(fam), C.byref(t), C.byref(e), C.byref(fin))
            name = lib.autref_format_name(k).decode()
            self.formats[name] = (k, (fam.value, t.value, e.value, fin.value))

    def index(self, name: str) -> int:
        return self.formats[name][0]

    def desc(self, name: str):
        return self.formats[name][1]

    def encode(self, name: str, values) -> np.ndarray:
        v = np.ascontiguousarray(values, dtype=np.float64)
        out = np.empty(v.size, np.uint32)
        self.lib.autref_encode_array(self.index(name), v, v.size, out)
        return out

    def decode_f64(self, name: str, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        out = np.empty(c.size, np.float64)
        self.lib.autref_decode_array_f64(self.index(name), c, c.size, out)
        return out

    def decode_f32(self, name: str, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        out = np.empty(c.size, np.float32)
        self.lib.autref_decode_array_f32(self.index(name), c, c.size, out)
        return out

    def pack_dense(self, bits: int, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        wc = int(self.lib.autref_dense_word_count(bits, c.size))
        out = np.empty(wc, np.uint32)
        self.lib.autref_pack_dense(bits, c, c.size, out, wc)
        return out

    def dot_v1_cases(self):
        return [self.lib.autref_dot_v1_case_id(k).decode()
                for k in range(self.lib.autref_dot_v1_case_count())]

    def dot_v1(self, case: int, vector_id: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.autref_dot_v1_fill(case, vector_id, n, out)
        return out

    def dot_dense(self, name: str, stride_bits: int, x_words, y_words, n: int, threads: int = 1):
        x = np.ascontiguousarray(x_words).view(np.uint32)
        y = np.ascontiguousarray(y_words).view(np.uint32)
        d, s = _d2(), _d2()
        self.lib.autref_dot_dense(self.index(name), stride_bits, x, y, n, threads, d, s)
        return _ld_pair(d), _ld_pair(s)

    def dot_raw(self, x, y, threads: int = 1):
        x = np.ascontiguousarray(x)
        y = np.ascontiguousarray(y)
        d, s = _d2(), _d2()
        self.lib.autref_dot_raw(1 if x.dtype == np.float64 else 0,
                                x.ctypes.data, y.ctypes.data, x.size, threads, d, s)
        return _ld_pair(d), _ld_pair(s)


class ReferenceGpu:
    """The reference's own GPU DOT kernels (oracle/_ref/librefgpu.so, built
    from its headers for sm_100a): run on device buffers the caller owns."""

    def __init__(self, path: str = REFGPU_SO):
        lib = C.CDLL(path)
        self.lib = lib
        lib.refgpu_variant_count.restype = C.c_int
        lib.refgpu_variant_name.restype = C.c_char_p
        lib.refgpu_variant_name.argtypes = [C.c_int]
        lib.refgpu_run.restype = C.c_int
        lib.refgpu_run.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_uint64, C.c_int,
                                   C.POINTER(C.c_double), C.POINTER(C.c_double)]
        self.variants = [lib.refgpu_variant_name(i).decode()
                         for i in range(lib.refgpu_variant_count())]

    def run(self, name: str, x_ptr: int, y_ptr: int, n: int, reps: int = 10):
        """(result, ms per DOT) of variant `name`."""
        res, ms = C.c_double(), C.c_double()
        rc = self.lib.refgpu_run(self.variants.index(name), x_ptr, y_ptr, n, reps,
                                 C.byref(res), C.byref(ms))
        if rc != 0:
            raise RuntimeError(f"reference kernel {name} failed ({rc})")
        return res.value, ms.value


def reference_gpu():
    """The reference's GPU kernels, or None when librefgpu.so was not built."""
    return ReferenceGpu() if os.path.exists(REFGPU_SO) else None


def oracle() -> Oracle:
    global _oracle
    with _lock:
        if _oracle is None:
            _oracle = Oracle()
        return _oracle


def reference():
    """The reference library, or None when it cannot be built here."""
    global _reference, _reference_tried
    with _lock:
        if _reference is None and not _reference_tried:
            _reference_tried = True
            if not os.path.exists(REF_SO):
                try:
                    build_reference()
                except (OSError, subprocess.CalledProcessError):
                    return None
            if os.path.exists(REF_SO):
                _reference = Reference()
        return _reference

"""ctypes binding of libautdot.so (the C ABI declared in include/autdot.h).

This is plumbing for Python callers (tests, bench.py): every compute call
goes straight to the CUDA library.  There is no Python or CPU fallback --
loading fails with ImportError when the library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libautdot.so")

AUT_OK = 0
AUT_ERR_INVALID_ARGUMENT = 1
AUT_ERR_UNSUPPORTED = 2
AUT_ERR_CUDA = 3
AUT_ERR_TOO_LARGE = 4
AUT_ERR_NO_DEVICE = 5
AUT_ERR_COMM = 6
COMM_ID_BYTES = 128

FAMILY_BINARY, FAMILY_PREFIX, FAMILY_LNS, FAMILY_RAW_FP32, FAMILY_RAW_FP64 = range(5)
DENSE, PADDED = 0, 1
ACC_FP32, ACC_FP64 = 0, 1
TARGET_FP32, TARGET_FP64 = 0, 1
STRATEGY_AUTO, STRATEGY_LDG, STRATEGY_TMA, STRATEGY_SCALAR, STRATEGY_COOPERATIVE = 0, 1, 2, 3, 4
(DECODER_AUTO, DECODER_DIRECT, DECODER_FULL_LUT, DECODER_FRACTION_LUT,
 DECODER_FRACTION_LUT_FUSED, DECODER_FUSED_SUM_LUT, DECODER_EX2_APPROX,
 DECODER_PREFIX_LUT, DECODER_SUBNORMAL_LUT) = range(9)
STATUS_WAIT_TIMEOUT = 1
GEN_SIGNED_UNIT_F64, GEN_SIGNED_UNIT_F32, GEN_NORMAL, GEN_LNS_CANCEL, GEN_POSITIVE_UNIT_F64 = range(5)

# C signatures: name -> (restype, argtypes)
_i32, _u32, _u64, _dbl = C.c_int32, C.c_uint32, C.c_uint64, C.c_double
_vp, _cp = C.c_void_p, C.c_char_p
_i32p = C.POINTER(C.c_int32)
SIGNATURES = {
    "aut_version": (_cp, []),
    "aut_abi_version": (_i32, []),
    "aut_last_error": (_cp, []),
    "aut_format_count": (_i32, []),
    "aut_format_id": (_i32, [_cp]),
    "aut_format_name": (_cp, [_i32]),
    "aut_format_info": (_i32, [_i32, _i32p, _i32p, _i32p, _i32p]),
    "aut_dot_supported": (_i32, [_i32, _i32, _i32]),
    "aut_storage_bytes": (_u64, [_i32, _i32, _u64]),
    "aut_packed_bytes": (_dbl, [_i32, _u64]),
    "aut_workspace_create": (_i32, [_i32, C.POINTER(_vp)]),
    "aut_workspace_destroy": (_i32, [_vp]),
    "aut_workspace_prepare": (_i32, [_vp, _i32]),
    "aut_workspace_info": (_i32, [_vp, _i32p, _i32p]),
    "aut_workspace_status": (_i32, [_vp, C.POINTER(_u32), _i32]),
    "aut_workspace_inject_stall": (_i32, [_vp, _u64, _u64]),
    "aut_dot": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _u64, _vp, _vp]),
    "aut_dot_strategy": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _u64, _vp, _vp]),
    "aut_dot_variant": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _u64, _vp, _vp]),
    "aut_dot_batched": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _u64, _u32, _u64, _vp, _vp]),
    "aut_gemv": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _u64, _u64, _vp, _vp]),
    "aut_dot_noalloc": (_i32, [_i32, _i32, _i32, _vp, _vp, _u64, _u32, _u64, _vp, _vp]),
    "aut_comm_unique_id": (_i32, [_vp]),
    "aut_comm_create": (_i32, [_vp, _i32, _i32, _i32, C.POINTER(_vp)]),
    "aut_comm_wrap": (_i32, [_vp, _i32, C.POINTER(_vp)]),
    "aut_comm_destroy": (_i32, [_vp]),
    "aut_comm_allreduce": (_i32, [_vp, _vp, _u64, _vp]),
    "aut_dot_sharded": (_i32, [_vp, _vp, _i32, _i32, _i32, _vp, _vp, _u64, _vp, _vp]),
    "aut_decode": (_i32, [_vp, _i32, _i32, _i32, _vp, _u64, _vp, _vp]),
    "aut_encode": (_i32, [_vp, _i32, _i32, _vp, _u64, _vp, _vp]),
    "aut_generate": (_i32, [_i32, _u64, _i32, _u64, _u64, _vp, _vp]),
    "aut_generate_dot_v1": (_i32, [_i32, _u64, _i32, _i32, _u64, _u64, _u64, _vp, _vp]),
    "aut_encode_host": (_i32, [_i32, _vp, _u64, _vp]),
    "aut_decode_host": (_i32, [_i32, _vp, _u64, _vp]),
    "aut_pack_host": (_i32, [_i32, _i32, _vp, _u64, _vp]),
    "aut_unpack_host": (_i32, [_i32, _i32, _vp, _u64, _vp]),
}

_lib = None


class AutError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"autdot status {status}: {message}")
        self.status = status


def load(path: str = LIB_PATH) -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with "
            "`python -m accessor_universal_test_b200.build` (needs nvcc)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != AUT_OK:
        msg = load().aut_last_error().decode(errors="replace")
        raise AutError(status, msg)


def format_id(name: str) -> int:
    fid = load().aut_format_id(name.encode())
    if fid < 0:
        raise KeyError(f"unknown storage format {name!r}")
    return fid


def format_info(fmt: int):
    fam, t, e, fin = C.c_int32(), C.c_int32(), C.c_int32(), C.c_int32()
    check(load().aut_format_info(fmt, C.byref(fam), C.byref(t), C.byref(e), C.byref(fin)))
    return fam.value, t.value, e.value, fin.value


def storage_bytes(fmt: int, layout: int, n: int) -> int:
    return int(load().aut_storage_bytes(fmt, layout, n))


class Workspace:
    """Owns an aut_workspace (grid-reduction scratch + decode tables)."""

    def __init__(self, device: int = 0):
        lib = load()
        h = C.c_void_p()
        check(lib.aut_workspace_create(device, C.byref(h)))
        self.handle = h
        self.device = device
        sm, mb = C.c_int32(), C.c_int32()
        check(lib.aut_workspace_info(h, C.byref(sm), C.byref(mb)))
        self.sm_count, self.max_blocks = sm.value, mb.value

    def close(self) -> None:
        if self.handle:
            load().aut_workspace_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def prepare(self, fmt: int) -> None:
        check(load().aut_workspace_prepare(self.handle, fmt))

    def dot(self, fmt, layout, accum, x_ptr, y_ptr, n, result_ptr, stream=0,
            strategy: int = 0, decoder: int = 0) -> None:
        check(load().aut_dot_variant(self.handle, fmt, layout, accum, strategy, decoder,
                                     x_ptr, y_ptr, n, result_ptr, stream))

    def status(self, clear: bool = True) -> int:
        word = C.c_uint32()
        check(load().aut_workspace_status(self.handle, C.byref(word), 1 if clear else 0))
        return word.value

    def inject_stall(self, stall_tile: int = 2**64 - 1, wait_cycles: int = 0) -> None:
        """Failure-detection test hook: the bulk-copy kernels withhold the
        copies of tile `stall_tile`, so their bounded wait runs out."""
        check(load().aut_workspace_inject_stall(self.handle, stall_tile, wait_cycles))

    def dot_batched(self, fmt, layout, accum, x_ptr, y_ptr, n, batch, stride_bytes,
                    results_ptr, stream=0) -> None:
        check(load().aut_dot_batched(self.handle, fmt, layout, accum, x_ptr, y_ptr, n,
                                     batch, stride_bytes, results_ptr, stream))

    def gemv(self, fmt, layout, accum, matrix_ptr, vector_ptr, rows, columns, result_ptr,
             stream=0, strategy: int = 0, decoder: int = 0) -> None:
        check(load().aut_gemv(self.handle, fmt, layout, accum, strategy, decoder, matrix_ptr,
                              vector_ptr, rows, columns, result_ptr, stream))

    def decode(self, fmt, layout, target, codes_ptr, n, out_ptr, stream=0) -> None:
        check(load().aut_decode(self.handle, fmt, layout, target, codes_ptr, n, out_ptr, stream))

    def encode(self, fmt, layout, values_ptr, n, codes_ptr, stream=0) -> None:
        check(load().aut_encode(self.handle, fmt, layout, values_ptr, n, codes_ptr, stream))


def generate_dot_v1(family: int, seed: int, parameter: int, vector_id: int, count: int,
                    out_ptr, first: int = 0, n: int | None = None, stream=0) -> None:
    """Values [first, first + n) of a dot_v1 case vector (FP32, on the device)."""
    n = count - first if n is None else n
    check(load().aut_generate_dot_v1(family, seed, parameter, vector_id, count, first, n,
                                     out_ptr, stream))


def comm_unique_id() -> bytes:
    """A fresh NCCL communicator id for Comm(); one rank makes it."""
    buf = C.create_string_buffer(COMM_ID_BYTES)
    check(load().aut_comm_unique_id(buf))
    return buf.raw


class Comm:
    """An aut_comm: this rank's NCCL communicator for aut_dot_sharded."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int):
        if len(unique_id) != COMM_ID_BYTES:
            raise ValueError(f"communicator id must be {COMM_ID_BYTES} bytes")
        h = C.c_void_p()
        check(load().aut_comm_create(unique_id, nranks, rank, device, C.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            check(load().aut_comm_destroy(self.handle))
            self.handle = None

    def allreduce(self, values_ptr, count: int, stream=0) -> None:
        check(load().aut_comm_allreduce(self.handle, values_ptr, count, stream))

    def dot(self, ws: "Workspace", fmt, layout, accum, x_ptr, y_ptr, n_local, result_ptr,
            stream=0) -> None:
        check(load().aut_dot_sharded(self.handle, ws.handle, fmt, layout, accum, x_ptr, y_ptr,
                                     n_local, result_ptr, stream))


def generate(kind: int, seed: int, vector_id: int, first: int, n: int, out_ptr, stream=0) -> None:
    check(load().aut_generate(kind, seed, vector_id, first, n, out_ptr, stream))

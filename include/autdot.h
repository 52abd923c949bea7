/*
 * autdot.h -- C ABI of the B200 decode-fused DOT library (libautdot.so).
 *
 * The reference (accessor_universal_test) exposes its DOT path as header-only
 * C++ templates driven by benchmark CLIs; it has no FFI layer.  This header
 * is the boundary a binding (ctypes, cgo, JNI, N-API) or the C++ wrappers in
 * include/aut/ call.  Each entry point names the reference interface it
 * replaces.  Conventions:
 *   - plain integers, pointers and sizes only; no C++ or torch types;
 *   - device pointers are CUDA global memory on the workspace's device;
 *   - every device call is asynchronous and ordered on `stream`
 *     (a cudaStream_t passed as void*; NULL = legacy default stream);
 *   - the return value is a status code; aut_last_error() gives the
 *     message of the calling thread's last failure (the reference throws
 *     std::runtime_error from CUDA_CHECK, src/bitwidth_strategy_bench.cu:32-47).
 */
#ifndef AUTDOT_H_
#define AUTDOT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AUTDOT_ABI_VERSION 1

typedef int32_t aut_status;
enum {
  AUT_OK = 0,
  AUT_ERR_INVALID_ARGUMENT = 1, /* bad pointer, size, enum value       */
  AUT_ERR_UNSUPPORTED = 2,      /* no kernel for format/layout/accum   */
  AUT_ERR_CUDA = 3,             /* a CUDA runtime call failed          */
  AUT_ERR_TOO_LARGE = 4,        /* size beyond a documented maximum    */
  AUT_ERR_NO_DEVICE = 5,        /* no usable CUDA device / wrong arch  */
  AUT_ERR_COMM = 6              /* NCCL missing, or a collective failed */
};

/* Format families (runtime descriptor of a storage format). */
enum {
  AUT_FAMILY_BINARY = 0,      /* storage::binary_format<T,E,finite>        */
  AUT_FAMILY_FP64_PREFIX = 1, /* storage::fp64_prefix<F>                   */
  AUT_FAMILY_LNS = 2,         /* lns::format<B,R>; exponent_bits holds R   */
  AUT_FAMILY_RAW_FP32 = 3,    /* IEEE binary32 storage                     */
  AUT_FAMILY_RAW_FP64 = 4     /* IEEE binary64 storage                     */
};

/* Format ids with a decode-fused DOT kernel.  Every other registered format
 * (storage_formats.hpp:110-262, lns_benchmark_core.hpp:44-61) has an id from
 * aut_format_id() and host/device codecs, but no DOT kernel yet. */
enum {
  AUT_FMT_FP32 = 0,      /* raw binary32                                  */
  AUT_FMT_FP64 = 1,      /* raw binary64                                  */
  AUT_FMT_E2M3 = 2,      /* FP6 E2M3, finite (storage_formats.hpp:132)    */
  AUT_FMT_E8M0 = 3,      /* 9-bit E8 (storage_formats.hpp:161)            */
  AUT_FMT_E8M1 = 4,      /* 10-bit E8 (:165)                              */
  AUT_FMT_E8M3 = 5,      /* 12-bit E8 (:170)                              */
  AUT_FMT_E8M5 = 6,      /* 14-bit E8 (:174)                              */
  AUT_FMT_BF16_E8M7 = 7, /* 16-bit E8 (cuda_storage_formats.cuh:37-43)    */
  AUT_FMT_E8M15 = 8,     /* 24-bit E8 (:203)                              */
  AUT_FMT_LNS8_R3 = 9,   /* lns_benchmark_core.hpp:48                     */
  AUT_FMT_LNS16_R11 = 10 /* lns_benchmark_core.hpp:56                     */
};

/* Storage layouts (bitwidth_benchmark_core.hpp:23).
 * DENSE:  value i at bits [B*i, B*i+B) of little-endian uint32 words, plus
 *         one zero guard word: aut_storage_bytes() = 4*(ceil(n*B/32)+1).
 * PADDED: one code per uint8/uint16/uint32 container (storage_type_t). */
enum { AUT_LAYOUT_DENSE = 0, AUT_LAYOUT_PADDED = 1 };

/* Per-thread accumulator of the fused DOT (compute_kind, :22).  Block and
 * grid reductions are FP64 for both; FP32 partial sums are carried into
 * FP64 at least every 128 products. */
enum { AUT_ACCUM_FP32 = 0, AUT_ACCUM_FP64 = 1 };

/* Decode target type. */
enum { AUT_TARGET_FP32 = 0, AUT_TARGET_FP64 = 1 };

/* How the fused DOT streams its operands (access_method,
 * bitwidth_benchmark_core.hpp:24).  AUTO picks the measured best per format. */
enum {
  AUT_STRATEGY_AUTO = 0,
  AUT_STRATEGY_LDG = 1,   /* 16-byte vector loads straight into registers   */
  AUT_STRATEGY_TMA = 2,   /* cp.async.bulk tiles into a shared-memory ring   */
  AUT_STRATEGY_SCALAR = 3, /* one code per load (the reference's scalar
                             access method); the slow baseline            */
  AUT_STRATEGY_COOPERATIVE = 4 /* groups of lanes load a chunk's words once
                             and share them by warp shuffles
                             (cooperative_shuffle; dense E8 and e2m3) */
};

/* How the fused DOT turns codes into values (decoder_kind,
 * bitwidth_benchmark_core.hpp:25-40, lns_decoder_strategies.cuh:19-34).
 * AUTO picks the measured best per format and accumulator. */
enum {
  AUT_DECODER_AUTO = 0,
  AUT_DECODER_DIRECT = 1,      /* bit moves / hardware conversion (E8, e2m3, raw) */
  AUT_DECODER_FULL_LUT = 2,     /* one shared-memory lookup per code (LNS)     */
  AUT_DECODER_FRACTION_LUT = 3, /* fraction table + exponent add (lns16_r11)   */
  AUT_DECODER_FRACTION_LUT_FUSED = 4, /* logs added, one fraction lookup per
                                         pair: multiply_kind::fused (lns16_r11) */
  AUT_DECODER_FUSED_SUM_LUT = 5, /* logs added, one lookup per pair in a table of
                                   every product: fused_sum_lut_shared (lns8_r3) */
  AUT_DECODER_EX2_APPROX = 6,   /* logs added, one hardware ex2.approx.f32 per
                                   pair (ex2_approx with the fused multiply,
                                   lns_decoder_strategies.cuh:215-224; lns8_r3,
                                   lns16_r11).  APPROXIMATE: relative error up to
                                   2^-21 per product; never chosen by AUTO */
  AUT_DECODER_PREFIX_LUT = 7,   /* sign+exponent table, mantissa ORed in:
                                   prefix_lut_shared (e8m1, e8m3, e8m5) */
  AUT_DECODER_SUBNORMAL_LUT = 8 /* table of the subnormal values, bit moves for
                                   the rest: subnormal_lut_shared (e8m1, e8m3,
                                   e8m5) */
};

/* Sticky device status bits reported by aut_workspace_status(). */
enum {
  AUT_STATUS_WAIT_TIMEOUT = 1 /* a bounded pipeline wait gave up; the
                                 affected results were written as NaN */
};

/* Synthetic generators for aut_generate (seeded, counter based, identical
 * on host and device for every index). */
enum {
  AUT_GEN_SIGNED_UNIT_F64 = 0, /* uniform [-1,1), 2^-51 grid (dot_bench.cu:389-393) */
  AUT_GEN_SIGNED_UNIT_F32 = 1, /* uniform [-1,1), 2^-22 grid (dot_dataset.hpp:149-153) */
  AUT_GEN_NORMAL = 2,          /* Irwin-Hall(12) - 6, approximately N(0,1)   */
  AUT_GEN_LNS_CANCEL = 3,      /* vector 0: x ~ U[-1,1); vector 1:
                                  y_i = s_i x_i (1 + 1e-6 u_i), s alternating */
  AUT_GEN_POSITIVE_UNIT_F64 = 4 /* uniform (0,1], 2^-53 grid (dot_bench.cu:375-379) */
};

/* ---- library / format registry ---------------------------------------- */
const char *aut_version(void);
int32_t aut_abi_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char *aut_last_error(void);

int32_t aut_format_count(void);
/* Id of a format by its reference name ("e2m3", "bf16_e8m7", "lns16_r11",
 * "fp32", ...); -1 when unknown. */
int32_t aut_format_id(const char *name);
const char *aut_format_name(int32_t format);
aut_status aut_format_info(int32_t format, int32_t *family,
                           int32_t *total_bits, int32_t *exponent_bits,
                           int32_t *finite);
/* 1 when aut_dot has a fused kernel for this combination, else 0. */
int32_t aut_dot_supported(int32_t format, int32_t layout, int32_t accum);
/* Bytes a caller allocates for n values (dense: includes the guard word;
 * replaces dense_word_count/dense_data_bytes, bitwidth_benchmark_core.hpp:160-169). */
uint64_t aut_storage_bytes(int32_t format, int32_t layout, uint64_t n);
/* Algorithmic (packed) bytes of n values: n * total_bits / 8. */
double aut_packed_bytes(int32_t format, uint64_t n);

/* ---- workspace: per-device scratch and decode tables ------------------- */
typedef struct aut_workspace aut_workspace;
/* Allocates the grid-reduction scratch and binds the library to `device`.
 * Replaces the reference's partials/result buffers
 * (src/bitwidth_strategy_bench.cu:466, device_buffer<value_type> partials_(512)).
 * Every DOT and GEMV call on a workspace uses its one scratch area: calls on
 * one stream follow each other; streams that run calls at the same time need
 * a workspace each. */
aut_status aut_workspace_create(int32_t device, aut_workspace **out);
aut_status aut_workspace_destroy(aut_workspace *ws);
/* Builds (once) the decode tables of `format` so that later calls issue no
 * host-to-device copies; call before capturing aut_dot in a CUDA graph. */
aut_status aut_workspace_prepare(aut_workspace *ws, int32_t format);
/* Number of SMs and the maximum grid the DOT kernels launch on them. */
aut_status aut_workspace_info(const aut_workspace *ws, int32_t *sm_count,
                              int32_t *max_blocks);
/* Waits for the device, then reports (and with clear != 0 resets) the
 * sticky AUT_STATUS_* bits the kernels of this workspace raised. */
aut_status aut_workspace_status(aut_workspace *ws, uint32_t *status,
                                int32_t clear);
/* Failure-detection test hook (no counterpart in the reference, which has no
 * bounded waits).  Until called again, the bulk-copy (TMA) DOT kernels
 * launched through `ws` arm the ring stage of tile `stall_tile` of every
 * pair without issuing its copies, and bound every barrier wait by
 * `wait_cycles` SM clock cycles (0: the default, ~2 s).  The wait for that
 * stage therefore runs out: the block lets its other copies land, sets
 * AUT_STATUS_WAIT_TIMEOUT and the DOT's result is NaN.  No copy is left in
 * flight, nothing waits without a bound, and the context stays usable.
 * stall_tile = UINT64_MAX switches the hook off.  Not for production use. */
aut_status aut_workspace_inject_stall(aut_workspace *ws, uint64_t stall_tile,
                                      uint64_t wait_cycles);

/* ---- the decode-fused DOT ---------------------------------------------- */
/* result[0] = sum_i decode(x_i) * decode(y_i), written to device memory.
 * Replaces dot_thread_kernel + finalize_dot_kernel
 * (bitwidth_benchmark_kernels.cuh:403-457), the LNS dot_thread_kernel
 * (lns_benchmark_kernels.cuh:80-131), raw_dot_kernel (:681-703) and the
 * accessor DOT (src/accessor_dot_bench.cu:417-474) in one call: one launch,
 * single-pass grid reduction, deterministic for a given device.
 * x and y hold n values in `layout`; 16-byte aligned pointers take the
 * vectorised path.  n = 0 writes 0. */
aut_status aut_dot(aut_workspace *ws, int32_t format, int32_t layout,
                   int32_t accum, const void *x, const void *y, uint64_t n,
                   double *result, void *stream);

/* aut_dot with an explicit access strategy (AUT_STRATEGY_*), the axis the
 * reference's strategy benchmarks sweep (src/bitwidth_strategy_bench.cu:704-742). */
aut_status aut_dot_strategy(aut_workspace *ws, int32_t format, int32_t layout,
                            int32_t accum, int32_t strategy, const void *x,
                            const void *y, uint64_t n, double *result,
                            void *stream);

/* aut_dot with explicit access strategy and decoder (AUT_DECODER_*), the two
 * axes of the reference's strategy matrix (src/bitwidth_strategy_bench.cu:744-782,
 * src/lns_strategy_bench.cu:961-1025).  Combinations without a kernel return
 * AUT_ERR_UNSUPPORTED. */
aut_status aut_dot_variant(aut_workspace *ws, int32_t format, int32_t layout,
                           int32_t accum, int32_t strategy, int32_t decoder,
                           const void *x, const void *y, uint64_t n,
                           double *result, void *stream);

/* `batch` independent DOTs in one launch: pair b reads
 * x + b*batch_stride_bytes and y + b*batch_stride_bytes; results[b]. */
aut_status aut_dot_batched(aut_workspace *ws, int32_t format, int32_t layout,
                           int32_t accum, const void *x, const void *y,
                           uint64_t n, uint32_t batch,
                           uint64_t batch_stride_bytes, double *results,
                           void *stream);

/* Matrix-vector product over compact storage, the reference's other kernel
 * (gemv_thread_kernel, bitwidth_benchmark_kernels.cuh:459-501; raw FP32/FP64
 * raw_gemv_kernel, :705-728):
 *   result[r] = sum_c decode(matrix[r * columns + c]) * decode(vector[c])
 * for r < rows, written to device memory as FP64.  The matrix is one stream
 * of rows * columns values in `layout` (row-major), the vector one stream of
 * `columns` values, both in `format`.  Each row is a fused DOT of the same
 * kernels as aut_dot_variant; when columns * bits-per-slot is a multiple of
 * 128 every row starts on a 16-byte boundary and takes the vectorised path,
 * otherwise rows are read value by value.  rows = 0 does nothing; columns =
 * 0 writes zeros. */
aut_status aut_gemv(aut_workspace *ws, int32_t format, int32_t layout,
                    int32_t accum, int32_t strategy, int32_t decoder,
                    const void *matrix, const void *vector, uint64_t rows,
                    uint64_t columns, double *result, void *stream);

/* The fused DOT without a workspace, for callers that cannot allocate device
 * memory (a host framework that owns the GPU's memory through its own pool,
 * a latency-critical path that cannot absorb cudaMalloc's device-wide
 * synchronisation, a foreign-language caller with nowhere to keep a
 * workspace).  No counterpart in the reference: it always allocates its
 * partials with cudaMalloc.  The reduction scratch is a fixed 32 KiB device
 * array inside the library (held on every GPU that loads it until exit):
 * at most 64 DOTs per call (batch > 64 -> AUT_ERR_TOO_LARGE); table-decoded
 * formats (LNS) -> AUT_ERR_UNSUPPORTED.  All calls share that array, so
 * calls that overlap on one GPU race; serialise them.  The first call on a
 * device looks up the array's address; make it before any stream capture
 * (a failed lookup is not kept: the next call tries again; after
 * cudaDeviceReset the kept address is stale, so do not reset a device this
 * entry point has used).  There is no status query: a DOT whose bounded
 * bulk-copy wait gave up reports it only as NaN in its results[b].  A call
 * refused for its arguments or format enqueues nothing.
 * Arguments as in aut_dot_batched, on the calling thread's current device. */
aut_status aut_dot_noalloc(int32_t format, int32_t layout, int32_t accum,
                           const void *x, const void *y, uint64_t n,
                           uint32_t batch, uint64_t batch_stride_bytes,
                           double *results, void *stream);

/* ---- multi-GPU: contiguous shards and one NCCL all-reduce --------------- */
/* The reference runs one GPU and has no collective; a DOT over a vector too
 * long for one GPU, or spread over the GPUs of a node, is the sum of the
 * ranks' shard DOTs.  One rank per GPU; every rank calls the same
 * collective entry points in the same order.  NCCL (libnccl.so.2) is loaded
 * at the first call below; without it they return AUT_ERR_COMM. */
typedef struct aut_comm aut_comm;
#define AUT_COMM_ID_BYTES 128
/* A fresh communicator id (ncclGetUniqueId) into id[AUT_COMM_ID_BYTES]; one
 * rank makes it and hands it to the others (any host channel). */
aut_status aut_comm_unique_id(void *id);
/* Joins the communicator `id` as `rank` of `nranks` on `device` (blocks
 * until every rank has joined). */
aut_status aut_comm_create(const void *id, int32_t nranks, int32_t rank,
                           int32_t device, aut_comm **out);
/* Uses a caller's ncclComm_t (same NCCL library as this process loads) on
 * `device`; aut_comm_destroy then frees only the wrapper. */
aut_status aut_comm_wrap(void *nccl_comm, int32_t device, aut_comm **out);
aut_status aut_comm_destroy(aut_comm *comm);
/* In-place sum over the ranks of `count` FP64 values, ordered on `stream`. */
aut_status aut_comm_allreduce(aut_comm *comm, double *values, uint64_t count,
                              void *stream);
/* result[0] = the DOT of the global vectors: aut_dot of this rank's shard
 * (x, y hold its n_local values; for dense streams a shard that starts on a
 * whole 16-byte packet, 128 / gcd(bits, 128) values, is a byte offset into
 * the global stream) followed by one ncclAllReduce of the FP64 partial on
 * the same stream.  Replaces nothing in the reference (single GPU only);
 * its per-GPU part is aut_dot. */
aut_status aut_dot_sharded(aut_comm *comm, aut_workspace *ws, int32_t format,
                           int32_t layout, int32_t accum, const void *x,
                           const void *y, uint64_t n_local, double *result,
                           void *stream);

/* ---- device codecs ------------------------------------------------------ */
/* out[i] = decode(codes[i]) as float or double, bit-identical to the
 * reference's host storage::decode / lns::decode (validate_decode_kernel,
 * lns_benchmark_kernels.cuh:359-374). */
aut_status aut_decode(aut_workspace *ws, int32_t format, int32_t layout,
                      int32_t target, const void *codes, uint64_t n,
                      void *out, void *stream);
/* Round-to-nearest-even encode of device doubles into `layout`
 * (encode_padded_kernel + pack_dense_kernel,
 * bitwidth_benchmark_kernels.cuh:625-668; lns_benchmark_kernels.cuh:309-357).
 * `codes` must hold aut_storage_bytes(format, layout, n) bytes.  LNS codes
 * equal the host encoder's for every input (threshold tables built from the
 * host log2). */
aut_status aut_encode(aut_workspace *ws, int32_t format, int32_t layout,
                      const double *values, uint64_t n, void *codes,
                      void *stream);
/* out[i] = generator value of index first + i. */
aut_status aut_generate(int32_t kind, uint64_t seed, int32_t vector_id,
                        uint64_t first, uint64_t n, double *out, void *stream);
/* out[i] = value first + i of vector `vector_id` (0: x, 1: y) of a dot_v1
 * validation case of `count` values: family 0 positive_uniform, 1
 * signed_uniform, 2 controlled_cancellation, 3 dynamic_range, with its seed
 * and parameter (aut::dataset::accuracy_cases), FP32, bit-identical to the
 * reference's generator (dot_dataset.hpp:72-152). */
aut_status aut_generate_dot_v1(int32_t family, uint64_t seed, int32_t parameter,
                               int32_t vector_id, uint64_t count, uint64_t first,
                               uint64_t n, float *out, void *stream);

/* ---- host codecs (the host half of storage::encode/decode) -------------- */
aut_status aut_encode_host(int32_t format, const double *values, uint64_t n,
                           uint32_t *codes);
aut_status aut_decode_host(int32_t format, const uint32_t *codes, uint64_t n,
                           double *out);
/* Pack codes (one per uint32) into `layout`; out holds aut_storage_bytes(). */
aut_status aut_pack_host(int32_t format, int32_t layout, const uint32_t *codes,
                         uint64_t n, void *out);
aut_status aut_unpack_host(int32_t format, int32_t layout, const void *packed,
                           uint64_t n, uint32_t *codes);

#ifdef __cplusplus
}
#endif

#endif /* AUTDOT_H_ */

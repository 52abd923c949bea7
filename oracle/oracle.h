/*
 * oracle.h -- CPU restatement of the reference's decode-fused DOT path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * product: only tests/, __graft_entry__.smoke() and the cpu_baseline /
 * reference legs of bench.py load it.  Nothing in the product links it.
 *
 * Each function restates one piece of the reference (accessor_universal_test)
 * in plain C and cites the reference file:line it follows:
 *   - storage codecs        include/storage_formats.hpp
 *   - dense bitstream       include/bitwidth_benchmark_core.hpp
 *   - LNS codec             include/lns_benchmark_core.hpp
 *   - dot_v1 dataset        include/dot_dataset.hpp
 *   - compensated reference src/dot_bench.cu:532-577
 *
 * Parity of this restatement is pinned two ways (tests/test_oracle_*.py):
 * bit-for-bit against the reference's own headers compiled into
 * oracle/_ref/libautref.so, and against the committed golden vectors in
 * tests/golden/ (dot_v1 fingerprints and reference dots, the reference's
 * unit-test known answers).
 */
#ifndef AUT_ORACLE_H_
#define AUT_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Format families (mirror the product's runtime descriptor). */
enum {
  ORC_FAMILY_BINARY = 0,     /* binary_format<T,E,finite>: E=0 fixed, E>=1 IEEE-like */
  ORC_FAMILY_FP64_PREFIX = 1,/* fp64_prefix<F>: T = 12 + F, E = 11             */
  ORC_FAMILY_LNS = 2,        /* lns::format<B,R>: exponent_bits carries R        */
  ORC_FAMILY_RAW_FP32 = 3,
  ORC_FAMILY_RAW_FP64 = 4
};

/* ---- single-value codecs ---------------------------------------------- */
uint32_t orc_encode(int family, int total_bits, int exponent_bits, int finite,
                    double value);
double orc_decode_f64(int family, int total_bits, int exponent_bits,
                      int finite, uint32_t raw);
float orc_decode_f32(int family, int total_bits, int exponent_bits,
                     int finite, uint32_t raw);

/* ---- array codecs ------------------------------------------------------ */
void orc_encode_array(int family, int total_bits, int exponent_bits,
                      int finite, const double *values, uint64_t count,
                      uint32_t *codes);
void orc_decode_array_f64(int family, int total_bits, int exponent_bits,
                          int finite, const uint32_t *codes, uint64_t count,
                          double *out);
void orc_decode_array_f32(int family, int total_bits, int exponent_bits,
                          int finite, const uint32_t *codes, uint64_t count,
                          float *out);

/* ---- dense LSB-first bitstream (bitwidth_benchmark_core.hpp:135-169) --- */
uint64_t orc_dense_word_count(int bits, uint64_t values);
uint64_t orc_dense_data_bytes(int bits, uint64_t values);
uint32_t orc_load_dense(int bits, const uint32_t *words, uint64_t index);
void orc_or_dense(int bits, uint32_t *words, uint64_t index, uint32_t raw);
/* Zero `words` (orc_dense_word_count entries) and pack `count` codes. */
void orc_pack_dense(int bits, const uint32_t *codes, uint64_t count,
                    uint32_t *words);
void orc_unpack_dense(int bits, const uint32_t *words, uint64_t count,
                      uint32_t *codes);

/* ---- datasets ---------------------------------------------------------- */
uint64_t orc_splitmix64(uint64_t value);
/* dot_dataset.hpp:191-214; family = dataset::family enum value. */
float orc_dot_v1_value(int kind, uint64_t seed, int parameter, int vector_id,
                       uint64_t index, uint64_t count);
void orc_dot_v1_fill(int kind, uint64_t seed, int parameter, int vector_id,
                     uint64_t count, float *out);
uint64_t orc_fnv1a_f32(const float *values, uint64_t count);

/* Synthetic workload generators shared with the device generator
 * (accessor_universal_test_b200/csrc/codec.cu).  kind:
 *   0 = signed uniform double in [-1,1) (dot_bench.cu:389-393 mapping)
 *   1 = signed uniform float  in [-1,1) (dot_dataset.hpp:149-153 mapping)
 *   2 = approximately N(0,1): Irwin-Hall sum of 12 uniforms minus 6
 *   3 = LNS cancellation partner: y_i = s_i * x_i * (1 + 1e-6 u_i)
 *   4 = positive uniform double in (0,1] (dot_bench.cu:375-379 mapping)
 */
double orc_synthetic_value(int kind, uint64_t seed, int vector_id,
                           uint64_t index);
void orc_synthetic_fill(int kind, uint64_t seed, int vector_id,
                        uint64_t first, uint64_t count, double *out);

/* ---- compensated long-double reference (dot_bench.cu:532-577) ---------- */
/* Results come back as (hi, lo) double pairs: hi + lo == the long double. */
void orc_dot_reference_f64(const double *x, const double *y, uint64_t count,
                           double out_dot[2], double out_sum_abs[2]);
void orc_dot_reference_f32(const float *x, const float *y, uint64_t count,
                           double out_dot[2], double out_sum_abs[2]);
/* Decode two code arrays (uint32 per code) and run the compensated DOT on
 * `threads` host threads over contiguous shards with a compensated merge. */
void orc_dot_codes(int family, int total_bits, int exponent_bits, int finite,
                   const uint32_t *x, const uint32_t *y, uint64_t count,
                   int threads, double out_dot[2], double out_sum_abs[2]);
/* Same, reading codes straight from packed dense words (stride = bits). */
void orc_dot_dense(int family, int total_bits, int exponent_bits, int finite,
                   int stride_bits, const uint32_t *x_words,
                   const uint32_t *y_words, uint64_t count, int threads,
                   double out_dot[2], double out_sum_abs[2]);

#ifdef __cplusplus
}
#endif

#endif

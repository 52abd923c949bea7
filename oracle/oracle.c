/*
 * oracle.c -- CPU restatement of the reference's decode-fused DOT path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Built with -ffp-contract=off so
 * that every floating-point step rounds exactly where the reference's host
 * code rounds.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* bit helpers (storage_formats.hpp:29-79)                                   */
/* ------------------------------------------------------------------------ */

static uint64_t dbits(double v) {
  uint64_t b;
  memcpy(&b, &v, sizeof b);
  return b;
}

static double dfrom(uint64_t b) {
  double v;
  memcpy(&v, &b, sizeof v);
  return v;
}

static int hsb64(uint64_t v) { return 63 - __builtin_clzll(v); }

/* detail::round_right_shift_even, storage_formats.hpp:64-79 */
static uint64_t rshift_rne(uint64_t value, unsigned shift) {
  if (shift == 0) return value;
  if (shift >= 64) return 0;
  uint64_t q = value >> shift;
  uint64_t rem = value & ((UINT64_C(1) << shift) - 1);
  uint64_t half = UINT64_C(1) << (shift - 1);
  int up = rem > half || (rem == half && (q & 1u));
  return q + (uint64_t)up;
}

static uint32_t mask_bits(int bits) {
  return bits >= 32 ? 0xffffffffu : ((UINT32_C(1) << bits) - 1u);
}

/* ------------------------------------------------------------------------ */
/* E = 0 signed fixed point, storage_formats.hpp:266-342                     */
/* ------------------------------------------------------------------------ */

static uint32_t fixed_encode(int T, double value) {
  const int F = T - 1;
  const uint64_t magmask = (UINT64_C(1) << F) - 1;
  const uint64_t src = dbits(value);
  const uint64_t sign = src >> 63;
  const uint64_t sexp = (src >> 52) & 0x7ffu;
  const uint64_t sfrac = src & ((UINT64_C(1) << 52) - 1);
  const uint64_t sfield = sign << (T - 1);
  if (sexp == 0x7ffu) return (uint32_t)(sfield | magmask); /* :286-290 */
  if (sexp == 0 && sfrac == 0) return (uint32_t)sfield;
  uint64_t sig;
  int unb;
  if (sexp == 0) {
    sig = sfrac;
    unb = -1022;
  } else {
    sig = (UINT64_C(1) << 52) | sfrac;
    unb = (int)sexp - 1023;
  }
  const int shift = 52 - F - unb; /* :306 */
  uint64_t mag;
  if (shift > 0) {
    mag = rshift_rne(sig, (unsigned)shift);
  } else {
    const unsigned ls = (unsigned)(-shift);
    if (ls >= 64 || sig > (magmask >> ls))
      mag = magmask;
    else
      mag = sig << ls;
  }
  if (mag > magmask) mag = magmask;
  return (uint32_t)(sfield | mag);
}

static double fixed_decode(int T, uint32_t stored) {
  const int F = T - 1;
  const uint64_t raw = (uint64_t)stored & ((UINT64_C(1) << T) - 1);
  const uint64_t sign = raw >> (T - 1);
  const uint64_t mag = raw & ((UINT64_C(1) << F) - 1);
  if (mag == 0) return dfrom(sign << 63);
  const int lead = hsb64(mag);
  const uint64_t e64 = (uint64_t)(lead - F + 1023);
  const uint64_t f64 = (mag - (UINT64_C(1) << lead)) << (52 - lead);
  return dfrom((sign << 63) | (e64 << 52) | f64);
}

/* ------------------------------------------------------------------------ */
/* E >= 1 IEEE-like codec, storage_formats.hpp:344-467                       */
/* ------------------------------------------------------------------------ */

static uint32_t ieee_encode(int T, int E, int finite, double value) {
  const int M = T - E - 1;
  const uint64_t fmask = (UINT64_C(1) << M) - 1;
  const uint64_t emask = (UINT64_C(1) << E) - 1;
  const int bias = (1 << (E - 1)) - 1;
  const uint64_t maxexp = finite ? emask : emask - 1;
  const uint64_t src = dbits(value);
  const uint64_t sign = src >> 63;
  const uint64_t sexp = (src >> 52) & 0x7ffu;
  const uint64_t sfrac = src & ((UINT64_C(1) << 52) - 1);
  const uint64_t sfield = sign << (T - 1);

  if (sexp == 0x7ffu) { /* :368-386 */
    if (finite) return (uint32_t)(sfield | (maxexp << M) | fmask);
    if (sfrac == 0) return (uint32_t)(sfield | (emask << M));
    uint64_t payload = sfrac >> (52 - M);
    if (payload == 0) payload = 1;
    return (uint32_t)(sfield | (emask << M) | (payload & fmask));
  }
  if (sexp == 0) return (uint32_t)sfield; /* :388-392 */

  const int unb = (int)sexp - 1023;
  int texp = unb + bias;
  if (texp <= 0) { /* gradual underflow, :397-410 */
    const uint64_t sig = (UINT64_C(1) << 52) | sfrac;
    const unsigned shift = (unsigned)(53 - unb - bias - M);
    const uint64_t sub = rshift_rne(sig, shift);
    if (sub == 0) return (uint32_t)sfield;
    if (sub >= (UINT64_C(1) << M))
      return (uint32_t)(sfield | (UINT64_C(1) << M));
    return (uint32_t)(sfield | sub);
  }
  uint64_t tfrac = rshift_rne(sfrac, (unsigned)(52 - M)); /* :412-417 */
  if (tfrac == (UINT64_C(1) << M)) {
    tfrac = 0;
    ++texp;
  }
  if (texp > (int)maxexp) { /* :419-428 */
    if (finite) return (uint32_t)(sfield | (maxexp << M) | fmask);
    return (uint32_t)(sfield | (emask << M));
  }
  return (uint32_t)(sfield | ((uint64_t)texp << M) | tfrac);
}

static double ieee_decode(int T, int E, int finite, uint32_t stored) {
  const int M = T - E - 1;
  const uint64_t raw = (uint64_t)stored & ((UINT64_C(1) << T) - 1);
  const uint64_t emask = (UINT64_C(1) << E) - 1;
  const int bias = (1 << (E - 1)) - 1;
  const uint64_t sign64 = (raw >> (T - 1)) << 63;
  const uint64_t exp = (raw >> M) & emask;
  const uint64_t frac = raw & ((UINT64_C(1) << M) - 1);
  if (exp == 0) { /* :443-453 */
    if (frac == 0) return dfrom(sign64);
    const int lead = hsb64(frac);
    const int unb = lead + 1 - bias - M;
    const uint64_t e64 = (uint64_t)(unb + 1023);
    const uint64_t f64 = (frac - (UINT64_C(1) << lead)) << (52 - lead);
    return dfrom(sign64 | (e64 << 52) | f64);
  }
  if (!finite && exp == emask) /* :455-461 */
    return dfrom(sign64 | (UINT64_C(0x7ff) << 52) | (frac << (52 - M)));
  const int unb = (int)exp - bias;
  return dfrom(sign64 | ((uint64_t)(unb + 1023) << 52) | (frac << (52 - M)));
}

/* ------------------------------------------------------------------------ */
/* FP64-prefix codec, storage_formats.hpp:561-592                            */
/* ------------------------------------------------------------------------ */

static uint32_t prefix_encode(int F, double value) {
  const int discarded = 52 - F;
  const uint64_t bits = dbits(value);
  const uint64_t exp = (bits >> 52) & 0x7ffu;
  const uint64_t frac = bits & ((UINT64_C(1) << 52) - 1);
  uint64_t kept = bits >> discarded;
  if (exp == 0x7ffu) {
    if (frac != 0 && (kept & ((UINT64_C(1) << F) - 1)) == 0) kept |= 1;
    return (uint32_t)(kept & mask_bits(12 + F));
  }
  const uint64_t dropped = bits & ((UINT64_C(1) << discarded) - 1);
  const uint64_t half = UINT64_C(1) << (discarded - 1);
  if (dropped > half || (dropped == half && (kept & 1u))) ++kept;
  return (uint32_t)(kept & mask_bits(12 + F));
}

static double prefix_decode(int F, uint32_t stored) {
  return dfrom((uint64_t)(stored & mask_bits(12 + F)) << (52 - F));
}

/* ------------------------------------------------------------------------ */
/* LNS codec, lns_benchmark_core.hpp:93-230                                  */
/* ------------------------------------------------------------------------ */

static uint32_t lns_log_mask(int B) { return (UINT32_C(1) << (B - 1)) - 1u; }
static uint32_t lns_sign_mask(int B) { return UINT32_C(1) << (B - 1); }
static uint32_t lns_special(int B) { return UINT32_C(1) << (B - 2); }

static int32_t lns_log_code(int B, uint32_t raw) { /* :143-151 */
  uint32_t code = raw & lns_log_mask(B);
  if (code & (UINT32_C(1) << (B - 2))) code |= ~lns_log_mask(B);
  return (int32_t)code;
}

static uint32_t lns_make_raw(int B, int negative, int32_t code) {
  return (negative ? lns_sign_mask(B) : 0u) |
         ((uint32_t)code & lns_log_mask(B));
}

static uint32_t lns_encode(int B, int R, double value) { /* :194-230 */
  if (value != value) return lns_sign_mask(B) | lns_special(B);
  const int32_t maxc = (int32_t)lns_special(B) - 1;
  const int32_t minc = -(int32_t)lns_special(B) + 1;
  if (value > DBL_MAX || value < -DBL_MAX)
    return lns_make_raw(B, value < 0.0, maxc);
  if (value == 0.0) return lns_special(B);
  const int negative = value < 0.0;
  const double mag = negative ? -value : value;
  const double scaled = log2(mag) * (double)(UINT64_C(1) << R);
  if (scaled <= (double)minc - 0.5) return lns_special(B);
  int64_t rounded = (int64_t)nearbyint(scaled);
  if (rounded < minc) rounded = minc;
  if (rounded > maxc) rounded = maxc;
  return lns_make_raw(B, negative, (int32_t)rounded);
}

static int lns_is_special(int B, uint32_t raw) {
  return (raw & lns_log_mask(B)) == lns_special(B);
}

static double lns_decode_f64(int B, int R, uint32_t raw) { /* :179-192 */
  raw &= mask_bits(B);
  if (lns_is_special(B, raw)) {
    if (raw & lns_sign_mask(B)) return NAN;
    return 0.0;
  }
  const double scale = (double)(UINT32_C(1) << R);
  double v = exp2((double)lns_log_code(B, raw) / scale);
  return (raw & lns_sign_mask(B)) ? -v : v;
}

static float lns_decode_f32(int B, int R, uint32_t raw) {
  raw &= mask_bits(B);
  if (lns_is_special(B, raw)) {
    if (raw & lns_sign_mask(B)) return NAN;
    return 0.0f;
  }
  const float scale = (float)(UINT32_C(1) << R);
  float v = exp2f((float)lns_log_code(B, raw) / scale);
  return (raw & lns_sign_mask(B)) ? -v : v;
}

/* ------------------------------------------------------------------------ */
/* dispatch                                                                  */
/* ------------------------------------------------------------------------ */

uint32_t orc_encode(int family, int T, int E, int finite, double value) {
  switch (family) {
  case ORC_FAMILY_BINARY:
    return E == 0 ? fixed_encode(T, value) : ieee_encode(T, E, finite, value);
  case ORC_FAMILY_FP64_PREFIX:
    return prefix_encode(T - 12, value);
  case ORC_FAMILY_LNS:
    return lns_encode(T, E, value);
  case ORC_FAMILY_RAW_FP32: {
    float f = (float)value;
    uint32_t b;
    memcpy(&b, &f, sizeof b);
    return b;
  }
  default:
    return 0;
  }
}

double orc_decode_f64(int family, int T, int E, int finite, uint32_t raw) {
  switch (family) {
  case ORC_FAMILY_BINARY:
    return E == 0 ? fixed_decode(T, raw) : ieee_decode(T, E, finite, raw);
  case ORC_FAMILY_FP64_PREFIX:
    return prefix_decode(T - 12, raw);
  case ORC_FAMILY_LNS:
    return lns_decode_f64(T, E, raw);
  case ORC_FAMILY_RAW_FP32: {
    float f;
    memcpy(&f, &raw, sizeof f);
    return (double)f;
  }
  default:
    return NAN;
  }
}

float orc_decode_f32(int family, int T, int E, int finite, uint32_t raw) {
  if (family == ORC_FAMILY_LNS) return lns_decode_f32(T, E, raw);
  /* Every binary format with E <= 8 and M <= 23 is exact in FP32, so the
   * FP32 target equals the narrowed FP64 decode (bitwidth_benchmark_core.hpp
   * decode_reference<fp32>, :234-240). */
  return (float)orc_decode_f64(family, T, E, finite, raw);
}

void orc_encode_array(int family, int T, int E, int finite,
                      const double *values, uint64_t count, uint32_t *codes) {
  for (uint64_t i = 0; i < count; ++i)
    codes[i] = orc_encode(family, T, E, finite, values[i]);
}

void orc_decode_array_f64(int family, int T, int E, int finite,
                          const uint32_t *codes, uint64_t count, double *out) {
  for (uint64_t i = 0; i < count; ++i)
    out[i] = orc_decode_f64(family, T, E, finite, codes[i]);
}

void orc_decode_array_f32(int family, int T, int E, int finite,
                          const uint32_t *codes, uint64_t count, float *out) {
  for (uint64_t i = 0; i < count; ++i)
    out[i] = orc_decode_f32(family, T, E, finite, codes[i]);
}

/* ------------------------------------------------------------------------ */
/* dense bitstream, bitwidth_benchmark_core.hpp:135-169                      */
/* ------------------------------------------------------------------------ */

uint64_t orc_dense_word_count(int bits, uint64_t values) {
  return (values * (uint64_t)bits + 31u) / 32u + 1u; /* +1 zero guard word */
}

uint64_t orc_dense_data_bytes(int bits, uint64_t values) {
  return (values * (uint64_t)bits + 7u) / 8u;
}

uint32_t orc_load_dense(int bits, const uint32_t *words, uint64_t index) {
  const uint64_t bit = index * (uint64_t)bits;
  const uint64_t w = bit >> 5;
  const unsigned shift = (unsigned)(bit & 31u);
  const uint64_t pair = (uint64_t)words[w] | ((uint64_t)words[w + 1] << 32);
  return (uint32_t)(pair >> shift) & mask_bits(bits);
}

void orc_or_dense(int bits, uint32_t *words, uint64_t index, uint32_t raw) {
  const uint64_t bit = index * (uint64_t)bits;
  const uint64_t w = bit >> 5;
  const unsigned shift = (unsigned)(bit & 31u);
  const uint64_t placed = (uint64_t)(raw & mask_bits(bits)) << shift;
  words[w] |= (uint32_t)placed;
  if (shift + (unsigned)bits > 32u) words[w + 1] |= (uint32_t)(placed >> 32);
}

void orc_pack_dense(int bits, const uint32_t *codes, uint64_t count,
                    uint32_t *words) {
  memset(words, 0, orc_dense_word_count(bits, count) * sizeof(uint32_t));
  for (uint64_t i = 0; i < count; ++i) orc_or_dense(bits, words, i, codes[i]);
}

void orc_unpack_dense(int bits, const uint32_t *words, uint64_t count,
                      uint32_t *codes) {
  for (uint64_t i = 0; i < count; ++i) codes[i] = orc_load_dense(bits, words, i);
}

/* ------------------------------------------------------------------------ */
/* dot_v1 dataset, dot_dataset.hpp:136-214                                   */
/* ------------------------------------------------------------------------ */

uint64_t orc_splitmix64(uint64_t v) {
  v += UINT64_C(0x9e3779b97f4a7c15);
  v = (v ^ (v >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
  v = (v ^ (v >> 27)) * UINT64_C(0x94d049bb133111eb);
  return v ^ (v >> 31);
}

static float positive_mantissa(uint64_t bits) {
  const uint32_t fraction = (uint32_t)(bits >> 41);
  return (float)((UINT32_C(1) << 23) + fraction) * 0x1p-24f;
}

static float signed_unit_f32(uint64_t bits) {
  const uint32_t fraction = (uint32_t)(bits >> 41);
  const int32_t centered = (int32_t)fraction - (1 << 22);
  return (float)centered * 0x1p-22f;
}

static float power_of_two_f32(int exponent) {
  float r = 1.0f;
  if (exponent >= 0)
    for (int i = 0; i < exponent; ++i) r *= 2.0f;
  else
    for (int i = 0; i > exponent; --i) r *= 0.5f;
  return r;
}

static uint64_t lane_seed(uint64_t seed, int vector_id) {
  return seed ^ (UINT64_C(0xd1b54a32d192ed03) * (uint64_t)(vector_id + 1));
}

/* kind: 0 positive_uniform, 1 signed_uniform, 2 controlled_cancellation,
 * 3 dynamic_range (dataset::family order, dot_dataset.hpp:80-85). */
float orc_dot_v1_value(int kind, uint64_t seed, int parameter, int vector_id,
                       uint64_t index, uint64_t count) {
  if (kind != 2) {
    const uint64_t bits = orc_splitmix64(index ^ lane_seed(seed, vector_id));
    if (kind == 0) return positive_mantissa(bits);
    if (kind == 1) return signed_unit_f32(bits);
    const int span = parameter;
    const int exponent =
        (int)((bits >> 1) % (uint64_t)(2 * span + 1)) - span;
    const float sign = (bits & 1u) ? -1.0f : 1.0f;
    return sign * positive_mantissa(bits) * power_of_two_f32(exponent);
  }
  const uint64_t half = count / 2;
  const uint64_t pair = half == 0 ? 0 : index % half;
  const float a = positive_mantissa(
      orc_splitmix64(pair ^ seed ^ UINT64_C(0x243f6a8885a308d3)));
  if (vector_id == 0) return a;
  const float b = positive_mantissa(
      orc_splitmix64(pair ^ seed ^ UINT64_C(0x13198a2e03707344)));
  if (index < half) return b;
  const float residual = power_of_two_f32(-parameter);
  return -b * (1.0f - residual);
}

void orc_dot_v1_fill(int kind, uint64_t seed, int parameter, int vector_id,
                     uint64_t count, float *out) {
  for (uint64_t i = 0; i < count; ++i)
    out[i] = orc_dot_v1_value(kind, seed, parameter, vector_id, i, count);
}

uint64_t orc_fnv1a_f32(const float *values, uint64_t count) {
  uint64_t h = UINT64_C(1469598103934665603);
  for (uint64_t i = 0; i < count; ++i) {
    uint32_t b;
    memcpy(&b, &values[i], sizeof b);
    h ^= b;
    h *= UINT64_C(1099511628211);
  }
  return h;
}

/* ------------------------------------------------------------------------ */
/* synthetic workload generators (restated by the device generator)          */
/* ------------------------------------------------------------------------ */

static double signed_unit_f64(uint64_t bits) { /* dot_bench.cu:389-393 */
  const int64_t fraction = (int64_t)(bits >> 12);
  const int64_t centered = fraction - (INT64_C(1) << 51);
  return (double)centered * 0x1p-51;
}

double orc_synthetic_value(int kind, uint64_t seed, int vector_id,
                           uint64_t index) {
  const uint64_t ls = lane_seed(seed, vector_id);
  switch (kind) {
  case 0:
    return signed_unit_f64(orc_splitmix64(index ^ ls));
  case 1:
    return (double)signed_unit_f32(orc_splitmix64(index ^ ls));
  case 2: {
    uint64_t acc = 0;
    for (uint64_t k = 0; k < 12; ++k)
      acc += orc_splitmix64((index * 12u + k) ^ ls) >> 11;
    return (double)acc * 0x1p-53 - 6.0;
  }
  case 3: {
    const double x = signed_unit_f64(orc_splitmix64(index ^ lane_seed(seed, 0)));
    if (vector_id == 0) return x;
    const double u = signed_unit_f64(orc_splitmix64(index ^ lane_seed(seed, 2)));
    const double t = 1e-6 * u;
    const double scale = 1.0 + t;
    const double p = x * scale;
    return (index & 1u) ? -p : p;
  }
  case 4: /* positive_unit<double>, dot_bench.cu:375-379 */
    return (double)((orc_splitmix64(index ^ ls) >> 11) + 1u) * 0x1p-53;
  default:
    return NAN;
  }
}

void orc_synthetic_fill(int kind, uint64_t seed, int vector_id, uint64_t first,
                        uint64_t count, double *out) {
  for (uint64_t i = 0; i < count; ++i)
    out[i] = orc_synthetic_value(kind, seed, vector_id, first + i);
}

/* ------------------------------------------------------------------------ */
/* compensated long-double reference, dot_bench.cu:532-577                   */
/* ------------------------------------------------------------------------ */

typedef struct {
  long double sum;
  long double correction;
} comp_sum;

static void comp_add(comp_sum *s, long double value) { /* :534-542 */
  const long double updated = s->sum + value;
  if (fabsl(s->sum) >= fabsl(value))
    s->correction += (s->sum - updated) + value;
  else
    s->correction += (value - updated) + s->sum;
  s->sum = updated;
}

static long double comp_value(const comp_sum *s) {
  return s->sum + s->correction;
}

static void split_ld(long double v, double out[2]) {
  const double hi = (double)v;
  out[0] = hi;
  out[1] = (double)(v - (long double)hi);
}

void orc_dot_reference_f64(const double *x, const double *y, uint64_t count,
                           double out_dot[2], double out_sum_abs[2]) {
  comp_sum dot = {0, 0}, sabs = {0, 0};
  for (uint64_t i = 0; i < count; ++i) {
    const long double p = (long double)x[i] * (long double)y[i];
    comp_add(&dot, p);
    comp_add(&sabs, fabsl(p));
  }
  split_ld(comp_value(&dot), out_dot);
  split_ld(comp_value(&sabs), out_sum_abs);
}

void orc_dot_reference_f32(const float *x, const float *y, uint64_t count,
                           double out_dot[2], double out_sum_abs[2]) {
  comp_sum dot = {0, 0}, sabs = {0, 0};
  for (uint64_t i = 0; i < count; ++i) {
    const long double p = (long double)x[i] * (long double)y[i];
    comp_add(&dot, p);
    comp_add(&sabs, fabsl(p));
  }
  split_ld(comp_value(&dot), out_dot);
  split_ld(comp_value(&sabs), out_sum_abs);
}

typedef struct {
  int family, T, E, finite, stride;
  const uint32_t *x, *y; /* codes (stride 0) or dense words */
  uint64_t first, count;
  comp_sum dot, sabs;
} shard_job;

static double decode_any(const shard_job *j, uint32_t raw) {
  return orc_decode_f64(j->family, j->T, j->E, j->finite,
                        raw & mask_bits(j->T));
}

static void *shard_run(void *arg) {
  shard_job *j = (shard_job *)arg;
  comp_sum dot = {0, 0}, sabs = {0, 0};
  for (uint64_t i = j->first; i < j->first + j->count; ++i) {
    long double a, b;
    if (j->family == ORC_FAMILY_RAW_FP64) {
      const uint64_t xa = (uint64_t)j->x[2 * i] | ((uint64_t)j->x[2 * i + 1] << 32);
      const uint64_t yb = (uint64_t)j->y[2 * i] | ((uint64_t)j->y[2 * i + 1] << 32);
      a = (long double)dfrom(xa);
      b = (long double)dfrom(yb);
    } else if (j->stride == 0) {
      a = (long double)decode_any(j, j->x[i]);
      b = (long double)decode_any(j, j->y[i]);
    } else {
      a = (long double)decode_any(j, orc_load_dense(j->stride, j->x, i));
      b = (long double)decode_any(j, orc_load_dense(j->stride, j->y, i));
    }
    const long double p = a * b;
    comp_add(&dot, p);
    comp_add(&sabs, fabsl(p));
  }
  j->dot = dot;
  j->sabs = sabs;
  return NULL;
}

static void run_shards(shard_job *proto, uint64_t count, int threads,
                       double out_dot[2], double out_sum_abs[2]) {
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > count && count > 0) threads = (int)count;
  shard_job *jobs = (shard_job *)calloc((size_t)threads, sizeof(shard_job));
  pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
  const uint64_t per = threads ? count / (uint64_t)threads : 0;
  uint64_t first = 0;
  for (int t = 0; t < threads; ++t) {
    jobs[t] = *proto;
    jobs[t].first = first;
    jobs[t].count = (t == threads - 1) ? count - first : per;
    first += jobs[t].count;
  }
  for (int t = 1; t < threads; ++t)
    pthread_create(&tids[t], NULL, shard_run, &jobs[t]);
  shard_run(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
  /* compensated merge of the shard sums, in shard order */
  comp_sum dot = {0, 0}, sabs = {0, 0};
  for (int t = 0; t < threads; ++t) {
    comp_add(&dot, jobs[t].dot.sum);
    comp_add(&dot, jobs[t].dot.correction);
    comp_add(&sabs, jobs[t].sabs.sum);
    comp_add(&sabs, jobs[t].sabs.correction);
  }
  split_ld(comp_value(&dot), out_dot);
  split_ld(comp_value(&sabs), out_sum_abs);
  free(jobs);
  free(tids);
}

void orc_dot_codes(int family, int T, int E, int finite, const uint32_t *x,
                   const uint32_t *y, uint64_t count, int threads,
                   double out_dot[2], double out_sum_abs[2]) {
  shard_job proto;
  memset(&proto, 0, sizeof proto);
  proto.family = family;
  proto.T = T;
  proto.E = E;
  proto.finite = finite;
  proto.stride = 0;
  proto.x = x;
  proto.y = y;
  run_shards(&proto, count, threads, out_dot, out_sum_abs);
}

void orc_dot_dense(int family, int T, int E, int finite, int stride_bits,
                   const uint32_t *x_words, const uint32_t *y_words,
                   uint64_t count, int threads, double out_dot[2],
                   double out_sum_abs[2]) {
  shard_job proto;
  memset(&proto, 0, sizeof proto);
  proto.family = family;
  proto.T = T;
  proto.E = E;
  proto.finite = finite;
  proto.stride = stride_bits;
  proto.x = x_words;
  proto.y = y_words;
  run_shards(&proto, count, threads, out_dot, out_sum_abs);
}

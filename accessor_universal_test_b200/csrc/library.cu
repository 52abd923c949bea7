// library.cu -- registry, errors, workspace, decode tables and the C ABI.
#include "internal.hpp"

#include "aut/detail/codec_core.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

namespace aut::lib {

aut_status gemv_launch(aut_workspace *ws, int32_t format, int32_t layout, int32_t accum,
                       int32_t strategy, int32_t decoder, const void *matrix,
                       const void *vector, uint64_t rows, uint64_t columns,
                       double *results, void *stream, bool *handled);
aut_status dot_launch(aut_workspace *ws, int32_t format, int32_t layout,
                      int32_t accum, int32_t strategy, int32_t decoder,
                      const void *x, const void *y, uint64_t n, uint32_t batch,
                      const batch_layout &bl, double *results, void *stream,
                      double *partials, unsigned int *tickets,
                      unsigned int *status, int max_blocks_total);
int32_t dot_supported(int32_t format, int32_t layout, int32_t accum);

// ---- format registry ----------------------------------------------------------
// Ids 0..10 are the formats with fused DOT kernels (autdot.h); the rest follow
// the reference's registries (storage_formats.hpp:110-262,
// lns_benchmark_core.hpp:44-61) in order.
namespace {
constexpr int B = AUT_FAMILY_BINARY, X = AUT_FAMILY_FP64_PREFIX,
              L = AUT_FAMILY_LNS;
const format_desc registry[] = {
    {"fp32", AUT_FAMILY_RAW_FP32, 32, 8, 0},
    {"fp64", AUT_FAMILY_RAW_FP64, 64, 11, 0},
    {"e2m3", B, 6, 2, 1},
    {"e8m0", B, 9, 8, 0},
    {"e8m1", B, 10, 8, 0},
    {"e8m3", B, 12, 8, 0},
    {"e8m5", B, 14, 8, 0},
    {"bf16_e8m7", B, 16, 8, 0},
    {"e8m15", B, 24, 8, 0},
    {"lns8_r3", L, 8, 3, 0},
    {"lns16_r11", L, 16, 11, 0},
    {"e0m1", B, 2, 0, 1},   {"e1m0", B, 2, 1, 0},   {"e0m2", B, 3, 0, 1},
    {"e1m1", B, 3, 1, 1},   {"e2m0", B, 3, 2, 0},   {"e0m3", B, 4, 0, 1},
    {"e1m2", B, 4, 1, 1},   {"fp4_e2m1", B, 4, 2, 1}, {"e3m0", B, 4, 3, 0},
    {"e0m4", B, 5, 0, 1},   {"e1m3", B, 5, 1, 1},   {"e2m2", B, 5, 2, 0},
    {"e3m1", B, 5, 3, 0},   {"e4m0", B, 5, 4, 0},   {"e0m5", B, 6, 0, 1},
    {"e1m4", B, 6, 1, 1},   {"e3m2", B, 6, 3, 1},   {"e4m1", B, 6, 4, 0},
    {"e5m0", B, 6, 5, 0},   {"e0m6", B, 7, 0, 1},   {"e2m4", B, 7, 2, 0},
    {"e3m3", B, 7, 3, 0},   {"e5m1", B, 7, 5, 0},   {"e6m0", B, 7, 6, 0},
    {"e0m7", B, 8, 0, 1},   {"e1m6", B, 8, 1, 1},   {"e2m5", B, 8, 2, 0},
    {"e3m4", B, 8, 3, 0},   {"e6m1", B, 8, 6, 0},   {"e7m0", B, 8, 7, 0},
    {"e0m8", B, 9, 0, 1},   {"e2m6", B, 9, 2, 0},   {"e4m4", B, 9, 4, 0},
    {"e5m3", B, 9, 5, 0},   {"e2m7", B, 10, 2, 0},  {"e5m4", B, 10, 5, 0},
    {"e0m11", B, 12, 0, 1}, {"e2m9", B, 12, 2, 0},  {"e5m6", B, 12, 5, 0},
    {"e2m11", B, 14, 2, 0}, {"e5m8", B, 14, 5, 0},  {"e0m15", B, 16, 0, 1},
    {"e1m14", B, 16, 1, 1}, {"e2m13", B, 16, 2, 0}, {"e3m12", B, 16, 3, 0},
    {"e4m11", B, 16, 4, 0}, {"e6m9", B, 16, 6, 0},  {"e7m8", B, 16, 7, 0},
    {"e9m6", B, 16, 9, 0},  {"e10m5", B, 16, 10, 0}, {"e2m14", B, 17, 2, 0},
    {"e5m11", B, 17, 5, 0}, {"e8m8", B, 17, 8, 0},  {"e2m17", B, 20, 2, 0},
    {"e5m14", B, 20, 5, 0}, {"e8m11", B, 20, 8, 0}, {"e0m23", B, 24, 0, 1},
    {"e2m21", B, 24, 2, 0}, {"e5m18", B, 24, 5, 0}, {"e2m25", B, 28, 2, 0},
    {"e4m23", B, 28, 4, 0}, {"e5m22", B, 28, 5, 0}, {"e8m19", B, 28, 8, 0},
    {"e0m31", B, 32, 0, 1}, {"e1m30", B, 32, 1, 1}, {"e2m29", B, 32, 2, 0},
    {"e3m28", B, 32, 3, 0}, {"e4m27", B, 32, 4, 0}, {"e5m26", B, 32, 5, 0},
    {"e6m25", B, 32, 6, 0}, {"e7m24", B, 32, 7, 0}, {"e9m22", B, 32, 9, 0},
    {"e10m21", B, 32, 10, 0},
    {"e11m0", X, 12, 11, 0}, {"e11m2", X, 14, 11, 0}, {"e11m4", X, 16, 11, 0},
    {"e11m5", X, 17, 11, 0}, {"e11m8", X, 20, 11, 0}, {"e11m12", X, 24, 11, 0},
    {"e11m16", X, 28, 11, 0}, {"e11m20", X, 32, 11, 0},
    {"lns4_r0", L, 4, 0, 0},  {"lns4_r1", L, 4, 1, 0},  {"lns6_r2", L, 6, 2, 0},
    {"lns8_r2", L, 8, 2, 0},  {"lns8_r4", L, 8, 4, 0},  {"lns8_r5", L, 8, 5, 0},
    {"lns10_r4", L, 10, 4, 0}, {"lns12_r6", L, 12, 6, 0}, {"lns16_r4", L, 16, 4, 0},
    {"lns16_r7", L, 16, 7, 0}, {"lns16_r10", L, 16, 10, 0},
    {"lns16_r12", L, 16, 12, 0}, {"lns16_r13", L, 16, 13, 0},
    {"lns32_r20", L, 32, 20, 0}, {"lns32_r23", L, 32, 23, 0},
    {"lns32_r28", L, 32, 28, 0},
};
constexpr int registry_size = sizeof(registry) / sizeof(registry[0]);

thread_local std::string last_error;
} // namespace

const format_desc *find_format(int32_t id) {
  return (id >= 0 && id < registry_size) ? &registry[id] : nullptr;
}

int container_bits(const format_desc &f) {
  if (f.family == AUT_FAMILY_RAW_FP64) return 64;
  return f.total_bits <= 8 ? 8 : (f.total_bits <= 16 ? 16 : 32);
}

int stride_bits(const format_desc &f, int layout) {
  if (f.family == AUT_FAMILY_RAW_FP32) return 32;
  if (f.family == AUT_FAMILY_RAW_FP64) return 64;
  return layout == AUT_LAYOUT_DENSE ? f.total_bits : container_bits(f);
}

aut_status fail(aut_status code, const std::string &message) {
  last_error = message;
  return code;
}

aut_status cuda_fail(cudaError_t err, const char *what) {
  last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
               cudaGetErrorString(err) + ")";
  // The error is reported through the returned status; take it out of the
  // runtime's per-thread last-error slot too, so that the caller's next
  // cudaGetLastError (a framework checking its own launches) does not see
  // it.  A sticky error (a lost context) stays whatever is done here.
  (void)cudaGetLastError();
  return AUT_ERR_CUDA;
}

void clear_error() { last_error.clear(); }

const std::string &error_text() { return last_error; }

// ---- host codecs (runtime descriptors) -----------------------------------------
uint32_t encode_host(const format_desc &f, double v) {
  using namespace aut::detail;
  switch (f.family) {
  case AUT_FAMILY_BINARY:
    return f.exponent_bits == 0 ? fixed_encode(f.total_bits, v)
                                : ieee_encode(f.total_bits, f.exponent_bits,
                                              f.finite != 0, v);
  case AUT_FAMILY_FP64_PREFIX: return prefix_encode(f.total_bits - 12, v);
  case AUT_FAMILY_RAW_FP32: {
    const float x = static_cast<float>(v);
    uint32_t b;
    std::memcpy(&b, &x, sizeof b);
    return b;
  }
  case AUT_FAMILY_LNS: {
    // lns_benchmark_core.hpp:194-230 with runtime (B, R).
    const int Bb = f.total_bits, R = f.exponent_bits;
    const uint32_t nan_raw = lns_sign_mask(Bb) | lns_special(Bb);
    const uint32_t zero_raw = lns_special(Bb);
    const int64_t lo = -static_cast<int64_t>(lns_special(Bb)) + 1;
    const int64_t hi = static_cast<int64_t>(lns_special(Bb)) - 1;
    auto make = [&](bool neg, int64_t c) {
      return (neg ? lns_sign_mask(Bb) : 0u) |
             (static_cast<uint32_t>(c) & lns_log_mask(Bb));
    };
    if (v != v) return nan_raw;
    const double big = std::numeric_limits<double>::max();
    if (v > big || v < -big) return make(v < 0.0, hi);
    if (v == 0.0) return zero_raw;
    const bool neg = v < 0.0;
    const double mag = neg ? -v : v;
    const double scaled =
        std::log2(mag) * static_cast<double>(uint64_t{1} << R);
    if (scaled <= static_cast<double>(lo) - 0.5) return zero_raw;
    int64_t r = static_cast<int64_t>(std::nearbyint(scaled));
    r = r < lo ? lo : (r > hi ? hi : r);
    return make(neg, r);
  }
  default: return 0;
  }
}

double decode_host(const format_desc &f, uint32_t raw) {
  using namespace aut::detail;
  switch (f.family) {
  case AUT_FAMILY_BINARY:
    return f.exponent_bits == 0 ? fixed_decode(f.total_bits, raw)
                                : ieee_decode(f.total_bits, f.exponent_bits,
                                              f.finite != 0, raw);
  case AUT_FAMILY_FP64_PREFIX: return prefix_decode(f.total_bits - 12, raw);
  case AUT_FAMILY_RAW_FP32: {
    float x;
    std::memcpy(&x, &raw, sizeof x);
    return x;
  }
  case AUT_FAMILY_LNS: {
    const int Bb = f.total_bits, R = f.exponent_bits;
    raw &= low_mask32(Bb);
    if ((raw & lns_log_mask(Bb)) == lns_special(Bb))
      return (raw & lns_sign_mask(Bb)) ? std::numeric_limits<double>::quiet_NaN()
                                       : 0.0;
    const double v = std::exp2(static_cast<double>(lns_log_code(Bb, raw)) /
                               static_cast<double>(uint32_t{1} << R));
    return (raw & lns_sign_mask(Bb)) ? -v : v;
  }
  default: return std::numeric_limits<double>::quiet_NaN();
  }
}

float decode_host_f32_lns(const format_desc &f, uint32_t raw) {
  using namespace aut::detail;
  const int Bb = f.total_bits, R = f.exponent_bits;
  raw &= low_mask32(Bb);
  if ((raw & lns_log_mask(Bb)) == lns_special(Bb))
    return (raw & lns_sign_mask(Bb)) ? std::numeric_limits<float>::quiet_NaN()
                                     : 0.0f;
  const float v = ::exp2f(static_cast<float>(lns_log_code(Bb, raw)) /
                          static_cast<float>(uint32_t{1} << R));
  return (raw & lns_sign_mask(Bb)) ? -v : v;
}

// ---- LNS tables ------------------------------------------------------------------
namespace {

int32_t lns_code_of(const format_desc &f, double x) {
  return aut::detail::lns_log_code(f.total_bits, encode_host(f, x));
}

// Smallest positive double whose host encoding has a log code above k
// (k = minimum - 1 asks for the smallest magnitude that is not zero).
double switch_point(const format_desc &f, int64_t k, double guess) {
  const uint32_t zero_raw = aut::detail::lns_special(f.total_bits);
  auto above = [&](double x) {
    const uint32_t raw = encode_host(f, x);
    if (raw == zero_raw) return false;
    return static_cast<int64_t>(aut::detail::lns_log_code(f.total_bits, raw)) > k;
  };
  double x = guess;
  int steps = 0;
  if (above(x)) {
    while (steps++ < 4096) {
      const double down = std::nextafter(x, 0.0);
      if (!above(down)) return x;
      x = down;
    }
  } else {
    while (steps++ < 4096) {
      x = std::nextafter(x, std::numeric_limits<double>::infinity());
      if (above(x)) return x;
    }
  }
  // Far from the guess: bisect on the bit pattern (positive doubles order
  // like their bit patterns).
  uint64_t lo_bits = 1, hi_bits = aut::detail::bits_of(std::numeric_limits<double>::max());
  while (lo_bits < hi_bits) {
    const uint64_t mid = lo_bits + (hi_bits - lo_bits) / 2;
    if (above(aut::detail::double_of(mid)))
      hi_bits = mid;
    else
      lo_bits = mid + 1;
  }
  return aut::detail::double_of(lo_bits);
}

aut_status build_code_tables(const format_desc &f, code_tables &t) {
  const int Bb = f.total_bits, R = f.exponent_bits;
  if (f.family != AUT_FAMILY_LNS) {
    // bit formats: the full table of every code (FP32: the value narrowed,
    // exact where the format's values are FP32 values)
    if (Bb > 14) return fail(AUT_ERR_UNSUPPORTED, "decode tables cover bit formats of <= 14 bits");
    const size_t full = size_t{1} << Bb;
    std::vector<float> full32(full);
    std::vector<double> full64(full);
    std::vector<uint32_t> hi(full);
    bool low_words_zero = true;
    for (size_t r = 0; r < full; ++r) {
      full64[r] = decode_host(f, static_cast<uint32_t>(r));
      full32[r] = static_cast<float>(full64[r]);
      uint64_t bits;
      std::memcpy(&bits, &full64[r], sizeof(bits));
      hi[r] = static_cast<uint32_t>(bits >> 32);
      if (static_cast<uint32_t>(bits) != 0u) low_words_zero = false;
    }
    AUT_CUDA_TRY(cudaMalloc(&t.full_f32, full * sizeof(float)));
    AUT_CUDA_TRY(cudaMalloc(&t.full_f64, full * sizeof(double)));
    AUT_CUDA_TRY(cudaMemcpy(t.full_f32, full32.data(), full * sizeof(float), cudaMemcpyHostToDevice));
    AUT_CUDA_TRY(cudaMemcpy(t.full_f64, full64.data(), full * sizeof(double), cudaMemcpyHostToDevice));
    if (Bb > 8 && low_words_zero) {
      AUT_CUDA_TRY(cudaMalloc(&t.full_hi, full * sizeof(uint32_t)));
      AUT_CUDA_TRY(cudaMemcpy(t.full_hi, hi.data(), full * sizeof(uint32_t), cudaMemcpyHostToDevice));
    }
    const int M = Bb - 1 - f.exponent_bits;
    if (f.family == AUT_FAMILY_BINARY && f.exponent_bits == 8 && M >= 1 && M <= 5) {
      // prefix entries: the value of (sign, exponent, mantissa 0) with its
      // fraction bits cleared; subnormal entries: the value of (0, 0, f)
      const uint32_t sub = 1u << M;
      std::vector<uint32_t> part(1024 + 2 * sub);
      for (uint32_t pfx = 0; pfx < 512; ++pfx) {
        const double v = decode_host(f, pfx << M);
        const float v32 = static_cast<float>(v);
        uint32_t b32;
        uint64_t b64;
        std::memcpy(&b32, &v32, sizeof b32);
        std::memcpy(&b64, &v, sizeof b64);
        part[pfx] = b32 & 0xff800000u;
        part[512 + pfx] = static_cast<uint32_t>(b64 >> 32) & 0xfff00000u;
      }
      for (uint32_t fr = 0; fr < sub; ++fr) {
        const double v = decode_host(f, fr);
        const float v32 = static_cast<float>(v);
        uint32_t b32;
        uint64_t b64;
        std::memcpy(&b32, &v32, sizeof b32);
        std::memcpy(&b64, &v, sizeof b64);
        part[1024 + fr] = b32;
        part[1024 + sub + fr] = static_cast<uint32_t>(b64 >> 32);
      }
      AUT_CUDA_TRY(cudaMalloc(&t.part, part.size() * sizeof(uint32_t)));
      AUT_CUDA_TRY(cudaMemcpy(t.part, part.data(), part.size() * sizeof(uint32_t),
                              cudaMemcpyHostToDevice));
      t.part_sub_entries = sub;
    }
    t.ready = 1;
    return AUT_OK;
  }
  if (Bb > 16)
    return fail(AUT_ERR_UNSUPPORTED, "device LNS tables cover B <= 16 bits");
  const size_t full = size_t{1} << Bb;
  const size_t frac = size_t{1} << R;
  std::vector<float> full32(full), frac32(frac);
  std::vector<double> full64(full), frac64(frac);
  for (size_t r = 0; r < full; ++r) {
    full32[r] = decode_host_f32_lns(f, static_cast<uint32_t>(r));
    full64[r] = decode_host(f, static_cast<uint32_t>(r));
  }
  for (size_t k = 0; k < frac; ++k) {
    frac32[k] = ::exp2f(static_cast<float>(k) / static_cast<float>(frac));
    frac64[k] = std::exp2(static_cast<double>(k) / static_cast<double>(frac));
  }
  // The fraction-table kernels decode +-2^q * T[f] with an exponent add;
  // record whether this host's libm makes that identical to the full decode
  // (the full-table kernels serve the format either way).
  t.split_f32 = t.split_f64 = 1;
  for (size_t r = 0; r < full; ++r) {
    const uint32_t raw = static_cast<uint32_t>(r);
    if ((raw & aut::detail::lns_log_mask(Bb)) == aut::detail::lns_special(Bb)) continue;
    const int32_t c = aut::detail::lns_log_code(Bb, raw);
    const int q = c >> R;
    const uint32_t fi = static_cast<uint32_t>(c) & static_cast<uint32_t>(frac - 1);
    const float s32 = std::ldexp(frac32[fi], q);
    const double s64 = std::ldexp(frac64[fi], q);
    const bool neg = (raw & aut::detail::lns_sign_mask(Bb)) != 0;
    if ((neg ? -s32 : s32) != full32[r]) t.split_f32 = 0;
    if ((neg ? -s64 : s64) != full64[r]) t.split_f64 = 0;
  }
  // Encode thresholds: thr[j] = smallest magnitude with log code > min + j.
  const int64_t lo = -static_cast<int64_t>(aut::detail::lns_special(Bb)) + 1;
  const int64_t hi = static_cast<int64_t>(aut::detail::lns_special(Bb)) - 1;
  const double scale = static_cast<double>(uint64_t{1} << R);
  std::vector<double> thr(static_cast<size_t>(hi - lo));
  for (int64_t k = lo; k < hi; ++k)
    thr[static_cast<size_t>(k - lo)] =
        switch_point(f, k, std::exp2((static_cast<double>(k) + 0.5) / scale));
  t.zero_threshold =
      switch_point(f, lo - 1, std::exp2((static_cast<double>(lo) - 0.5) / scale));
  (void)lns_code_of;

  AUT_CUDA_TRY(cudaMalloc(&t.full_f32, full * sizeof(float)));
  AUT_CUDA_TRY(cudaMalloc(&t.full_f64, full * sizeof(double)));
  AUT_CUDA_TRY(cudaMalloc(&t.frac_f32, frac * sizeof(float)));
  AUT_CUDA_TRY(cudaMalloc(&t.frac_f64, frac * sizeof(double)));
  AUT_CUDA_TRY(cudaMalloc(&t.thresholds, thr.size() * sizeof(double)));
  if (Bb <= 12) {
    // The fused-sum table (src/lns_strategy_bench.cu:359-374): the product of
    // two finite codes has a log in [-2 m, 2 m], m = 2^(B-2) - 1; the slots no
    // product reaches hold the nearest reachable magnitude.
    const int64_t m = static_cast<int64_t>(aut::detail::lns_special(Bb)) - 1;
    const int64_t bias = int64_t{1} << (Bb - 1);
    std::vector<float> prod32(full);
    std::vector<double> prod64(full);
    for (size_t i = 0; i < full; ++i) {
      int64_t lg = static_cast<int64_t>(i) - bias;
      lg = lg < -2 * m ? -2 * m : (lg > 2 * m ? 2 * m : lg);
      prod64[i] = std::exp2(static_cast<double>(lg) / scale);
      prod32[i] = static_cast<float>(prod64[i]);
    }
    AUT_CUDA_TRY(cudaMalloc(&t.prod_f32, full * sizeof(float)));
    AUT_CUDA_TRY(cudaMalloc(&t.prod_f64, full * sizeof(double)));
    AUT_CUDA_TRY(cudaMemcpy(t.prod_f32, prod32.data(), full * sizeof(float), cudaMemcpyHostToDevice));
    AUT_CUDA_TRY(cudaMemcpy(t.prod_f64, prod64.data(), full * sizeof(double), cudaMemcpyHostToDevice));
  }
  AUT_CUDA_TRY(cudaMemcpy(t.full_f32, full32.data(), full * sizeof(float), cudaMemcpyHostToDevice));
  AUT_CUDA_TRY(cudaMemcpy(t.full_f64, full64.data(), full * sizeof(double), cudaMemcpyHostToDevice));
  AUT_CUDA_TRY(cudaMemcpy(t.frac_f32, frac32.data(), frac * sizeof(float), cudaMemcpyHostToDevice));
  AUT_CUDA_TRY(cudaMemcpy(t.frac_f64, frac64.data(), frac * sizeof(double), cudaMemcpyHostToDevice));
  AUT_CUDA_TRY(cudaMemcpy(t.thresholds, thr.data(), thr.size() * sizeof(double), cudaMemcpyHostToDevice));
  t.ready = 1;
  return AUT_OK;
}

void free_code_tables(code_tables &t) {
  cudaFree(t.full_f32);
  cudaFree(t.full_f64);
  cudaFree(t.full_hi);
  cudaFree(t.part);
  cudaFree(t.frac_f32);
  cudaFree(t.frac_f64);
  cudaFree(t.prod_f32);
  cudaFree(t.prod_f64);
  cudaFree(t.thresholds);
  t = code_tables{};
}

// Makes ws->device current for the scope of a call and restores the caller's.
struct device_scope {
  int previous = -1;
  cudaError_t err = cudaSuccess;
  explicit device_scope(int device) {
    err = cudaGetDevice(&previous);
    if (err == cudaSuccess && previous != device) err = cudaSetDevice(device);
    else if (err == cudaSuccess) previous = -1;
  }
  ~device_scope() {
    if (previous >= 0) cudaSetDevice(previous);
  }
};

} // namespace

aut_status code_tables_for(aut_workspace *ws, int32_t format_id,
                          const code_tables **out) {
  const format_desc *f = find_format(format_id);
  if (f == nullptr ||
      !(f->family == AUT_FAMILY_LNS ||
        ((f->family == AUT_FAMILY_BINARY || f->family == AUT_FAMILY_FP64_PREFIX) &&
         f->total_bits <= 14)))
    return fail(AUT_ERR_INVALID_ARGUMENT, "no decode tables for this format");
  std::lock_guard<std::mutex> lock(ws->mutex);
  int slot = -1;
  for (int k = 0; k < kTableFormatsCached; ++k) {
    if (ws->table_ids[k] == format_id) {
      *out = &ws->tables[k];
      return AUT_OK;
    }
    if (slot < 0 && ws->table_ids[k] < 0) slot = k;
  }
  if (slot < 0) return fail(AUT_ERR_TOO_LARGE, "too many table-decoded formats in one workspace");
  const aut_status st = build_code_tables(*f, ws->tables[slot]);
  if (st != AUT_OK) {
    free_code_tables(ws->tables[slot]);
    return st;
  }
  ws->table_ids[slot] = format_id;
  *out = &ws->tables[slot];
  return AUT_OK;
}

// Device codec launchers (codec.cu).
aut_status launch_encode(aut_workspace *ws, const format_desc &f, int32_t format,
                         int32_t layout, const double *values, uint64_t n,
                         void *codes, cudaStream_t stream);
aut_status launch_decode(aut_workspace *ws, const format_desc &f, int32_t format,
                         int32_t layout, int32_t target, const void *codes,
                         uint64_t n, void *out, cudaStream_t stream);
aut_status launch_generate(int32_t kind, uint64_t seed, int32_t vector_id,
                           uint64_t first, uint64_t n, double *out,
                           cudaStream_t stream);
aut_status launch_generate_dot_v1(int32_t family, uint64_t seed, int32_t parameter,
                                  int32_t vector_id, uint64_t count, uint64_t first,
                                  uint64_t n, float *out, cudaStream_t stream);

} // namespace aut::lib

// ================================================================================
// C ABI
// ================================================================================
using namespace aut::lib;

extern "C" {

const char *aut_version(void) { return "autdot 0.1 (sm_100a)"; }
int32_t aut_abi_version(void) { return AUTDOT_ABI_VERSION; }
const char *aut_last_error(void) { return error_text().c_str(); }

int32_t aut_format_count(void) {
  int32_t n = 0;
  while (find_format(n) != nullptr) ++n;
  return n;
}

int32_t aut_format_id(const char *name) {
  if (name == nullptr) return -1;
  for (int32_t k = 0; find_format(k) != nullptr; ++k)
    if (std::strcmp(find_format(k)->name, name) == 0) return k;
  return -1;
}

const char *aut_format_name(int32_t format) {
  const format_desc *f = find_format(format);
  return f ? f->name : nullptr;
}

aut_status aut_format_info(int32_t format, int32_t *family, int32_t *total_bits,
                           int32_t *exponent_bits, int32_t *finite) {
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (family) *family = f->family;
  if (total_bits) *total_bits = f->total_bits;
  if (exponent_bits) *exponent_bits = f->exponent_bits;
  if (finite) *finite = f->finite;
  return AUT_OK;
}

int32_t aut_dot_supported(int32_t format, int32_t layout, int32_t accum) {
  return dot_supported(format, layout, accum);
}

uint64_t aut_storage_bytes(int32_t format, int32_t layout, uint64_t n) {
  const format_desc *f = find_format(format);
  if (f == nullptr) return 0;
  if (f->family == AUT_FAMILY_RAW_FP32) return n * 4;
  if (f->family == AUT_FAMILY_RAW_FP64) return n * 8;
  if (layout == AUT_LAYOUT_DENSE)
    return 4 * ((n * static_cast<uint64_t>(f->total_bits) + 31) / 32 + 1);
  return n * static_cast<uint64_t>(container_bits(*f) / 8);
}

double aut_packed_bytes(int32_t format, uint64_t n) {
  const format_desc *f = find_format(format);
  if (f == nullptr) return 0.0;
  return static_cast<double>(n) * f->total_bits / 8.0;
}

aut_status aut_workspace_create(int32_t device, aut_workspace **out) {
  clear_error();
  if (out == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
    return fail(AUT_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= count)
    return fail(AUT_ERR_INVALID_ARGUMENT, "device index out of range");
  device_scope scope(device);
  AUT_CUDA_TRY(scope.err);
  cudaDeviceProp prop{};
  AUT_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(AUT_ERR_NO_DEVICE, std::string("libautdot is built for sm_100a; device is sm_") +
                                       std::to_string(prop.major) + std::to_string(prop.minor));
  auto *ws = new aut_workspace();
  ws->device = device;
  ws->sm_count = prop.multiProcessorCount;
  ws->max_blocks = prop.multiProcessorCount * (prop.maxThreadsPerMultiProcessor / 256);
  const size_t np = static_cast<size_t>(kMaxBatchPerLaunch) * ws->max_blocks;
  const size_t nt = 2 * static_cast<size_t>(kMaxBatchPerLaunch) + 1;
  cudaError_t e = cudaMalloc(&ws->partials, np * sizeof(double));
  if (e == cudaSuccess) e = cudaMalloc(&ws->tickets, nt * sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(ws->tickets, 0, nt * sizeof(unsigned int));
  if (e == cudaSuccess) ws->claims = ws->tickets + kMaxBatchPerLaunch + 1;
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(ws->partials);
    cudaFree(ws->tickets);
    delete ws;
    return cuda_fail(e, "workspace allocation");
  }
  *out = ws;
  return AUT_OK;
}

aut_status aut_workspace_destroy(aut_workspace *ws) {
  if (ws == nullptr) return AUT_OK;
  {
    device_scope scope(ws->device);
    for (int k = 0; k < kTableFormatsCached; ++k)
      if (ws->table_ids[k] >= 0) free_code_tables(ws->tables[k]);
    cudaFree(ws->partials);
    cudaFree(ws->tickets);
  }
  delete ws;
  return AUT_OK;
}

aut_status aut_workspace_prepare(aut_workspace *ws, int32_t format) {
  clear_error();
  if (ws == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "workspace is NULL");
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  // bit formats with a table decoder: codes of at most 8 bits, and the E8
  // codes of 9 to 14 bits (FULL_LUT)
  const bool wide_e8 = format == AUT_FMT_E8M0 || format == AUT_FMT_E8M1 ||
                       format == AUT_FMT_E8M3 || format == AUT_FMT_E8M5;
  const bool narrow_bits = (f->total_bits <= 8 || wide_e8) &&
                           (f->family == AUT_FAMILY_BINARY ||
                            f->family == AUT_FAMILY_FP64_PREFIX);
  if (f->family != AUT_FAMILY_LNS && !narrow_bits) return AUT_OK;
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  const code_tables *t = nullptr;
  return code_tables_for(ws, format, &t);
}

aut_status aut_workspace_info(const aut_workspace *ws, int32_t *sm_count,
                              int32_t *max_blocks) {
  if (ws == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "workspace is NULL");
  if (sm_count) *sm_count = ws->sm_count;
  if (max_blocks) *max_blocks = ws->max_blocks;
  return AUT_OK;
}

aut_status aut_workspace_status(aut_workspace *ws, uint32_t *status,
                                int32_t clear) {
  clear_error();
  if (ws == nullptr || status == nullptr)
    return fail(AUT_ERR_INVALID_ARGUMENT, "workspace or status is NULL");
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  AUT_CUDA_TRY(cudaDeviceSynchronize());
  unsigned int word = 0;
  AUT_CUDA_TRY(cudaMemcpy(&word, ws->tickets + kMaxBatchPerLaunch, sizeof word,
                          cudaMemcpyDeviceToHost));
  *status = word;
  if (clear && word != 0)
    AUT_CUDA_TRY(cudaMemset(ws->tickets + kMaxBatchPerLaunch, 0, sizeof word));
  return AUT_OK;
}

aut_status aut_workspace_inject_stall(aut_workspace *ws, uint64_t stall_tile,
                                      uint64_t wait_cycles) {
  clear_error();
  if (ws == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "workspace is NULL");
  if (wait_cycles > static_cast<uint64_t>(aut::kWaitCyclesDefault))
    return fail(AUT_ERR_INVALID_ARGUMENT, "wait_cycles above the default bound");
  ws->stall_tile = stall_tile;
  ws->wait_cycles = wait_cycles == 0 ? aut::kWaitCyclesDefault
                                     : static_cast<long long>(wait_cycles);
  return AUT_OK;
}

static aut_status check_dot_args(aut_workspace *ws, int32_t format,
                                 int32_t layout, int32_t accum, const void *x,
                                 const void *y, uint64_t n, const double *res) {
  if (ws == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "workspace is NULL");
  if (find_format(format) == nullptr)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (layout != AUT_LAYOUT_DENSE && layout != AUT_LAYOUT_PADDED)
    return fail(AUT_ERR_INVALID_ARGUMENT, "layout must be DENSE or PADDED");
  if (accum != AUT_ACCUM_FP32 && accum != AUT_ACCUM_FP64)
    return fail(AUT_ERR_INVALID_ARGUMENT, "accum must be FP32 or FP64");
  if (res == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "result is NULL");
  if (n > 0 && (x == nullptr || y == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "x or y is NULL");
  if (!dot_supported(format, layout, accum))
    return fail(AUT_ERR_UNSUPPORTED,
                std::string("no fused DOT kernel for ") + find_format(format)->name);
  return AUT_OK;
}

aut_status aut_dot(aut_workspace *ws, int32_t format, int32_t layout,
                   int32_t accum, const void *x, const void *y, uint64_t n,
                   double *result, void *stream) {
  return aut_dot_strategy(ws, format, layout, accum, AUT_STRATEGY_AUTO, x, y,
                          n, result, stream);
}

aut_status aut_dot_strategy(aut_workspace *ws, int32_t format, int32_t layout,
                            int32_t accum, int32_t strategy, const void *x,
                            const void *y, uint64_t n, double *result,
                            void *stream) {
  return aut_dot_variant(ws, format, layout, accum, strategy, AUT_DECODER_AUTO,
                         x, y, n, result, stream);
}

aut_status aut_dot_variant(aut_workspace *ws, int32_t format, int32_t layout,
                           int32_t accum, int32_t strategy, int32_t decoder,
                           const void *x, const void *y, uint64_t n,
                           double *result, void *stream) {
  clear_error();
  aut_status st = check_dot_args(ws, format, layout, accum, x, y, n, result);
  if (st != AUT_OK) return st;
  if (strategy < AUT_STRATEGY_AUTO || strategy > AUT_STRATEGY_COOPERATIVE)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown access strategy");
  if (decoder < AUT_DECODER_AUTO || decoder > AUT_DECODER_SUBNORMAL_LUT)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown decoder");
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  return dot_launch(ws, format, layout, accum, strategy, decoder, x, y, n, 1,
                    batch_layout{}, result, stream, ws->partials, ws->tickets,
                    ws->tickets + kMaxBatchPerLaunch, ws->max_blocks);
}

aut_status aut_dot_batched(aut_workspace *ws, int32_t format, int32_t layout,
                           int32_t accum, const void *x, const void *y,
                           uint64_t n, uint32_t batch,
                           uint64_t batch_stride_bytes, double *results,
                           void *stream) {
  clear_error();
  aut_status st = check_dot_args(ws, format, layout, accum, x, y, n, results);
  if (st != AUT_OK) return st;
  if (batch == 0) return AUT_OK;
  if (batch > 1 && batch_stride_bytes < aut_storage_bytes(format, layout, n))
    return fail(AUT_ERR_INVALID_ARGUMENT, "batch stride smaller than one vector");
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  batch_layout bl;
  bl.x_stride = bl.y_stride = batch_stride_bytes;
  return dot_launch(ws, format, layout, accum, AUT_STRATEGY_AUTO,
                    AUT_DECODER_AUTO, x, y, n, batch, bl,
                    results, stream, ws->partials,
                    ws->tickets, ws->tickets + kMaxBatchPerLaunch,
                    ws->max_blocks);
}

aut_status aut_gemv(aut_workspace *ws, int32_t format, int32_t layout,
                    int32_t accum, int32_t strategy, int32_t decoder,
                    const void *matrix, const void *vector, uint64_t rows,
                    uint64_t columns, double *result, void *stream) {
  clear_error();
  aut_status st = check_dot_args(ws, format, layout, accum, matrix, vector,
                                 rows == 0 ? 0 : columns, result);
  if (st != AUT_OK) return st;
  if (strategy < AUT_STRATEGY_AUTO || strategy > AUT_STRATEGY_COOPERATIVE)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown access strategy");
  if (decoder < AUT_DECODER_AUTO || decoder > AUT_DECODER_SUBNORMAL_LUT)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown decoder");
  if (rows == 0) return AUT_OK;
  if (rows > 0xffffffffull)
    return fail(AUT_ERR_TOO_LARGE, "at most 2^32 - 1 rows per call");
  const uint64_t bits = static_cast<uint64_t>(stride_bits(*find_format(format), layout));
  if (columns > (uint64_t{1} << 56) / bits / rows)
    return fail(AUT_ERR_TOO_LARGE, "matrix larger than 2^53 bytes");
  // Row r is the DOT of values [r * columns, (r + 1) * columns) of the matrix
  // stream with the vector: rows that start on 16-byte boundaries are read by
  // byte stride on the vector paths, the others by absolute value index.
  batch_layout bl;
  const uint64_t row_bits = columns * bits;
  if (row_bits % 128 == 0)
    bl.x_stride = row_bits / 8;
  else
    bl.x_index_stride = columns;
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  bool handled = false;
  st = gemv_launch(ws, format, layout, accum, strategy, decoder, matrix, vector, rows,
                   columns, result, stream, &handled);
  if (st != AUT_OK || handled) return st;
  return dot_launch(ws, format, layout, accum, strategy, decoder, matrix, vector,
                    columns, static_cast<uint32_t>(rows), bl, result, stream,
                    ws->partials, ws->tickets, ws->tickets + kMaxBatchPerLaunch,
                    ws->max_blocks);
}

aut_status aut_decode(aut_workspace *ws, int32_t format, int32_t layout,
                      int32_t target, const void *codes, uint64_t n, void *out,
                      void *stream) {
  clear_error();
  if (ws == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "workspace is NULL");
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (target != AUT_TARGET_FP32 && target != AUT_TARGET_FP64)
    return fail(AUT_ERR_INVALID_ARGUMENT, "target must be FP32 or FP64");
  if (layout != AUT_LAYOUT_DENSE && layout != AUT_LAYOUT_PADDED)
    return fail(AUT_ERR_INVALID_ARGUMENT, "layout must be DENSE or PADDED");
  if (n > 0 && (codes == nullptr || out == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "codes or out is NULL");
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  return launch_decode(ws, *f, format, layout, target, codes, n, out,
                       static_cast<cudaStream_t>(stream));
}

aut_status aut_encode(aut_workspace *ws, int32_t format, int32_t layout,
                      const double *values, uint64_t n, void *codes,
                      void *stream) {
  clear_error();
  if (ws == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "workspace is NULL");
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (layout != AUT_LAYOUT_DENSE && layout != AUT_LAYOUT_PADDED)
    return fail(AUT_ERR_INVALID_ARGUMENT, "layout must be DENSE or PADDED");
  if (codes == nullptr || (n > 0 && values == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "values or codes is NULL");
  device_scope scope(ws->device);
  AUT_CUDA_TRY(scope.err);
  return launch_encode(ws, *f, format, layout, values, n, codes,
                       static_cast<cudaStream_t>(stream));
}

aut_status aut_generate(int32_t kind, uint64_t seed, int32_t vector_id,
                        uint64_t first, uint64_t n, double *out, void *stream) {
  clear_error();
  if (kind < AUT_GEN_SIGNED_UNIT_F64 || kind > AUT_GEN_POSITIVE_UNIT_F64)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown generator kind");
  if (n > 0 && out == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "out is NULL");
  return launch_generate(kind, seed, vector_id, first, n, out,
                         static_cast<cudaStream_t>(stream));
}

aut_status aut_generate_dot_v1(int32_t family, uint64_t seed, int32_t parameter,
                               int32_t vector_id, uint64_t count, uint64_t first,
                               uint64_t n, float *out, void *stream) {
  clear_error();
  if (family < 0 || family > 3)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown dataset family");
  if (vector_id != 0 && vector_id != 1)
    return fail(AUT_ERR_INVALID_ARGUMENT, "vector_id must be 0 (x) or 1 (y)");
  if (parameter < 0 || parameter > 126)
    return fail(AUT_ERR_INVALID_ARGUMENT, "parameter must lie in [0, 126]");
  if (first > count || n > count - first)
    return fail(AUT_ERR_INVALID_ARGUMENT, "[first, first + n) beyond the case's count");
  if (n > 0 && out == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "out is NULL");
  return launch_generate_dot_v1(family, seed, parameter, vector_id, count, first, n, out,
                                static_cast<cudaStream_t>(stream));
}

aut_status aut_encode_host(int32_t format, const double *values, uint64_t n,
                           uint32_t *codes) {
  clear_error();
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (f->family == AUT_FAMILY_RAW_FP64)
    return fail(AUT_ERR_UNSUPPORTED, "fp64 codes do not fit 32 bits");
  if (n > 0 && (values == nullptr || codes == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "values or codes is NULL");
  for (uint64_t i = 0; i < n; ++i) codes[i] = encode_host(*f, values[i]);
  return AUT_OK;
}

aut_status aut_decode_host(int32_t format, const uint32_t *codes, uint64_t n,
                           double *out) {
  clear_error();
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (f->family == AUT_FAMILY_RAW_FP64)
    return fail(AUT_ERR_UNSUPPORTED, "fp64 codes do not fit 32 bits");
  if (n > 0 && (codes == nullptr || out == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "codes or out is NULL");
  for (uint64_t i = 0; i < n; ++i) out[i] = decode_host(*f, codes[i]);
  return AUT_OK;
}

aut_status aut_pack_host(int32_t format, int32_t layout, const uint32_t *codes,
                         uint64_t n, void *out) {
  clear_error();
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (f->family == AUT_FAMILY_RAW_FP64)
    return fail(AUT_ERR_UNSUPPORTED, "fp64 codes do not fit 32 bits");
  if (out == nullptr || (n > 0 && codes == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "codes or out is NULL");
  const int bits = stride_bits(*f, layout);
  const uint32_t mask = aut::detail::low_mask32(f->total_bits);
  if (bits == 8 || bits == 16 || bits == 32) {
    for (uint64_t i = 0; i < n; ++i) {
      const uint32_t c = codes[i] & mask;
      if (bits == 8) static_cast<uint8_t *>(out)[i] = static_cast<uint8_t>(c);
      else if (bits == 16) static_cast<uint16_t *>(out)[i] = static_cast<uint16_t>(c);
      else static_cast<uint32_t *>(out)[i] = c;
    }
    if (layout == AUT_LAYOUT_DENSE && f->family != AUT_FAMILY_RAW_FP32) {
      // the guard word after the data
      const uint64_t words = (n * bits + 31) / 32;
      static_cast<uint32_t *>(out)[words] = 0u;
      if (bits != 32 && (n * bits) % 32 != 0) {
        // zero the unused tail of the last data word
        const uint64_t used_bytes = n * bits / 8;
        std::memset(static_cast<uint8_t *>(out) + used_bytes, 0, words * 4 - used_bytes);
      }
    }
    return AUT_OK;
  }
  uint32_t *w = static_cast<uint32_t *>(out);
  const uint64_t words = (n * bits + 31) / 32 + 1;
  std::memset(w, 0, words * 4);
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t bit = i * bits;
    const uint64_t k = bit >> 5;
    const unsigned sh = static_cast<unsigned>(bit & 31u);
    const uint64_t placed = static_cast<uint64_t>(codes[i] & mask) << sh;
    w[k] |= static_cast<uint32_t>(placed);
    if (sh + bits > 32) w[k + 1] |= static_cast<uint32_t>(placed >> 32);
  }
  return AUT_OK;
}

aut_status aut_unpack_host(int32_t format, int32_t layout, const void *packed,
                           uint64_t n, uint32_t *codes) {
  clear_error();
  const format_desc *f = find_format(format);
  if (f == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (f->family == AUT_FAMILY_RAW_FP64)
    return fail(AUT_ERR_UNSUPPORTED, "fp64 codes do not fit 32 bits");
  if (n > 0 && (packed == nullptr || codes == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "packed or codes is NULL");
  const int bits = stride_bits(*f, layout);
  const uint32_t mask = aut::detail::low_mask32(f->total_bits);
  for (uint64_t i = 0; i < n; ++i) {
    if (bits == 8) codes[i] = static_cast<const uint8_t *>(packed)[i] & mask;
    else if (bits == 16) codes[i] = static_cast<const uint16_t *>(packed)[i] & mask;
    else if (bits == 32) codes[i] = static_cast<const uint32_t *>(packed)[i] & mask;
    else {
      const uint32_t *w = static_cast<const uint32_t *>(packed);
      const uint64_t bit = i * bits;
      const uint64_t k = bit >> 5;
      const unsigned sh = static_cast<unsigned>(bit & 31u);
      const uint64_t pair = static_cast<uint64_t>(w[k]) |
                            (sh + bits > 32 ? static_cast<uint64_t>(w[k + 1]) << 32 : 0);
      codes[i] = static_cast<uint32_t>(pair >> sh) & mask;
    }
  }
  return AUT_OK;
}

} // extern "C"

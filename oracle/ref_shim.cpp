// ref_shim.cpp -- exposes the reference's OWN host code through a C ABI.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile against the
// reference's headers where they lie (REF/include, REF/tools) into
// oracle/_ref/libautref.so.  Nothing here re-implements an algorithm: every
// function forwards to the reference's templates:
//   aut::storage::encode/decode          include/storage_formats.hpp:603-614
//   aut::bitwidth::load/or_dense_scalar  include/bitwidth_benchmark_core.hpp:135-158
//   aut::lns::encode/decode              include/lns_benchmark_core.hpp:179-230
//   aut::dataset::value                  include/dot_dataset.hpp:191-214
//   compensated_sum                      tools/inspect_dot_dataset.cpp:17-34
// The oracle restatement (oracle.c) is checked bit-for-bit against this
// library, and bench.py's reference arm times the reference's CPU path
// (host decode + compensated long-double DOT) through autref_dot_dense.

#include "storage_formats.hpp"
#include "bitwidth_benchmark_core.hpp"
#include "lns_benchmark_core.hpp"
#include "dot_dataset.hpp"

// tools/inspect_dot_dataset.cpp keeps compensated_sum in an anonymous
// namespace next to its main(); include it with main renamed so the class
// is the reference's own code.
#define main aut_reference_dataset_inspect_main
#include "inspect_dot_dataset.cpp"
#undef main

#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <utility>
#include <vector>

namespace {

namespace st = aut::storage;
namespace bw = aut::bitwidth;
namespace ln = aut::lns;

enum family { binary = 0, prefix = 1, lns = 2 };

struct format_entry {
  const char *name;
  int family;
  int total_bits;
  int exponent_bits; // LNS: log fraction bits
  int finite;
  std::uint32_t (*encode)(double);
  double (*decode64)(std::uint32_t);
  float (*decode32)(std::uint32_t);
};

template <typename F> std::uint32_t enc_bin(double v) {
  return static_cast<std::uint32_t>(st::encode<F>(v));
}
template <typename F> double dec_bin(std::uint32_t raw) {
  return st::decode<F>(static_cast<st::storage_type_t<F>>(raw));
}
template <typename F> float dec_bin32(std::uint32_t raw) {
  return static_cast<float>(dec_bin<F>(raw));
}
template <typename F> std::uint32_t enc_lns(double v) {
  return ln::encode<F>(v);
}
template <typename F> double dec_lns(std::uint32_t raw) {
  return ln::decode<F, double>(raw);
}
template <typename F> float dec_lns32(std::uint32_t raw) {
  return ln::decode<F, float>(raw);
}

#define AUT_BIN(name_)                                                        \
  format_entry{#name_,          binary,           st::name_::total_bits,     \
               st::name_::exponent_bits, st::name_::finite ? 1 : 0,           \
               enc_bin<st::name_>, dec_bin<st::name_>, dec_bin32<st::name_>}
#define AUT_PREFIX(name_)                                                     \
  format_entry{#name_,          prefix,           st::name_::total_bits, 11,  \
               0,               enc_bin<st::name_>, dec_bin<st::name_>,       \
               dec_bin32<st::name_>}
#define AUT_LNS(name_)                                                        \
  format_entry{#name_,          lns,              ln::name_::total_bits,     \
               ln::name_::log_fraction_bits, 0, enc_lns<ln::name_>,           \
               dec_lns<ln::name_>, dec_lns32<ln::name_>}

// bf16_e8m7 lives in cuda_storage_formats.cuh behind CUDA's bf16 type; its
// bit layout is binary_format<16, 8, false>, whose generic codec is used here.
using bf16_layout = st::binary_format<16, 8, false>;
const format_entry bf16_entry{"bf16_e8m7",         binary, 16, 8, 0,
                              enc_bin<bf16_layout>, dec_bin<bf16_layout>,
                              dec_bin32<bf16_layout>};

const format_entry formats[] = {
    AUT_BIN(e0m1),  AUT_BIN(e1m0),   AUT_BIN(e0m2),   AUT_BIN(e1m1),
    AUT_BIN(e2m0),  AUT_BIN(e0m3),   AUT_BIN(e1m2),   AUT_BIN(fp4_e2m1),
    AUT_BIN(e3m0),  AUT_BIN(e0m4),   AUT_BIN(e1m3),   AUT_BIN(e2m2),
    AUT_BIN(e3m1),  AUT_BIN(e4m0),   AUT_BIN(e0m5),   AUT_BIN(e1m4),
    AUT_BIN(e2m3),  AUT_BIN(e3m2),   AUT_BIN(e4m1),   AUT_BIN(e5m0),
    AUT_BIN(e0m6),  AUT_BIN(e2m4),   AUT_BIN(e3m3),   AUT_BIN(e5m1),
    AUT_BIN(e6m0),  AUT_BIN(e0m7),   AUT_BIN(e1m6),   AUT_BIN(e2m5),
    AUT_BIN(e3m4),  AUT_BIN(e6m1),   AUT_BIN(e7m0),   AUT_BIN(e0m8),
    AUT_BIN(e2m6),  AUT_BIN(e4m4),   AUT_BIN(e5m3),   AUT_BIN(e8m0),
    AUT_BIN(e2m7),  AUT_BIN(e5m4),   AUT_BIN(e8m1),   AUT_BIN(e0m11),
    AUT_BIN(e2m9),  AUT_BIN(e5m6),   AUT_BIN(e8m3),   AUT_BIN(e2m11),
    AUT_BIN(e5m8),  AUT_BIN(e8m5),   AUT_BIN(e0m15),  AUT_BIN(e1m14),
    AUT_BIN(e2m13), AUT_BIN(e3m12),  AUT_BIN(e4m11),  AUT_BIN(e6m9),
    AUT_BIN(e7m8),  AUT_BIN(e9m6),   AUT_BIN(e10m5),  AUT_BIN(e2m14),
    AUT_BIN(e5m11), AUT_BIN(e8m8),   AUT_BIN(e2m17),  AUT_BIN(e5m14),
    AUT_BIN(e8m11), AUT_BIN(e0m23),  AUT_BIN(e2m21),  AUT_BIN(e5m18),
    AUT_BIN(e8m15), AUT_BIN(e2m25),  AUT_BIN(e4m23),  AUT_BIN(e5m22),
    AUT_BIN(e8m19), AUT_BIN(e0m31),  AUT_BIN(e1m30),  AUT_BIN(e2m29),
    AUT_BIN(e3m28), AUT_BIN(e4m27),  AUT_BIN(e5m26),  AUT_BIN(e6m25),
    AUT_BIN(e7m24), AUT_BIN(e9m22),  AUT_BIN(e10m21), bf16_entry,
    AUT_PREFIX(e11m0), AUT_PREFIX(e11m2), AUT_PREFIX(e11m4),
    AUT_PREFIX(e11m5), AUT_PREFIX(e11m8), AUT_PREFIX(e11m12),
    AUT_PREFIX(e11m16), AUT_PREFIX(e11m20),
    AUT_LNS(lns4_r0), AUT_LNS(lns4_r1), AUT_LNS(lns6_r2), AUT_LNS(lns8_r2),
    AUT_LNS(lns8_r3), AUT_LNS(lns8_r4), AUT_LNS(lns8_r5), AUT_LNS(lns10_r4),
    AUT_LNS(lns12_r6), AUT_LNS(lns16_r4), AUT_LNS(lns16_r7),
    AUT_LNS(lns16_r10), AUT_LNS(lns16_r11), AUT_LNS(lns16_r12),
    AUT_LNS(lns16_r13), AUT_LNS(lns32_r20), AUT_LNS(lns32_r23),
    AUT_LNS(lns32_r28),
};
constexpr int format_count = sizeof(formats) / sizeof(formats[0]);

template <int Bits>
std::uint32_t load_bits(const std::uint32_t *words, std::size_t i) {
  return bw::load_dense_scalar<Bits>(words, i);
}
template <int Bits>
void or_bits(std::uint32_t *words, std::size_t i, std::uint32_t raw) {
  bw::or_dense_scalar<Bits>(words, i, raw);
}

using load_fn = std::uint32_t (*)(const std::uint32_t *, std::size_t);
using or_fn = void (*)(std::uint32_t *, std::size_t, std::uint32_t);

template <int... B>
constexpr std::array<load_fn, sizeof...(B)> make_loads(std::integer_sequence<int, B...>) {
  return {load_bits<B + 2>...};
}
template <int... B>
constexpr std::array<or_fn, sizeof...(B)> make_ors(std::integer_sequence<int, B...>) {
  return {or_bits<B + 2>...};
}
const auto loads = make_loads(std::make_integer_sequence<int, 31>{});
const auto ors = make_ors(std::make_integer_sequence<int, 31>{});

void split(long double v, double out[2]) {
  const double hi = static_cast<double>(v);
  out[0] = hi;
  out[1] = static_cast<double>(v - static_cast<long double>(hi));
}

} // namespace

extern "C" {

int autref_format_count() { return format_count; }

const char *autref_format_name(int i) {
  if (i < 0 || i >= format_count) return nullptr;
  return formats[i].name;
}

void autref_format_desc(int i, int *family, int *total_bits,
                        int *exponent_bits, int *finite) {
  const auto &f = formats[i];
  *family = f.family;
  *total_bits = f.total_bits;
  *exponent_bits = f.exponent_bits;
  *finite = f.finite;
}

std::uint32_t autref_encode(int i, double v) { return formats[i].encode(v); }
double autref_decode_f64(int i, std::uint32_t raw) {
  return formats[i].decode64(raw);
}
float autref_decode_f32(int i, std::uint32_t raw) {
  return formats[i].decode32(raw);
}

void autref_encode_array(int i, const double *v, std::uint64_t n,
                         std::uint32_t *out) {
  for (std::uint64_t k = 0; k < n; ++k) out[k] = formats[i].encode(v[k]);
}
void autref_decode_array_f64(int i, const std::uint32_t *raw, std::uint64_t n,
                             double *out) {
  for (std::uint64_t k = 0; k < n; ++k) out[k] = formats[i].decode64(raw[k]);
}
void autref_decode_array_f32(int i, const std::uint32_t *raw, std::uint64_t n,
                             float *out) {
  for (std::uint64_t k = 0; k < n; ++k) out[k] = formats[i].decode32(raw[k]);
}

std::uint64_t autref_dense_word_count(int bits, std::uint64_t n) {
  // dense_word_count is a template over Bits; every width shares one formula.
  switch (bits) {
  case 6: return bw::dense_word_count<6>(n);
  case 9: return bw::dense_word_count<9>(n);
  case 24: return bw::dense_word_count<24>(n);
  default: return (n * static_cast<std::uint64_t>(bits) + 31u) / 32u + 1u;
  }
}

void autref_pack_dense(int bits, const std::uint32_t *codes, std::uint64_t n,
                       std::uint32_t *words, std::uint64_t word_count) {
  std::memset(words, 0, word_count * sizeof(std::uint32_t));
  const auto put = ors[bits - 2];
  for (std::uint64_t k = 0; k < n; ++k) put(words, k, codes[k]);
}

std::uint32_t autref_load_dense(int bits, const std::uint32_t *words,
                                std::uint64_t i) {
  return loads[bits - 2](words, i);
}

int autref_dot_v1_case_count() {
  return static_cast<int>(aut::dataset::accuracy_cases.size());
}
const char *autref_dot_v1_case_id(int c) {
  return aut::dataset::accuracy_cases[c].id;
}
void autref_dot_v1_fill(int c, int vector_id, std::uint64_t count,
                        float *out) {
  const auto spec = aut::dataset::accuracy_cases[c].values;
  for (std::uint64_t k = 0; k < count; ++k)
    out[k] = aut::dataset::value(spec, vector_id, k, count);
}

// The reference's CPU path for a DOT over stored vectors: host decode of
// both operands (storage::decode / lns::decode) and the compensated long
// double sum, split over `threads` contiguous shards whose (sum, |sum|)
// pairs are merged with the same compensated_sum.
void autref_dot_dense(int i, int stride_bits, const std::uint32_t *x,
                      const std::uint32_t *y, std::uint64_t n, int threads,
                      double out_dot[2], double out_sum_abs[2]) {
  if (threads < 1) threads = 1;
  const auto load = loads[stride_bits - 2];
  const auto decode = formats[i].decode64;
  const std::uint32_t mask = formats[i].total_bits >= 32
                                 ? 0xffffffffu
                                 : (1u << formats[i].total_bits) - 1u;
  std::vector<compensated_sum> dots(threads), sabs(threads);
  std::vector<std::thread> pool;
  const std::uint64_t per = n / static_cast<std::uint64_t>(threads);
  auto work = [&](int t) {
    const std::uint64_t first = per * t;
    const std::uint64_t last = t == threads - 1 ? n : first + per;
    compensated_sum d, a;
    for (std::uint64_t k = first; k < last; ++k) {
      const auto xv = static_cast<long double>(decode(load(x, k) & mask));
      const auto yv = static_cast<long double>(decode(load(y, k) & mask));
      const auto p = xv * yv;
      d.add(p);
      a.add(std::fabs(p));
    }
    dots[t] = d;
    sabs[t] = a;
  };
  for (int t = 1; t < threads; ++t) pool.emplace_back(work, t);
  work(0);
  for (auto &th : pool) th.join();
  compensated_sum d, a;
  for (int t = 0; t < threads; ++t) {
    d.add(dots[t].value());
    a.add(sabs[t].value());
  }
  split(d.value(), out_dot);
  split(a.value(), out_sum_abs);
}

// Same CPU path for raw FP32 / FP64 storage (src/dot_bench.cu:551-577).
void autref_dot_raw(int is_fp64, const void *x, const void *y,
                    std::uint64_t n, int threads, double out_dot[2],
                    double out_sum_abs[2]) {
  if (threads < 1) threads = 1;
  std::vector<compensated_sum> dots(threads), sabs(threads);
  std::vector<std::thread> pool;
  const std::uint64_t per = n / static_cast<std::uint64_t>(threads);
  auto work = [&](int t) {
    const std::uint64_t first = per * t;
    const std::uint64_t last = t == threads - 1 ? n : first + per;
    compensated_sum d, a;
    for (std::uint64_t k = first; k < last; ++k) {
      long double xv, yv;
      if (is_fp64) {
        xv = static_cast<const double *>(x)[k];
        yv = static_cast<const double *>(y)[k];
      } else {
        xv = static_cast<const float *>(x)[k];
        yv = static_cast<const float *>(y)[k];
      }
      const auto p = xv * yv;
      d.add(p);
      a.add(std::fabs(p));
    }
    dots[t] = d;
    sabs[t] = a;
  };
  for (int t = 1; t < threads; ++t) pool.emplace_back(work, t);
  work(0);
  for (auto &th : pool) th.join();
  compensated_sum d, a;
  for (int t = 0; t < threads; ++t) {
    d.add(dots[t].value());
    a.add(sabs[t].value());
  }
  split(d.value(), out_dot);
  split(a.value(), out_sum_abs);
}

} // extern "C"

// aut/dot_dataset.hpp -- the dot_v1 validation datasets (host + device).
//
// Drop-in for the reference's include/dot_dataset.hpp: the same case table
// (ids, families, seeds, parameters; :18-70) and the same counter-based
// generators (:72-152), so that every index of every case is reproducible on
// the host and on the GPU and the published fingerprints and reference DOTs
// (datasets/dot_v1/validation_n1048576.csv) hold for data made here.  The
// values must agree bit for bit with the reference's, so each generator
// performs the same float operations in the same order:
//   positive_uniform        1.m with 23 random fraction bits, scaled by 1/2
//   signed_uniform          a 23-bit random integer centred on 0, * 2^-22
//   controlled_cancellation x_i = a_p, y_i = b_p for the first half and
//                           -b_p (1 - 2^-parameter) for the second, p the
//                           index within a half: the DOT cancels to about
//                           sum a b 2^-parameter
//   dynamic_range           +-positive_uniform * 2^e, e uniform in
//                           [-parameter, parameter]
#ifndef AUT_DOT_DATASET_HPP_
#define AUT_DOT_DATASET_HPP_

#include "detail/codec_core.hpp"

#include <array>
#include <cstddef>
#include <cstdint>

namespace aut::dataset {

enum class family : std::uint8_t {
  positive_uniform,
  signed_uniform,
  controlled_cancellation,
  dynamic_range
};

struct parameters {
  family kind{};
  std::uint64_t seed{};
  int parameter{};
};

struct case_spec {
  const char *id;
  parameters values;
  const char *purpose;
};

inline constexpr std::uint64_t base_seed = 0x123456789abcdef0ULL;

inline constexpr case_spec performance_case{
    "signed_uniform_seed0", {family::signed_uniform, base_seed, 0},
    "signed uniform FP32 values: the throughput case"};

inline constexpr std::array<case_spec, 9> accuracy_cases{{
    {"positive_uniform", {family::positive_uniform, base_seed, 0},
     "all products positive (condition number 1)"},
    {"signed_uniform_seed0", {family::signed_uniform, base_seed, 0},
     "independent signed values, seed 0"},
    {"signed_uniform_seed1", {family::signed_uniform, 0x8c3c010cb4754c9dULL, 0},
     "independent signed values, seed 1"},
    {"signed_uniform_seed2", {family::signed_uniform, 0xd2b74407b1ce6e93ULL, 0},
     "independent signed values, seed 2"},
    {"cancellation_1e2", {family::controlled_cancellation, base_seed, 6},
     "halves that cancel: condition number about 2^7"},
    {"cancellation_1e4", {family::controlled_cancellation, base_seed, 13},
     "halves that cancel: condition number about 2^14"},
    {"cancellation_1e6", {family::controlled_cancellation, base_seed, 19},
     "halves that cancel: condition number about 2^20"},
    {"near_orthogonal", {family::controlled_cancellation, base_seed, 22},
     "halves that cancel: condition number about 2^23"},
    {"dynamic_range_40", {family::dynamic_range, 0xa4093822299f31d0ULL, 20},
     "signed values with exponents spread over [-20, 20]"},
}};

AUT_HD AUT_INLINE std::uint64_t splitmix64(std::uint64_t v) {
  v += 0x9e3779b97f4a7c15ULL;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ULL;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebULL;
  return v ^ (v >> 31);
}

// [0.5, 1): the top 23 bits of `bits` below an implicit leading one, / 2^24
AUT_HD AUT_INLINE float positive_mantissa(std::uint64_t bits) {
  const std::uint32_t fraction = static_cast<std::uint32_t>(bits >> 41);
  return static_cast<float>((1u << 23) + fraction) * 0x1p-24f;
}

// [-1, 1) in steps of 2^-22
AUT_HD AUT_INLINE float signed_unit(std::uint64_t bits) {
  const std::int32_t centred =
      static_cast<std::int32_t>(static_cast<std::uint32_t>(bits >> 41)) - (1 << 22);
  return static_cast<float>(centred) * 0x1p-22f;
}

// 2^e as a float, built by repeated exact doubling or halving
AUT_HD AUT_INLINE float power_of_two(int e) {
  float r = 1.0f;
  for (; e > 0; --e) r *= 2.0f;
  for (; e < 0; ++e) r *= 0.5f;
  return r;
}

AUT_HD AUT_INLINE float independent_value(std::uint64_t index, std::uint64_t seed,
                                          int vector_id, family kind, int parameter) {
  const std::uint64_t lane =
      seed ^ (0xd1b54a32d192ed03ULL * static_cast<std::uint64_t>(vector_id + 1));
  const std::uint64_t bits = splitmix64(index ^ lane);
  if (kind == family::positive_uniform) return positive_mantissa(bits);
  if (kind == family::signed_uniform) return signed_unit(bits);
  // dynamic range: exponent from the bits above the sign bit
  const int e = static_cast<int>((bits >> 1) % static_cast<std::uint64_t>(2 * parameter + 1)) -
                parameter;
  const float sign = (bits & 1ULL) ? -1.0f : 1.0f;
  return sign * positive_mantissa(bits) * power_of_two(e);
}

// Value `index` of vector `vector_id` (0: x, 1: y) of a case with `count`
// values in all.
AUT_HD AUT_INLINE float value(parameters spec, int vector_id, std::uint64_t index,
                              std::uint64_t count) {
  if (spec.kind != family::controlled_cancellation)
    return independent_value(index, spec.seed, vector_id, spec.kind, spec.parameter);
  const std::uint64_t half = count / 2;
  const std::uint64_t pair = half == 0 ? 0 : index % half;
  const float a = positive_mantissa(splitmix64(pair ^ spec.seed ^ 0x243f6a8885a308d3ULL));
  if (vector_id == 0) return a;
  const float b = positive_mantissa(splitmix64(pair ^ spec.seed ^ 0x13198a2e03707344ULL));
  if (index < half) return b;
  return -b * (1.0f - power_of_two(-spec.parameter));
}

} // namespace aut::dataset

#endif

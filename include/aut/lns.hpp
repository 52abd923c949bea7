// aut/lns.hpp -- logarithmic number storage (host + device).
//
// Drop-in for the reference's include/lns_benchmark_core.hpp:28-272: a
// B-bit code is a sign bit plus an R-fraction-bit two's-complement log2 of
// the magnitude; the most negative log code is reserved (+ = zero, - = NaN).
// decode<F, T> returns +-2^(code / 2^R) computed with the target type's exp2
// (exp2f for float, exp2 for double) and encode rounds log2|v| * 2^R to the
// nearest integer, saturating at the largest code and flushing values at or
// below half a step under the smallest code to zero.
#ifndef AUT_LNS_HPP_
#define AUT_LNS_HPP_

#include "detail/codec_core.hpp"

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <type_traits>

namespace aut::lns {

template <int Bits, int FractionBits> struct format {
  static_assert(Bits >= 2 && Bits <= 32);
  static_assert(FractionBits >= 0 && FractionBits < Bits - 1);
  static constexpr int total_bits = Bits;
  static constexpr int log_fraction_bits = FractionBits;
  static constexpr int log_integer_bits = Bits - 1 - FractionBits;
  static constexpr int exponent_bits = log_integer_bits;
  static constexpr int fraction_bits = log_fraction_bits;
};

#define AUT_LNS_FORMAT(name_, bits_, frac_)                                   \
  struct name_ : format<bits_, frac_> {                                      \
    static constexpr const char *name = #name_;                              \
  }
AUT_LNS_FORMAT(lns4_r0, 4, 0);    AUT_LNS_FORMAT(lns4_r1, 4, 1);
AUT_LNS_FORMAT(lns6_r2, 6, 2);    AUT_LNS_FORMAT(lns8_r2, 8, 2);
AUT_LNS_FORMAT(lns8_r3, 8, 3);    AUT_LNS_FORMAT(lns8_r4, 8, 4);
AUT_LNS_FORMAT(lns8_r5, 8, 5);    AUT_LNS_FORMAT(lns10_r4, 10, 4);
AUT_LNS_FORMAT(lns12_r6, 12, 6);  AUT_LNS_FORMAT(lns16_r4, 16, 4);
AUT_LNS_FORMAT(lns16_r7, 16, 7);  AUT_LNS_FORMAT(lns16_r10, 16, 10);
AUT_LNS_FORMAT(lns16_r11, 16, 11); AUT_LNS_FORMAT(lns16_r12, 16, 12);
AUT_LNS_FORMAT(lns16_r13, 16, 13); AUT_LNS_FORMAT(lns32_r20, 32, 20);
AUT_LNS_FORMAT(lns32_r23, 32, 23); AUT_LNS_FORMAT(lns32_r28, 32, 28);
#undef AUT_LNS_FORMAT

template <typename F> AUT_HD AUT_INLINE constexpr std::uint32_t raw_mask() {
  return aut::detail::low_mask32(F::total_bits);
}
template <typename F> AUT_HD AUT_INLINE constexpr std::uint32_t log_mask() {
  return aut::detail::lns_log_mask(F::total_bits);
}
template <typename F> AUT_HD AUT_INLINE constexpr std::uint32_t sign_mask() {
  return aut::detail::lns_sign_mask(F::total_bits);
}
template <typename F>
AUT_HD AUT_INLINE constexpr std::uint32_t special_log_code() {
  return aut::detail::lns_special(F::total_bits);
}
template <typename F>
AUT_HD AUT_INLINE constexpr std::int32_t minimum_finite_log_code() {
  return -static_cast<std::int32_t>(special_log_code<F>()) + 1;
}
template <typename F>
AUT_HD AUT_INLINE constexpr std::int32_t maximum_finite_log_code() {
  return static_cast<std::int32_t>(special_log_code<F>()) - 1;
}
template <typename F> AUT_HD AUT_INLINE bool is_special(std::uint32_t raw) {
  return (raw & log_mask<F>()) == special_log_code<F>();
}
template <typename F> AUT_HD AUT_INLINE bool is_zero(std::uint32_t raw) {
  return is_special<F>(raw) && (raw & sign_mask<F>()) == 0;
}
template <typename F> AUT_HD AUT_INLINE bool is_nan(std::uint32_t raw) {
  return is_special<F>(raw) && (raw & sign_mask<F>()) != 0;
}
template <typename F> AUT_HD AUT_INLINE bool sign(std::uint32_t raw) {
  return (raw & sign_mask<F>()) != 0;
}
template <typename F> AUT_HD AUT_INLINE std::int32_t log_code(std::uint32_t raw) {
  return aut::detail::lns_log_code(F::total_bits, raw);
}
template <typename F>
AUT_HD AUT_INLINE std::uint32_t make_raw(bool negative, std::int32_t code) {
  return (negative ? sign_mask<F>() : 0u) |
         (static_cast<std::uint32_t>(code) & log_mask<F>());
}
template <typename F> AUT_HD AUT_INLINE std::uint32_t zero_raw() {
  return special_log_code<F>();
}
template <typename F> AUT_HD AUT_INLINE std::uint32_t nan_raw() {
  return sign_mask<F>() | special_log_code<F>();
}

template <typename F, typename Target>
AUT_HD AUT_INLINE Target decode(std::uint32_t raw) {
  raw &= raw_mask<F>();
  if (is_zero<F>(raw)) return Target{0};
  if (is_nan<F>(raw)) return std::numeric_limits<Target>::quiet_NaN();
  constexpr Target scale =
      static_cast<Target>(std::uint32_t{1} << F::log_fraction_bits);
  Target v;
  if constexpr (std::is_same_v<Target, float>)
    v = ::exp2f(static_cast<float>(log_code<F>(raw)) / scale);
  else
    v = ::exp2(static_cast<double>(log_code<F>(raw)) / scale);
  return sign<F>(raw) ? -v : v;
}

// Host encode.  Device code encodes LNS through the threshold tables of the
// C ABI (aut_encode), because device log2 rounds differently from the host's.
template <typename F, typename Source>
inline std::uint32_t encode(Source value) {
  const double wide = static_cast<double>(value);
  if (wide != wide) return nan_raw<F>();
  constexpr double big = std::numeric_limits<double>::max();
  if (wide > big || wide < -big)
    return make_raw<F>(value < Source{0}, maximum_finite_log_code<F>());
  if (value == Source{0}) return zero_raw<F>();
  const bool negative = value < Source{0};
  const double magnitude = negative ? -wide : wide;
  const double scaled =
      std::log2(magnitude) *
      static_cast<double>(std::uint64_t{1} << F::log_fraction_bits);
  const auto lo = static_cast<std::int64_t>(minimum_finite_log_code<F>());
  const auto hi = static_cast<std::int64_t>(maximum_finite_log_code<F>());
  if (scaled <= static_cast<double>(lo) - 0.5) return zero_raw<F>();
  auto r = static_cast<std::int64_t>(std::nearbyint(scaled));
  r = r < lo ? lo : (r > hi ? hi : r);
  return make_raw<F>(negative, static_cast<std::int32_t>(r));
}

// A fused product adds two finite log codes, each within +-(special - 1), so
// the sum lies in [-(2 special - 2), 2 special - 2]; biased by 2 special - 2
// it indexes a table of 4 special - 3 <= 2^B entries (product_log_bias /
// product_log_entries, lns_benchmark_core.hpp:108-121).
template <typename F>
AUT_HD AUT_INLINE constexpr std::int32_t product_log_bias() {
  return 2 * static_cast<std::int32_t>(special_log_code<F>()) - 2;
}
template <typename F>
AUT_HD AUT_INLINE constexpr std::size_t product_log_entries() {
  return std::size_t{1} << F::total_bits;
}

template <typename F> struct product_code {
  bool negative{};
  bool zero{};
  bool nan{};
  std::int64_t log{};
};

template <typename F>
AUT_HD AUT_INLINE product_code<F> multiply_codes(std::uint32_t a,
                                                 std::uint32_t b) {
  if (is_nan<F>(a) || is_nan<F>(b)) return {false, false, true, 0};
  if (is_zero<F>(a) || is_zero<F>(b)) return {sign<F>(a) != sign<F>(b), true, false, 0};
  return {sign<F>(a) != sign<F>(b), false, false,
          static_cast<std::int64_t>(log_code<F>(a)) +
              static_cast<std::int64_t>(log_code<F>(b))};
}

// The value of a product code: +-2^(log / 2^R) in the target type (one
// exp2 of the summed logs, so one rounding instead of two), signed zero, or
// NaN (decode_product / multiply_fused, lns_benchmark_core.hpp:256-272).
template <typename F, typename Target>
AUT_HD AUT_INLINE Target decode_product(product_code<F> p) {
  if (p.nan) return std::numeric_limits<Target>::quiet_NaN();
  if (p.zero) return p.negative ? -Target{0} : Target{0};
  constexpr Target scale = static_cast<Target>(std::uint32_t{1} << F::log_fraction_bits);
  Target v;
  if constexpr (std::is_same_v<Target, float>)
    v = ::exp2f(static_cast<float>(p.log) / scale);
  else
    v = ::exp2(static_cast<double>(p.log) / scale);
  return p.negative ? -v : v;
}

template <typename F, typename Target>
AUT_HD AUT_INLINE Target multiply_fused(std::uint32_t a, std::uint32_t b) {
  return decode_product<F, Target>(multiply_codes<F>(a, b));
}

} // namespace aut::lns

#endif

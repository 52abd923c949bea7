// aut/decoder.hpp -- scalar decode strategies of one stored code (host + device).
//
// Drop-in for the reference's include/decoder_strategy_core.hpp interface:
// the binary_layout<T, E, policy> descriptors with the reference's layout
// names (:18-67), and decoders that turn one code into a binary64 value,
// each exact (bit-identical to storage::decode):
//   decode_words_branchy  field-by-field with branches        (:191-226)
//   decode_words_masked   the same cases selected by masks    (:228-262)
//   decode_via_fp32       an FP32 bit move + one power-of-two  (:297-353)
//                         multiply, widened (E <= 8, M <= 23)
//   decode_fixed_integer  E = 0:  magnitude * 2^-M             (:362-375)
//   decode_e1_integer     E = 1, finite: integer * 2^(1-M)    (:377-390)
//   decode_exponent_only  M = 0:  2^(e - bias)                (:392-405)
//   decode_prefix_words   FP64 prefix: the code is the top bits (:264-272)
// The word-returning decoders give the binary64 as two 32-bit words (what
// a GPU assembles before one move into a double register).
#ifndef AUT_DECODER_HPP_
#define AUT_DECODER_HPP_

#include "detail/codec_core.hpp"

#include <cstdint>

namespace aut::decoder {

enum class special_policy { ieee, finite_all, fixed_e0, e4m3fn, fp64_prefix };

template <int TotalBits, int ExponentBits, special_policy Policy>
struct binary_layout {
  static_assert(TotalBits >= 2 && TotalBits <= 32);
  static_assert(ExponentBits >= 0 && ExponentBits < TotalBits);
  static constexpr int total_bits = TotalBits;
  static constexpr int exponent_bits = ExponentBits;
  static constexpr int fraction_bits = TotalBits - 1 - ExponentBits;
  static constexpr special_policy policy = Policy;
  // E = 0 fixed point reads as a subnormal-only format with bias 1
  static constexpr int bias = ExponentBits == 0 ? 1 : (1 << (ExponentBits - 1)) - 1;
};

// The reference's named layouts.
using e0m1_layout = binary_layout<2, 0, special_policy::fixed_e0>;
using e1m0_layout = binary_layout<2, 1, special_policy::ieee>;
using e0m3_layout = binary_layout<4, 0, special_policy::fixed_e0>;
using e1m2_layout = binary_layout<4, 1, special_policy::finite_all>;
using fp4_e2m1_layout = binary_layout<4, 2, special_policy::finite_all>;
using e3m0_layout = binary_layout<4, 3, special_policy::ieee>;
using e0m7_layout = binary_layout<8, 0, special_policy::fixed_e0>;
using e1m6_layout = binary_layout<8, 1, special_policy::finite_all>;
using e2m5_layout = binary_layout<8, 2, special_policy::ieee>;
using e3m4_layout = binary_layout<8, 3, special_policy::ieee>;
using fp8_e4m3_layout = binary_layout<8, 4, special_policy::e4m3fn>;
using fp8_e5m2_layout = binary_layout<8, 5, special_policy::ieee>;
using e6m1_layout = binary_layout<8, 6, special_policy::ieee>;
using e7m0_layout = binary_layout<8, 7, special_policy::ieee>;
using e0m15_layout = binary_layout<16, 0, special_policy::fixed_e0>;
using e1m14_layout = binary_layout<16, 1, special_policy::finite_all>;
using e2m13_layout = binary_layout<16, 2, special_policy::ieee>;
using e3m12_layout = binary_layout<16, 3, special_policy::ieee>;
using e4m11_layout = binary_layout<16, 4, special_policy::ieee>;
using fp16_e5m10_layout = binary_layout<16, 5, special_policy::ieee>;
using e6m9_layout = binary_layout<16, 6, special_policy::ieee>;
using e7m8_layout = binary_layout<16, 7, special_policy::ieee>;
using bf16_e8m7_layout = binary_layout<16, 8, special_policy::ieee>;
using e9m6_layout = binary_layout<16, 9, special_policy::ieee>;
using e10m5_layout = binary_layout<16, 10, special_policy::ieee>;
using e11m4_layout = binary_layout<16, 11, special_policy::fp64_prefix>;
using e0m31_layout = binary_layout<32, 0, special_policy::fixed_e0>;
using e1m30_layout = binary_layout<32, 1, special_policy::finite_all>;
using e2m29_layout = binary_layout<32, 2, special_policy::ieee>;
using e3m28_layout = binary_layout<32, 3, special_policy::ieee>;
using e4m27_layout = binary_layout<32, 4, special_policy::ieee>;
using e5m26_layout = binary_layout<32, 5, special_policy::ieee>;
using e6m25_layout = binary_layout<32, 6, special_policy::ieee>;
using e7m24_layout = binary_layout<32, 7, special_policy::ieee>;
using fp32_e8m23_layout = binary_layout<32, 8, special_policy::ieee>;
using e9m22_layout = binary_layout<32, 9, special_policy::ieee>;
using e10m21_layout = binary_layout<32, 10, special_policy::ieee>;
using e11m20_layout = binary_layout<32, 11, special_policy::fp64_prefix>;

// A binary64 as its high and low 32-bit words.
struct fp64_words {
  std::uint32_t high;
  std::uint32_t low;
};

AUT_HD AUT_INLINE double words_to_double(fp64_words w) {
  return aut::detail::double_of((static_cast<std::uint64_t>(w.high) << 32) | w.low);
}

AUT_HD AUT_INLINE float bits_to_float(std::uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(b);
#else
  float f;
  std::memcpy(&f, &b, sizeof f);
  return f;
#endif
}

AUT_HD AUT_INLINE std::uint32_t float_to_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  std::uint32_t b;
  std::memcpy(&b, &f, sizeof b);
  return b;
#endif
}

namespace detail {
AUT_HD AUT_INLINE constexpr fp64_words split(std::uint64_t b) {
  return {static_cast<std::uint32_t>(b >> 32), static_cast<std::uint32_t>(b)};
}
constexpr std::uint64_t kExpInfNan = std::uint64_t{0x7ff} << 52;
constexpr std::uint64_t kQuietNan = kExpInfNan | (std::uint64_t{1} << 51);

// Is (e, f) the layout's infinity/NaN encoding?  (ieee: top exponent;
// e4m3fn: only the all-ones code, which is NaN.)
template <class L>
AUT_HD AUT_INLINE bool is_inf_nan(std::uint32_t e, std::uint32_t f) {
  constexpr std::uint32_t emax = (1u << L::exponent_bits) - 1u;
  constexpr std::uint32_t fmax = aut::detail::low_mask32(L::fraction_bits);
  if constexpr (L::policy == special_policy::ieee) return e == emax;
  else if constexpr (L::policy == special_policy::e4m3fn) return e == emax && f == fmax;
  else return false;
}

// Binary64 bits of the magnitude m * 2^(1 - bias - M) for 0 < m < 2^M (the
// subnormal range, and all of E = 0 fixed point).
template <class L>
AUT_HD AUT_INLINE std::uint64_t small_magnitude(std::uint32_t m) {
  constexpr int M = L::fraction_bits;
  const int lead = aut::detail::top_bit(m);
  const std::uint64_t exponent =
      static_cast<std::uint64_t>(lead + 1 - L::bias - M + 1023);
  const std::uint64_t fraction =
      (static_cast<std::uint64_t>(m) ^ (std::uint64_t{1} << lead)) << (52 - lead);
  return (exponent << 52) | fraction;
}
} // namespace detail

template <class L>
AUT_HD AUT_INLINE fp64_words decode_words_branchy(std::uint32_t raw) {
  static_assert(L::policy != special_policy::fp64_prefix,
                "FP64 prefixes decode with decode_prefix_words");
  constexpr int T = L::total_bits, E = L::exponent_bits, M = L::fraction_bits;
  raw &= aut::detail::low_mask32(T);
  const std::uint64_t sign = static_cast<std::uint64_t>(raw >> (T - 1)) << 63;
  const std::uint32_t f = raw & aut::detail::low_mask32(M);
  const std::uint32_t e = E == 0 ? 0u : (raw >> M) & aut::detail::low_mask32(E);
  if (e == 0) {
    if (f == 0) return detail::split(sign);
    return detail::split(sign | detail::small_magnitude<L>(f));
  }
  if (detail::is_inf_nan<L>(e, f)) {
    if constexpr (L::policy == special_policy::e4m3fn) return detail::split(sign | detail::kQuietNan);
    return detail::split(sign | detail::kExpInfNan |
                         (static_cast<std::uint64_t>(f) << (52 - M)));
  }
  const std::uint64_t exponent = static_cast<std::uint64_t>(static_cast<int>(e) - L::bias + 1023);
  return detail::split(sign | (exponent << 52) | (static_cast<std::uint64_t>(f) << (52 - M)));
}

template <class L>
AUT_HD AUT_INLINE fp64_words decode_words_masked(std::uint32_t raw) {
  static_assert(L::policy != special_policy::fp64_prefix,
                "FP64 prefixes decode with decode_prefix_words");
  constexpr int T = L::total_bits, E = L::exponent_bits, M = L::fraction_bits;
  raw &= aut::detail::low_mask32(T);
  const std::uint64_t sign = static_cast<std::uint64_t>(raw >> (T - 1)) << 63;
  const std::uint32_t f = raw & aut::detail::low_mask32(M);
  const std::uint32_t e = E == 0 ? 0u : (raw >> M) & aut::detail::low_mask32(E);
  // every case computed, one selected: m_sub (e = 0, f != 0), m_zero
  // (e = 0, f = 0), m_special (inf / NaN), m_normal (the rest)
  const std::uint64_t sub =
      detail::small_magnitude<L>(f | static_cast<std::uint32_t>(f == 0));  // f = 0: masked
  const std::uint64_t special =
      L::policy == special_policy::e4m3fn
          ? detail::kQuietNan
          : detail::kExpInfNan | (static_cast<std::uint64_t>(f) << (52 - M));
  const std::uint64_t normal =
      (static_cast<std::uint64_t>(static_cast<int>(e) - L::bias + 1023) << 52) |
      (static_cast<std::uint64_t>(f) << (52 - M));
  const std::uint64_t m_e0 = 0 - static_cast<std::uint64_t>(e == 0);
  const std::uint64_t m_f0 = 0 - static_cast<std::uint64_t>(f == 0);
  const std::uint64_t m_special = 0 - static_cast<std::uint64_t>(detail::is_inf_nan<L>(e, f));
  const std::uint64_t magnitude = (sub & m_e0 & ~m_f0) | (special & ~m_e0 & m_special) |
                                  (normal & ~m_e0 & ~m_special);
  return detail::split(sign | magnitude);
}

// The code moved into FP32 bit positions (exponent field on FP32's, fraction
// at its top), rebiased by one exact multiply by 2^(127 - bias) -- the
// hardware's subnormal arithmetic covers e = 0 -- with inf/NaN built
// explicitly where the layout has them.  Returns the FP32 bit pattern.
template <class L>
AUT_HD AUT_INLINE std::uint32_t decode_fp32_bits(std::uint32_t raw) {
  constexpr int T = L::total_bits, E = L::exponent_bits, M = L::fraction_bits;
  static_assert(E <= 8 && M <= 23 && L::policy != special_policy::fp64_prefix,
                "the layout's values are not all FP32 values");
  raw &= aut::detail::low_mask32(T);
  const std::uint32_t sign = (raw >> (T - 1)) << 31;
  const std::uint32_t magnitude = raw & aut::detail::low_mask32(T - 1);
  if constexpr (E == 0) {
    // fixed point: magnitude * 2^-M, exact while the magnitude fits 24 bits
    const float scale = bits_to_float(static_cast<std::uint32_t>(127 - M) << 23);
    return sign | float_to_bits(static_cast<float>(magnitude) * scale);
  } else {
    const std::uint32_t f = magnitude & aut::detail::low_mask32(M);
    const std::uint32_t e = magnitude >> M;
    if (detail::is_inf_nan<L>(e, f)) {
      if constexpr (L::policy == special_policy::e4m3fn) return sign | 0x7fc00000u;
      return sign | 0x7f800000u | (f << (23 - M));
    }
    const float placed = bits_to_float(magnitude << (23 - M));
    if constexpr (E == 8) {
      return sign | float_to_bits(placed);
    } else {
      const float rebias = bits_to_float(static_cast<std::uint32_t>(127 - L::bias + 127) << 23);
      return sign | float_to_bits(placed * rebias);
    }
  }
}

template <class L>
AUT_HD AUT_INLINE double decode_via_fp32(std::uint32_t raw) {
  return static_cast<double>(bits_to_float(decode_fp32_bits<L>(raw)));
}

template <class L>
AUT_HD AUT_INLINE double decode_fixed_integer(std::uint32_t raw) {
  static_assert(L::policy == special_policy::fixed_e0);
  constexpr int T = L::total_bits, M = L::fraction_bits;
  raw &= aut::detail::low_mask32(T);
  const double scale = aut::detail::double_of(static_cast<std::uint64_t>(1023 - M) << 52);
  const double v = static_cast<double>(raw & aut::detail::low_mask32(T - 1)) * scale;
  return (raw >> (T - 1)) ? -v : v;
}

template <class L>
AUT_HD AUT_INLINE double decode_e1_integer(std::uint32_t raw) {
  static_assert(L::policy == special_policy::finite_all && L::exponent_bits == 1);
  constexpr int T = L::total_bits, M = L::fraction_bits;
  raw &= aut::detail::low_mask32(T);
  // with one exponent bit and bias 0 the exponent and fraction fields read
  // together are the integer significand: value = field * 2^(1 - M)
  const double scale = aut::detail::double_of(static_cast<std::uint64_t>(1023 + 1 - M) << 52);
  const double v = static_cast<double>(raw & aut::detail::low_mask32(T - 1)) * scale;
  return (raw >> (T - 1)) ? -v : v;
}

template <class L>
AUT_HD AUT_INLINE double decode_exponent_only(std::uint32_t raw) {
  static_assert(L::fraction_bits == 0 && L::policy == special_policy::ieee);
  constexpr int T = L::total_bits, E = L::exponent_bits;
  raw &= aut::detail::low_mask32(T);
  const std::uint64_t sign = static_cast<std::uint64_t>(raw >> (T - 1)) << 63;
  const std::uint32_t e = raw & aut::detail::low_mask32(E);
  if (e == 0) return aut::detail::double_of(sign);
  if (e == aut::detail::low_mask32(E)) return aut::detail::double_of(sign | detail::kExpInfNan);
  return aut::detail::double_of(
      sign | (static_cast<std::uint64_t>(static_cast<int>(e) - L::bias + 1023) << 52));
}

template <int FractionBits>
AUT_HD AUT_INLINE fp64_words decode_prefix_words(std::uint32_t raw) {
  static_assert(FractionBits >= 0 && FractionBits <= 20);
  const std::uint64_t code = raw & aut::detail::low_mask32(12 + FractionBits);
  return detail::split(code << (52 - FractionBits));
}

} // namespace aut::decoder

#endif

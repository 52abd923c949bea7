// aut/storage_formats.hpp -- compact storage formats, host + device.
//
// Drop-in for the reference's include/storage_formats.hpp interface:
// binary_format<T, E, Finite>, the named format registry, codec<F>,
// storage_type_t<F>, encode<F>(double) and decode<F>(storage_type_t<F>)
// (storage_formats.hpp:95-103, :110-262, :603-614).  Round-to-nearest-even
// encode from binary64 with gradual underflow; exact decode to binary64.
// Finite formats saturate; the others keep inf and NaN.
#ifndef AUT_STORAGE_FORMATS_HPP_
#define AUT_STORAGE_FORMATS_HPP_

#include "detail/codec_core.hpp"

#include <cstdint>
#include <type_traits>

namespace aut::storage {

namespace detail {
template <int Bits> struct uint_for {
  static_assert(Bits >= 2 && Bits <= 32, "storage formats span 2..32 bits");
  using type = std::conditional_t<
      (Bits <= 8), std::uint8_t,
      std::conditional_t<(Bits <= 16), std::uint16_t, std::uint32_t>>;
};
} // namespace detail

template <int TotalBits, int ExponentBits, bool Finite> struct binary_format {
  static_assert(TotalBits >= 2 && TotalBits <= 32);
  static_assert(ExponentBits >= 0 && ExponentBits <= 11);
  static_assert(ExponentBits < TotalBits);
  static constexpr int total_bits = TotalBits;
  static constexpr int exponent_bits = ExponentBits;
  static constexpr int fraction_bits = TotalBits - ExponentBits - 1;
  static constexpr bool finite = Finite;
};

template <int FractionBits> struct fp64_prefix {
  static_assert(FractionBits >= 0 && FractionBits <= 20);
  static constexpr int total_bits = 12 + FractionBits;
  static constexpr int exponent_bits = 11;
  static constexpr int fraction_bits = FractionBits;
  static constexpr bool finite = false;
  static constexpr bool is_prefix = true;
};

#define AUT_FORMAT(name_, bits_, exp_, finite_)                               \
  struct name_ : binary_format<bits_, exp_, finite_> {                       \
    static constexpr const char *name = #name_;                              \
  }
#define AUT_PREFIX_FORMAT(name_, frac_)                                       \
  struct name_ : fp64_prefix<frac_> {                                        \
    static constexpr const char *name = #name_;                              \
  }

// The registry: every named layout of the reference, same name, same layout.
AUT_FORMAT(e0m1, 2, 0, true);   AUT_FORMAT(e1m0, 2, 1, false);
AUT_FORMAT(e0m2, 3, 0, true);   AUT_FORMAT(e1m1, 3, 1, true);
AUT_FORMAT(e2m0, 3, 2, false);
AUT_FORMAT(e0m3, 4, 0, true);   AUT_FORMAT(e1m2, 4, 1, true);
AUT_FORMAT(fp4_e2m1, 4, 2, true); AUT_FORMAT(e3m0, 4, 3, false);
AUT_FORMAT(e0m4, 5, 0, true);   AUT_FORMAT(e1m3, 5, 1, true);
AUT_FORMAT(e2m2, 5, 2, false);  AUT_FORMAT(e3m1, 5, 3, false);
AUT_FORMAT(e4m0, 5, 4, false);
AUT_FORMAT(e0m5, 6, 0, true);   AUT_FORMAT(e1m4, 6, 1, true);
AUT_FORMAT(e2m3, 6, 2, true);   AUT_FORMAT(e3m2, 6, 3, true);
AUT_FORMAT(e4m1, 6, 4, false);  AUT_FORMAT(e5m0, 6, 5, false);
AUT_FORMAT(e0m6, 7, 0, true);   AUT_FORMAT(e2m4, 7, 2, false);
AUT_FORMAT(e3m3, 7, 3, false);  AUT_FORMAT(e5m1, 7, 5, false);
AUT_FORMAT(e6m0, 7, 6, false);
AUT_FORMAT(e0m7, 8, 0, true);   AUT_FORMAT(e1m6, 8, 1, true);
AUT_FORMAT(e2m5, 8, 2, false);  AUT_FORMAT(e3m4, 8, 3, false);
AUT_FORMAT(e6m1, 8, 6, false);  AUT_FORMAT(e7m0, 8, 7, false);
AUT_FORMAT(e0m8, 9, 0, true);   AUT_FORMAT(e2m6, 9, 2, false);
AUT_FORMAT(e4m4, 9, 4, false);  AUT_FORMAT(e5m3, 9, 5, false);
AUT_FORMAT(e8m0, 9, 8, false);
AUT_FORMAT(e2m7, 10, 2, false); AUT_FORMAT(e5m4, 10, 5, false);
AUT_FORMAT(e8m1, 10, 8, false);
AUT_FORMAT(e0m11, 12, 0, true); AUT_FORMAT(e2m9, 12, 2, false);
AUT_FORMAT(e5m6, 12, 5, false); AUT_FORMAT(e8m3, 12, 8, false);
AUT_FORMAT(e2m11, 14, 2, false); AUT_FORMAT(e5m8, 14, 5, false);
AUT_FORMAT(e8m5, 14, 8, false);
AUT_FORMAT(e0m15, 16, 0, true); AUT_FORMAT(e1m14, 16, 1, true);
AUT_FORMAT(e2m13, 16, 2, false); AUT_FORMAT(e3m12, 16, 3, false);
AUT_FORMAT(e4m11, 16, 4, false); AUT_FORMAT(e6m9, 16, 6, false);
AUT_FORMAT(e7m8, 16, 7, false);  AUT_FORMAT(e9m6, 16, 9, false);
AUT_FORMAT(e10m5, 16, 10, false); AUT_FORMAT(bf16_e8m7, 16, 8, false);
AUT_FORMAT(e2m14, 17, 2, false); AUT_FORMAT(e5m11, 17, 5, false);
AUT_FORMAT(e8m8, 17, 8, false);
AUT_FORMAT(e2m17, 20, 2, false); AUT_FORMAT(e5m14, 20, 5, false);
AUT_FORMAT(e8m11, 20, 8, false);
AUT_FORMAT(e0m23, 24, 0, true);  AUT_FORMAT(e2m21, 24, 2, false);
AUT_FORMAT(e5m18, 24, 5, false); AUT_FORMAT(e8m15, 24, 8, false);
AUT_FORMAT(e2m25, 28, 2, false); AUT_FORMAT(e4m23, 28, 4, false);
AUT_FORMAT(e5m22, 28, 5, false); AUT_FORMAT(e8m19, 28, 8, false);
AUT_FORMAT(e0m31, 32, 0, true);  AUT_FORMAT(e1m30, 32, 1, true);
AUT_FORMAT(e2m29, 32, 2, false); AUT_FORMAT(e3m28, 32, 3, false);
AUT_FORMAT(e4m27, 32, 4, false); AUT_FORMAT(e5m26, 32, 5, false);
AUT_FORMAT(e6m25, 32, 6, false); AUT_FORMAT(e7m24, 32, 7, false);
AUT_FORMAT(e9m22, 32, 9, false); AUT_FORMAT(e10m21, 32, 10, false);
AUT_PREFIX_FORMAT(e11m0, 0);   AUT_PREFIX_FORMAT(e11m2, 2);
AUT_PREFIX_FORMAT(e11m4, 4);   AUT_PREFIX_FORMAT(e11m5, 5);
AUT_PREFIX_FORMAT(e11m8, 8);   AUT_PREFIX_FORMAT(e11m12, 12);
AUT_PREFIX_FORMAT(e11m16, 16); AUT_PREFIX_FORMAT(e11m20, 20);

#undef AUT_FORMAT
#undef AUT_PREFIX_FORMAT

template <typename Format, typename = void> struct is_prefix : std::false_type {};
template <typename Format>
struct is_prefix<Format, std::void_t<decltype(Format::is_prefix)>>
    : std::bool_constant<Format::is_prefix> {};

// codec<F>: encode(double) -> storage_type, decode(storage_type) -> double.
template <typename Format> struct codec {
  using storage_type = typename detail::uint_for<Format::total_bits>::type;

  AUT_HD AUT_INLINE static storage_type encode(double value) {
    if constexpr (is_prefix<Format>::value) {
      return static_cast<storage_type>(
          aut::detail::prefix_encode(Format::fraction_bits, value));
    } else if constexpr (Format::exponent_bits == 0) {
      static_assert(Format::finite, "E0 formats are saturating fixed point");
      return static_cast<storage_type>(
          aut::detail::fixed_encode(Format::total_bits, value));
    } else {
      return static_cast<storage_type>(aut::detail::ieee_encode(
          Format::total_bits, Format::exponent_bits, Format::finite, value));
    }
  }

  AUT_HD AUT_INLINE static double decode(storage_type stored) {
    const auto raw = static_cast<std::uint32_t>(stored);
    if constexpr (is_prefix<Format>::value) {
      return aut::detail::prefix_decode(Format::fraction_bits, raw);
    } else if constexpr (Format::exponent_bits == 0) {
      return aut::detail::fixed_decode(Format::total_bits, raw);
    } else {
      return aut::detail::ieee_decode(Format::total_bits,
                                      Format::exponent_bits, Format::finite,
                                      raw);
    }
  }
};

template <typename Format>
using storage_type_t = typename codec<Format>::storage_type;

template <typename Format>
AUT_HD AUT_INLINE storage_type_t<Format> encode(double value) {
  return codec<Format>::encode(value);
}

template <typename Format>
AUT_HD AUT_INLINE double decode(storage_type_t<Format> value) {
  return codec<Format>::decode(value);
}

static_assert(sizeof(storage_type_t<e1m6>) == 1);
static_assert(sizeof(storage_type_t<e11m4>) == 2);
static_assert(sizeof(storage_type_t<e11m20>) == 4);

} // namespace aut::storage

#endif

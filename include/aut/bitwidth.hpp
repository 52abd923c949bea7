// aut/bitwidth.hpp -- the dense LSB-first bitstream layout and the per-code
// decoders of the bit-width study (host + device).
//
// Drop-in for the reference's include/bitwidth_benchmark_core.hpp: the axis
// enums (:22-40), compute_traits (:42-53), format_layout (:55-70), the dense
// and cooperative geometries (:70-121), the dense-storage helpers
// (:123-169) and decode_reference / decode_raw (:236-295).  Value i of a
// B-bit stream occupies bits [B*i, B*i + B) of an array of little-endian
// uint32 words; a field may straddle two words.  A stream of n values owns
// dense_word_count<B>(n) words: the data words plus one zero guard word, so
// every two-word read stays inside the allocation.
#ifndef AUT_BITWIDTH_HPP_
#define AUT_BITWIDTH_HPP_

#include "decoder.hpp"
#include "detail/codec_core.hpp"
#include "storage_formats.hpp"

#include <cstddef>
#include <cstdint>
#include <type_traits>

namespace aut::bitwidth {

enum class compute_kind { fp32, fp64 };
enum class storage_layout { dense, padded };
// How a DOT kernel reads its operands (the reference's access_method; the
// B200 library's strategies are AUT_STRATEGY_* in autdot.h).
enum class access_method { scalar, thread_packet, cooperative_shuffle };
// How a code becomes a value (the reference's decoder_kind).
enum class decoder_kind {
  generic_reference,
  direct_branchy,
  direct_masked,
  fixed_integer,
  e1_integer,
  exponent_only,
  full_lut_global,
  full_lut_shared,
  prefix_lut_global,
  prefix_lut_shared,
  subnormal_lut_global,
  subnormal_lut_shared,
  native_scalar,
  native_packed
};

template <compute_kind Kind> struct compute_traits;
template <> struct compute_traits<compute_kind::fp32> {
  using type = float;
  static constexpr const char *name = "fp32";
};
template <> struct compute_traits<compute_kind::fp64> {
  using type = double;
  static constexpr const char *name = "fp64";
};
template <compute_kind Kind> using compute_t = typename compute_traits<Kind>::type;

// The decoder layout of a storage format.
template <typename Format> struct format_layout {
  static constexpr decoder::special_policy policy =
      aut::storage::is_prefix<Format>::value ? decoder::special_policy::fp64_prefix
      : Format::exponent_bits == 0           ? decoder::special_policy::fixed_e0
      : Format::finite                       ? decoder::special_policy::finite_all
                                             : decoder::special_policy::ieee;
  using type = decoder::binary_layout<Format::total_bits, Format::exponent_bits, policy>;
};
template <typename Format> using format_layout_t = typename format_layout<Format>::type;

template <typename Format>
using padded_storage_t = aut::storage::storage_type_t<Format>;

template <int Bits> struct dense_geometry {
  static_assert(Bits >= 2 && Bits <= 32);
  static constexpr int gcd = [] {
    int a = Bits, b = 32;
    while (b != 0) {
      const int r = a % b;
      a = b;
      b = r;
    }
    return a;
  }();
  static constexpr int values_per_aligned_chunk = 32 / gcd;
  static constexpr int words_per_aligned_chunk = Bits / gcd;
  static constexpr int chunk_bits = values_per_aligned_chunk * Bits;
};

// Cooperative loading (the reference's cooperative_shuffle access): one
// aligned chunk of `values` codes spans `words` 32-bit words; `consumers`
// lanes (a power of two, more than `words`, so one lane always holds the
// zero guard) share the chunk through warp shuffles, each decoding
// values / consumers codes.
template <int Bits> struct cooperative_geometry {
  static_assert(Bits >= 2 && Bits < 32, "a 32-bit code is one word already");
  static constexpr int values = dense_geometry<Bits>::values_per_aligned_chunk;
  static constexpr int words = dense_geometry<Bits>::words_per_aligned_chunk;
  // at least four lanes, a lane per word plus the guard lane, and at most
  // four codes per lane; never more lanes than codes
  static constexpr int consumers = [] {
    int above = 1;
    while (above <= words) above *= 2;
    int c = above > 4 ? above : 4;
    if (values / 4 > c) c = values / 4;
    return c < values ? c : values;
  }();
  static constexpr int values_per_consumer = values / consumers;
  static_assert(values * Bits == words * 32 && values % consumers == 0);
  static_assert(words < consumers && 32 % consumers == 0);
};
template <int Bits> inline constexpr bool cooperative_supported_v = Bits < 32;

template <int Bits> AUT_HD AUT_INLINE constexpr std::uint32_t raw_mask() {
  return aut::detail::low_mask32(Bits);
}

template <int Bits>
AUT_HD AUT_INLINE std::uint32_t load_dense_scalar(const std::uint32_t *words,
                                                  std::size_t index) {
  const std::size_t bit = index * static_cast<std::size_t>(Bits);
  const std::size_t w = bit >> 5;
  const unsigned shift = static_cast<unsigned>(bit & 31u);
  const std::uint64_t pair = static_cast<std::uint64_t>(words[w]) |
                             (static_cast<std::uint64_t>(words[w + 1]) << 32);
  return static_cast<std::uint32_t>(pair >> shift) & raw_mask<Bits>();
}

template <int Bits>
AUT_HD AUT_INLINE void or_dense_scalar(std::uint32_t *words, std::size_t index,
                                       std::uint32_t raw) {
  const std::size_t bit = index * static_cast<std::size_t>(Bits);
  const std::size_t w = bit >> 5;
  const unsigned shift = static_cast<unsigned>(bit & 31u);
  const std::uint64_t placed = static_cast<std::uint64_t>(raw & raw_mask<Bits>())
                               << shift;
  words[w] |= static_cast<std::uint32_t>(placed);
  if (shift + Bits > 32) words[w + 1] |= static_cast<std::uint32_t>(placed >> 32);
}

template <int Bits> constexpr std::size_t dense_word_count(std::size_t values) {
  return (values * static_cast<std::size_t>(Bits) + 31u) / 32u + 1u;
}

template <int Bits> constexpr std::size_t dense_data_bytes(std::size_t values) {
  return (values * static_cast<std::size_t>(Bits) + 7u) / 8u;
}

// ---- per-code decode ------------------------------------------------------
// The host decoder's value in the compute type.
template <typename Format, compute_kind Compute>
AUT_HD AUT_INLINE compute_t<Compute> decode_reference(std::uint32_t raw) {
  using stored = aut::storage::storage_type_t<Format>;
  return static_cast<compute_t<Compute>>(aut::storage::decode<Format>(static_cast<stored>(raw)));
}

// One code decoded by the named strategy; every strategy is exact.  The
// table and native-conversion kinds need device state (a decode table, the
// sm_100 conversion instructions) and are served by the fused DOT kernels
// of libautdot (AUT_DECODER_FULL_LUT / AUT_DECODER_DIRECT).
template <typename Format, compute_kind Compute, decoder_kind Decoder>
AUT_HD AUT_INLINE compute_t<Compute> decode_raw(std::uint32_t raw) {
  using L = format_layout_t<Format>;
  using T = compute_t<Compute>;
  constexpr bool prefix = L::policy == decoder::special_policy::fp64_prefix;
  if constexpr (Decoder == decoder_kind::generic_reference) {
    return decode_reference<Format, Compute>(raw);
  } else if constexpr (Decoder == decoder_kind::direct_branchy ||
                       Decoder == decoder_kind::direct_masked) {
    if constexpr (prefix) {
      return static_cast<T>(
          decoder::words_to_double(decoder::decode_prefix_words<Format::fraction_bits>(raw)));
    } else if constexpr (Compute == compute_kind::fp32 && Format::exponent_bits <= 8 &&
                         Format::fraction_bits <= 23 && Format::total_bits <= 25) {
      return decoder::bits_to_float(decoder::decode_fp32_bits<L>(raw));
    } else if constexpr (Decoder == decoder_kind::direct_branchy) {
      return static_cast<T>(decoder::words_to_double(decoder::decode_words_branchy<L>(raw)));
    } else {
      return static_cast<T>(decoder::words_to_double(decoder::decode_words_masked<L>(raw)));
    }
  } else if constexpr (Decoder == decoder_kind::fixed_integer) {
    return static_cast<T>(decoder::decode_fixed_integer<L>(raw));
  } else if constexpr (Decoder == decoder_kind::e1_integer) {
    return static_cast<T>(decoder::decode_e1_integer<L>(raw));
  } else if constexpr (Decoder == decoder_kind::exponent_only) {
    return static_cast<T>(decoder::decode_exponent_only<L>(raw));
  } else {
    static_assert(Decoder == decoder_kind::generic_reference,
                  "table and native decoders run inside the fused DOT kernels");
    return T{};
  }
}

static_assert(dense_geometry<6>::values_per_aligned_chunk == 16);
static_assert(dense_geometry<6>::words_per_aligned_chunk == 3);
static_assert(dense_geometry<24>::values_per_aligned_chunk == 4);
static_assert(dense_geometry<24>::words_per_aligned_chunk == 3);

} // namespace aut::bitwidth

#endif

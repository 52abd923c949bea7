// aut/bitwidth.hpp -- the dense LSB-first bitstream layout (host + device).
//
// Drop-in for the dense-storage helpers of the reference's
// include/bitwidth_benchmark_core.hpp:70-85 and :123-169.  Value i of a
// B-bit stream occupies bits [B*i, B*i + B) of an array of little-endian
// uint32 words; a field may straddle two words.  A stream of n values owns
// dense_word_count<B>(n) words: the data words plus one zero guard word, so
// every two-word read stays inside the allocation.
#ifndef AUT_BITWIDTH_HPP_
#define AUT_BITWIDTH_HPP_

#include "detail/codec_core.hpp"

#include <cstddef>
#include <cstdint>

namespace aut::bitwidth {

enum class compute_kind { fp32, fp64 };
enum class storage_layout { dense, padded };

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

static_assert(dense_geometry<6>::values_per_aligned_chunk == 16);
static_assert(dense_geometry<6>::words_per_aligned_chunk == 3);
static_assert(dense_geometry<24>::values_per_aligned_chunk == 4);
static_assert(dense_geometry<24>::words_per_aligned_chunk == 3);

} // namespace aut::bitwidth

#endif

// codec_core.hpp -- runtime-parameterised storage codecs (host + device).
//
// One implementation serves three callers: the aut::storage / aut::lns
// templates (compile-time parameters fold into constants), the C ABI's host
// codec entry points (runtime format descriptors) and the device encode /
// decode kernels.  The bit-level rules are fixed by the reference's stored
// data, so they follow it exactly:
//   E = 0 fixed point      storage_formats.hpp:266-342
//   E >= 1 IEEE-like       storage_formats.hpp:344-467
//   FP64 prefix            storage_formats.hpp:561-592
//   LNS special codes      lns_benchmark_core.hpp:93-168
#ifndef AUT_DETAIL_CODEC_CORE_HPP_
#define AUT_DETAIL_CODEC_CORE_HPP_

#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define AUT_HD __host__ __device__
#define AUT_INLINE __forceinline__
#else
#define AUT_HD
#define AUT_INLINE inline
#endif

namespace aut::detail {

AUT_HD AUT_INLINE std::uint64_t bits_of(double v) {
#if defined(__CUDA_ARCH__)
  return static_cast<std::uint64_t>(__double_as_longlong(v));
#else
  std::uint64_t b;
  std::memcpy(&b, &v, sizeof b);
  return b;
#endif
}

AUT_HD AUT_INLINE double double_of(std::uint64_t b) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double(static_cast<long long>(b));
#else
  double v;
  std::memcpy(&v, &b, sizeof v);
  return v;
#endif
}

AUT_HD AUT_INLINE int top_bit(std::uint64_t v) {
#if defined(__CUDA_ARCH__)
  return 63 - __clzll(static_cast<long long>(v));
#else
  return 63 - __builtin_clzll(v);
#endif
}

AUT_HD AUT_INLINE constexpr std::uint32_t low_mask32(int bits) {
  return bits >= 32 ? 0xffffffffu : ((std::uint32_t{1} << bits) - 1u);
}

// Round-to-nearest-even right shift of an integer significand.
AUT_HD AUT_INLINE std::uint64_t shift_right_rne(std::uint64_t v, unsigned s) {
  if (s == 0) return v;
  if (s >= 64) return 0;
  const std::uint64_t q = v >> s;
  const std::uint64_t r = v & ((std::uint64_t{1} << s) - 1);
  const std::uint64_t h = std::uint64_t{1} << (s - 1);
  return q + static_cast<std::uint64_t>(r > h || (r == h && (q & 1u)));
}

// ---- E = 0: sign + (T-1)-bit fraction, saturating --------------------------
AUT_HD AUT_INLINE std::uint32_t fixed_encode(int T, double value) {
  const int F = T - 1;
  const std::uint64_t magmask = (std::uint64_t{1} << F) - 1;
  const std::uint64_t b = bits_of(value);
  const std::uint64_t sfield = (b >> 63) << (T - 1);
  const std::uint64_t e = (b >> 52) & 0x7ffu;
  const std::uint64_t f = b & ((std::uint64_t{1} << 52) - 1);
  if (e == 0x7ffu) return static_cast<std::uint32_t>(sfield | magmask);
  if (e == 0 && f == 0) return static_cast<std::uint32_t>(sfield);
  const std::uint64_t sig = e == 0 ? f : ((std::uint64_t{1} << 52) | f);
  const int unb = e == 0 ? -1022 : static_cast<int>(e) - 1023;
  const int shift = 52 - F - unb;
  std::uint64_t mag;
  if (shift > 0) {
    mag = shift_right_rne(sig, static_cast<unsigned>(shift));
  } else {
    const unsigned ls = static_cast<unsigned>(-shift);
    mag = (ls >= 64 || sig > (magmask >> ls)) ? magmask : (sig << ls);
  }
  if (mag > magmask) mag = magmask;
  return static_cast<std::uint32_t>(sfield | mag);
}

AUT_HD AUT_INLINE double fixed_decode(int T, std::uint32_t stored) {
  const int F = T - 1;
  const std::uint64_t raw = stored & low_mask32(T);
  const std::uint64_t s64 = (raw >> (T - 1)) << 63;
  const std::uint64_t mag = raw & ((std::uint64_t{1} << F) - 1);
  if (mag == 0) return double_of(s64);
  const int lead = top_bit(mag);
  return double_of(s64 | (static_cast<std::uint64_t>(lead - F + 1023) << 52) |
                   ((mag - (std::uint64_t{1} << lead)) << (52 - lead)));
}

// ---- E >= 1: IEEE-like, gradual underflow, finite or inf/NaN ---------------
AUT_HD AUT_INLINE std::uint32_t ieee_encode(int T, int E, bool finite,
                                            double value) {
  const int M = T - E - 1;
  const std::uint64_t fmask = (std::uint64_t{1} << M) - 1;
  const std::uint64_t emask = (std::uint64_t{1} << E) - 1;
  const int bias = (1 << (E - 1)) - 1;
  const std::uint64_t top_exp = finite ? emask : emask - 1;
  const std::uint64_t b = bits_of(value);
  const std::uint64_t sfield = (b >> 63) << (T - 1);
  const std::uint64_t se = (b >> 52) & 0x7ffu;
  const std::uint64_t sf = b & ((std::uint64_t{1} << 52) - 1);
  const std::uint64_t saturated = sfield | (top_exp << M) | fmask;
  const std::uint64_t infinity = sfield | (emask << M);
  if (se == 0x7ffu) {
    if (finite) return static_cast<std::uint32_t>(saturated);
    if (sf == 0) return static_cast<std::uint32_t>(infinity);
    std::uint64_t payload = sf >> (52 - M);
    if (payload == 0) payload = 1;
    return static_cast<std::uint32_t>(infinity | (payload & fmask));
  }
  if (se == 0) return static_cast<std::uint32_t>(sfield);
  const int unb = static_cast<int>(se) - 1023;
  int te = unb + bias;
  if (te <= 0) {
    const std::uint64_t sig = (std::uint64_t{1} << 52) | sf;
    const std::uint64_t sub = shift_right_rne(
        sig, static_cast<unsigned>(53 - unb - bias - M));
    if (sub == 0) return static_cast<std::uint32_t>(sfield);
    if (sub >= (std::uint64_t{1} << M))
      return static_cast<std::uint32_t>(sfield | (std::uint64_t{1} << M));
    return static_cast<std::uint32_t>(sfield | sub);
  }
  std::uint64_t tf = shift_right_rne(sf, static_cast<unsigned>(52 - M));
  if (tf == (std::uint64_t{1} << M)) {
    tf = 0;
    ++te;
  }
  if (te > static_cast<int>(top_exp))
    return static_cast<std::uint32_t>(finite ? saturated : infinity);
  return static_cast<std::uint32_t>(
      sfield | (static_cast<std::uint64_t>(te) << M) | tf);
}

AUT_HD AUT_INLINE double ieee_decode(int T, int E, bool finite,
                                     std::uint32_t stored) {
  const int M = T - E - 1;
  const std::uint64_t raw = stored & low_mask32(T);
  const std::uint64_t emask = (std::uint64_t{1} << E) - 1;
  const int bias = (1 << (E - 1)) - 1;
  const std::uint64_t s64 = (raw >> (T - 1)) << 63;
  const std::uint64_t e = (raw >> M) & emask;
  const std::uint64_t f = raw & ((std::uint64_t{1} << M) - 1);
  if (e == 0) {
    if (f == 0) return double_of(s64);
    const int lead = top_bit(f);
    return double_of(
        s64 | (static_cast<std::uint64_t>(lead + 1 - bias - M + 1023) << 52) |
        ((f - (std::uint64_t{1} << lead)) << (52 - lead)));
  }
  if (!finite && e == emask)
    return double_of(s64 | (std::uint64_t{0x7ff} << 52) | (f << (52 - M)));
  return double_of(s64 |
                   (static_cast<std::uint64_t>(static_cast<int>(e) - bias + 1023)
                    << 52) |
                   (f << (52 - M)));
}

// ---- FP64 prefix: the top 12 + F bits of a binary64, RNE -------------------
AUT_HD AUT_INLINE std::uint32_t prefix_encode(int F, double value) {
  const int dropped = 52 - F;
  const std::uint64_t b = bits_of(value);
  const std::uint64_t e = (b >> 52) & 0x7ffu;
  const std::uint64_t f = b & ((std::uint64_t{1} << 52) - 1);
  std::uint64_t kept = b >> dropped;
  if (e == 0x7ffu) {
    if (f != 0 && (kept & ((std::uint64_t{1} << F) - 1)) == 0) kept |= 1;
    return static_cast<std::uint32_t>(kept) & low_mask32(12 + F);
  }
  const std::uint64_t lost = b & ((std::uint64_t{1} << dropped) - 1);
  const std::uint64_t half = std::uint64_t{1} << (dropped - 1);
  if (lost > half || (lost == half && (kept & 1u))) ++kept;
  return static_cast<std::uint32_t>(kept) & low_mask32(12 + F);
}

AUT_HD AUT_INLINE double prefix_decode(int F, std::uint32_t stored) {
  return double_of(static_cast<std::uint64_t>(stored & low_mask32(12 + F))
                   << (52 - F));
}

// ---- LNS code fields (Universal-style sign + two's-complement log2) --------
AUT_HD AUT_INLINE constexpr std::uint32_t lns_log_mask(int B) {
  return (std::uint32_t{1} << (B - 1)) - 1u;
}
AUT_HD AUT_INLINE constexpr std::uint32_t lns_sign_mask(int B) {
  return std::uint32_t{1} << (B - 1);
}
AUT_HD AUT_INLINE constexpr std::uint32_t lns_special(int B) {
  return std::uint32_t{1} << (B - 2);
}
AUT_HD AUT_INLINE std::int32_t lns_log_code(int B, std::uint32_t raw) {
  std::uint32_t c = raw & lns_log_mask(B);
  if (c & (std::uint32_t{1} << (B - 2))) c |= ~lns_log_mask(B);
  return static_cast<std::int32_t>(c);
}

} // namespace aut::detail

#endif

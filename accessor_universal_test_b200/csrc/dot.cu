// dot.cu -- the decode-fused DOT kernels and aut_dot / aut_dot_batched.
//
// One persistent kernel per (format, layout, accumulator, access strategy)
// does the whole DOT: stream both code vectors, decode in registers, FMA into
// per-thread accumulators, warp-shuffle + shared-memory block sum and a
// single-pass grid reduction into the device result.  This replaces the
// reference's dot_thread_kernel + finalize_dot_kernel pair
// (bitwidth_benchmark_kernels.cuh:403-457), the LNS dot_thread_kernel
// (lns_benchmark_kernels.cuh:80-131), raw_dot_kernel (:681-703) and the
// accessor map-reduce (src/accessor_dot_bench.cu:417-454).
//
// Access strategies (the reference's access_method axis,
// bitwidth_benchmark_core.hpp:24):
//   LDG -- each thread loads whole 16-byte packets into registers;
//   TMA -- one thread per block streams contiguous tiles of both vectors into
//          a shared-memory ring with plain cp.async.bulk copies (each block
//          reads only this GPU's memory into its own shared memory) and an
//          mbarrier per stage; threads decode their units from shared memory.
#include "dot_device.cuh"
#include "internal.hpp"

#include "aut/bitwidth.hpp"

#include <cuda_fp16.h>

#include <cstdio>
#include <cstring>
#include <type_traits>

namespace aut::dev {

// Decode parameters of a format without a dedicated codec (rt_codec below).
struct rt_params {
  uint32_t bits;          // B: code width (padded containers: the code's own width)
  uint32_t exponent;      // E (0: fixed point)
  uint32_t special_from;  // top-aligned magnitudes >= this are inf/NaN to build (0: none)
  uint32_t pad;
  float scale32;          // 2^(127 - bias) (fixed point: 2^126)
  uint32_t pad2;
  double scale64;         // 2^(1023 - bias) (fixed point: 2^1022)
};

struct dot_params {
  const unsigned char *x;
  const unsigned char *y;
  uint64_t n;
  uint64_t x_stride;      // bytes between the pairs of a batch
  uint64_t y_stride;
  uint64_t x_first;       // value index of this launch's first x / y (per-value path)
  uint64_t y_first;
  uint64_t x_index_stride;  // values between pairs whose streams do not start
  uint64_t y_index_stride;  // on a byte (per-value path only)
  int vector_ok;          // both streams 16-byte aligned
  const void *table;      // decode table (LNS formats)
  double *partials;       // [gridDim.y][gridDim.x]
  unsigned int *tickets;  // [gridDim.y]
  double *results;        // [gridDim.y]
  unsigned int *status;   // sticky error bits (AUT_STATUS_*)
  rt_params rt;           // rt_codec only
  long long wait_cycles;  // bound of every bulk-copy wait (SM clock cycles)
  uint64_t stall_tile;    // failure-detection test: this tile's stage is
                          // armed but its copies are never issued, so the
                          // wait for it runs out (~0: none)
  unsigned int *claims;   // [gridDim.y] tile counters of the bulk-copy kernel's
                          // dynamic tail (order-free codecs), zero between
                          // launches; nullptr: every tile assigned statically
};

// ---------------------------------------------------------------------------
// Codecs.  Each supplies kS (bits per stored slot), kU (LDG packets per thread
// per tile), kTableBytes (dynamic shared memory), kExactLanes (uses the four
// float lanes for exact partial sums), prepare(), values<NV>() decoding NV
// consecutive codes from a word array and scalar() for ragged tails.
// ---------------------------------------------------------------------------

// IEEE-like formats with an 8-bit exponent (e8m0 ... e8m15, bf16, and raw
// FP32 as W = 32): the FP32 bit pattern is the code shifted to the top of
// the word (decoder_strategy_core.hpp:319-322), exact for normals,
// subnormals, infinities and NaNs.
template <int S, int W> struct e8_codec {
  static constexpr int kS = S;
  static constexpr int kU = packet_shape<S>::Q == 1 ? 4 : (S == 24 ? 2 : 1);
  static constexpr int kTableBytes = 0;
  static constexpr bool kExactLanes = false;
  __device__ static void prepare(const dot_params &, unsigned char *) {}

  // With at most 11 mantissa bits the FP32 product of two decoded values is
  // exact unless it underflows or overflows, so the FP64 accumulator widens
  // the product (one conversion per pair) instead of both operands (two
  // conversions, which bound the kernel on the conversion pipe).  A call
  // whose smallest |product| is below 2^-126 (zeros included) or whose sum is
  // not finite is redone with both operands widened: the result is the same
  // FP64 sum of exact products either way.
  static constexpr bool kProductWidening = W - 9 <= 11;
  static constexpr int kW = W;

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *, const unsigned char *) {
    if constexpr (kProductWidening && std::is_same_v<Acc, acc_f64>) {
      constexpr int C = NV < 16 ? NV : 16;  // values per check
      static_assert(NV % C == 0, "whole chunks");
#pragma unroll
      for (int c0 = 0; c0 < NV; c0 += C) {
        double s0 = 0.0, s1 = 0.0;
        float smallest = __int_as_float(0x7f800000);
#pragma unroll
        for (int v = c0; v < c0 + C; ++v) {
          const float p = __uint_as_float(field_top<S, W>(xw, v)) *
                          __uint_as_float(field_top<S, W>(yw, v));
          smallest = fminf(smallest, fabsf(p));
          if (v & 2)  // adjacent values share a chain (see acc_f32)
            s1 += static_cast<double>(p);
          else
            s0 += static_cast<double>(p);
        }
        const double s = s0 + s1;
        if (smallest >= 1.17549435e-38f && fabs(s) <= 1.7976931348623157e308) {
          acc.add_exact(s);
        } else {
#pragma unroll
          for (int v = c0; v < c0 + C; ++v)
            acc.mac(v, __uint_as_float(field_top<S, W>(xw, v)),
                    __uint_as_float(field_top<S, W>(yw, v)));
        }
      }
    } else {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const float a = __uint_as_float(field_top<S, W>(xw, v));
        const float b = __uint_as_float(field_top<S, W>(yw, v));
        acc.mac(v, a, b);
      }
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *) {
    const float a = __uint_as_float(load_code<S, W>(xb, i) << (32 - W));
    const float b = __uint_as_float(load_code<S, W>(yb, j) << (32 - W));
    acc.mac_d(0, static_cast<double>(a), static_cast<double>(b));
  }
};

// Raw binary64 storage.
struct f64_codec {
  static constexpr int kS = 64;
  static constexpr int kU = 4;
  static constexpr int kTableBytes = 0;
  static constexpr bool kExactLanes = false;
  __device__ static void prepare(const dot_params &, unsigned char *) {}

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *, const unsigned char *) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const double a = __hiloint2double(static_cast<int>(xw[2 * v + 1]),
                                        static_cast<int>(xw[2 * v]));
      const double b = __hiloint2double(static_cast<int>(yw[2 * v + 1]),
                                        static_cast<int>(yw[2 * v]));
      acc.mac_d(v, a, b);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *) {
    acc.mac_d(0, __ldg(reinterpret_cast<const double *>(xb) + i),
              __ldg(reinterpret_cast<const double *>(yb) + j));
  }
};

// FP6 E2M3 (finite).  Four 6-bit codes are spread into the low 6 bits of four
// bytes, the hardware converts byte pairs to f16x2 exactly, and the
// mixed-precision FMA multiplies two f16 values exactly into an FP32 lane.
// Every e2m3 value is k/8 with |k| <= 60, so products are multiples of 2^-6
// below 57 and an FP32 sum of up to 4096 of them is exact: the lanes are
// carried into FP64 once per tile, which makes the DOT exact up to its final
// rounding for both accumulator kinds.
template <int S> struct e2m3_codec {
  static_assert(S == 6 || S == 8, "dense 6-bit or one code per byte");
  static constexpr int kS = S;
  static constexpr int kW = 6;
  static constexpr int kU = S == 8 ? 4 : 2;
  // dense: the shift multipliers in shared memory (see bytes4)
  static constexpr int kTableBytes = S == 6 ? 16 : 0;
  static constexpr bool kExactLanes = true;
  __device__ static void prepare(const dot_params &, unsigned char *smem) {
    if constexpr (S == 6) {
      if (threadIdx.x == 0) {
        uint32_t *m = reinterpret_cast<uint32_t *>(smem);
        m[0] = 1u << 24;
        m[1] = 1u << 4;
        m[2] = 1u << 2;
        m[3] = 0u;
      }
    }
  }

  // Codes 4g .. 4g+3 of the word array, one per byte (low 6 bits).  The
  // conversion reads the low 6 bits of each byte and ignores bits 6-7 (the
  // fp6 storage byte of cuda_fp6.h), so the bytes may carry neighbouring
  // bits there and no mask is needed: with q holding the four codes at bits
  // 0, 6, 12, 18 (anything above bit 24), one byte permute takes bytes 0-1
  // of q and bytes 2-3 of q << 4 (codes 2, 3 at bits 16, 22), a second takes
  // bytes 0, 2 of that and bytes 1, 3 of it << 2 (codes 1, 3 at bits 8, 24).
  // The shifts are integer multiplies by factors read from shared memory,
  // so they run on the FMA pipe beside the permutes on the ALU pipe (dense
  // e2m3, N = 2^27: 5677 -> 5746 GB/s against two mask-and-multiply steps);
  // a group at bit 8 of a word is moved by the high word of w * 2^24.
  __device__ __forceinline__ static uint32_t bytes4(const uint32_t *w, int g,
                                                    const unsigned char *smem) {
    if constexpr (S == 8) {
      return w[g];  // one code per byte; bits 6-7 are zero, and ignored
    } else {
      const uint32_t *m = reinterpret_cast<const uint32_t *>(smem);
      const int b = 24 * g, i = b >> 5, sh = b & 31;
      uint32_t q;  // v3 v2 v1 v0, 6 bits each, anything above bit 24
      if (sh == 0)
        q = w[i];
      else if (sh == 8)
        q = __umulhi(w[i], m[0]);
      else
        q = field_low<24, 24>(w, g);
      const uint32_t p = __byte_perm(q, q * m[1], 0x7610);  // v3v2 -> [16,28)
      return __byte_perm(p, p * m[2], 0x7250);               // v1, v3 up by two
    }
  }

  __device__ __forceinline__ static uint32_t to_f16x2(uint32_t two_bytes) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e2m3x2 %0, %1;"
        : "=r"(h2)
        : "h"(static_cast<unsigned short>(two_bytes)));
    return h2;
  }

  // both byte pairs of a word: the halves are register halves, no shift
  __device__ __forceinline__ static void to_f16x2x2(uint32_t four, uint32_t &lo,
                                                    uint32_t &hi) {
    asm("{\n\t.reg .b16 l, h;\n\t"
        "mov.b32 {l, h}, %2;\n\t"
        "cvt.rn.f16x2.e2m3x2 %0, l;\n\t"
        "cvt.rn.f16x2.e2m3x2 %1, h;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(four));
  }

  __device__ __forceinline__ static void fma2(float &lo, float &hi, uint32_t x2,
                                              uint32_t y2) {
    asm("{\n\t.reg .f16 xl, xh, yl, yh;\n\t"
        "mov.b32 {xl, xh}, %2;\n\t"
        "mov.b32 {yl, yh}, %3;\n\t"
        "fma.rn.f32.f16 %0, xl, yl, %0;\n\t"
        "fma.rn.f32.f16 %1, xh, yh, %1;\n\t}"
        : "+f"(lo), "+f"(hi)
        : "r"(x2), "r"(y2));
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &,
                                                float *lanes,
                                                const unsigned char *smem) {
    static_assert(NV % 4 == 0, "e2m3 decodes groups of four codes");
#pragma unroll
    for (int g = 0; g < NV / 4; ++g) {
      uint32_t xl, xh, yl, yh;
      to_f16x2x2(bytes4(xw, g, smem), xl, xh);
      to_f16x2x2(bytes4(yw, g, smem), yl, yh);
      fma2(lanes[0], lanes[1], xl, yl);
      fma2(lanes[2], lanes[3], xh, yh);
    }
  }

  __device__ __forceinline__ static float decode1(uint32_t c) {
    const uint32_t h2 = to_f16x2(c & 0x3fu);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h2)));
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *) {
    acc.mac_d(0, static_cast<double>(decode1(load_code<S, 6>(xb, i))),
              static_cast<double>(decode1(load_code<S, 6>(yb, j))));
  }
};

// Copies of a small decode table in shared memory, one per lane (C = 32),
// so a warp's lookups never share a bank: entry e of copy c at element
// e * kCopies + c.  (8-byte entries are conflict-free with 16 copies, a
// half warp per wavefront; for the full lns8_r3 table the extra blocks that
// the halved table lets onto an SM then saturate the shared-memory pipe --
// FP64, 3650 -> 3355 GB/s -- so it keeps 32, while the fused-sum table,
// one lookup per pair, takes 16.)
template <typename T, int C = 32> struct lane_table {
  static constexpr int kCopies = C;
  static constexpr uint32_t kEntryBytes = kCopies * static_cast<uint32_t>(sizeof(T));
  static constexpr int bytes(int entries) { return entries * static_cast<int>(kEntryBytes); }
  __device__ __forceinline__ static uint32_t lane_offset() {
    return (threadIdx.x & (kCopies - 1)) * static_cast<uint32_t>(sizeof(T));
  }
  __device__ static void fill(T *s, const T *g, int entries) {
    for (int e = threadIdx.x; e < entries * kCopies; e += blockDim.x) s[e] = g[e / kCopies];
  }
  // entry `code` of this lane's copy
  __device__ __forceinline__ static T at(const unsigned char *smem, uint32_t code,
                                         uint32_t lane_off) {
    return *reinterpret_cast<const T *>(smem + (code * kEntryBytes + lane_off));
  }
};

// lns8_r3 (one code per byte): a full 256-entry decode table in per-lane
// copies (lane_table; C copies, 32 for the DOTs, 16 for the FP64 GEMV rows).
// Table values come from the host exp2f / exp2 and are the reference's
// decoded values bit for bit.
template <typename T, int C = 32> struct lns8_codec {
  using table = lane_table<T, C>;
  static constexpr int kS = 8;
  static constexpr int kW = 8;
  static constexpr int kU = 4;
  static constexpr int kTableBytes = table::bytes(256);
  static constexpr bool kExactLanes = false;
  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    table::fill(reinterpret_cast<T *>(smem), static_cast<const T *>(p.table), 256);
  }

  // Byte k of a word is moved to bits [0, 8) by one byte permute (ALU pipe)
  // and scaled into a table offset by one integer multiply-add (FMA pipe),
  // so the two decode steps of every code use different pipes.
  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *,
                                                const unsigned char *smem) {
    const uint32_t lane_off = table::lane_offset();
#pragma unroll
    for (int w = 0; w < NV / 4; ++w) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t bx = __byte_perm(xw[w], 0u, 0x4440u + k);
        const uint32_t by = __byte_perm(yw[w], 0u, 0x4440u + k);
        const T a = table::at(smem, bx, lane_off);
        const T b = table::at(smem, by, lane_off);
        if constexpr (sizeof(T) == 4)
          acc.mac(4 * w + k, a, b);
        else
          acc.mac_d(4 * w + k, a, b);
      }
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *smem) {
    const uint32_t lane_off = table::lane_offset();
    acc.mac_d(0, static_cast<double>(table::at(smem, load_code<8, 8>(xb, i), lane_off)),
              static_cast<double>(table::at(smem, load_code<8, 8>(yb, j), lane_off)));
  }
};

// lns8_r3 with the fused-sum decoder (fused_sum_lut_shared,
// lns_decoder_strategies.cuh:327-347): the two log codes are added and one
// lookup in a table of every signed product serves the pair.  Each 7-bit
// log code is biased by 2^6 (reserved code -> 0, finite codes -> [1, 127]),
// so one 32-bit add sums the four byte lanes of a word pair without a carry
// crossing them: byte k of the sum is the biased product log h of pair k.
// The table holds 512 signed products, entry s * 256 + h = (-1)^s *
// T(exp2((h - 128) / 8)) (the reference's product table shifted by two
// slots, and its negation), with entries 0 and 256 = +0; one byte permute
// per pair builds the index from byte k of the sums and byte k of the
// product signs (moved to bit 0 of each byte once per word).  The table is
// replicated per lane (entry i of lane l at i * kCopies + l % kCopies), so
// the lookups of a warp never share a bank.  Reserved codes follow
// lns::multiply_codes (lns_benchmark_core.hpp:241-254) without branches:
// adding 0x7f to a biased byte sets its top bit exactly when the code is not
// reserved, a sign-replicating byte permute spreads that bit over its byte,
// and the sums are masked with it once per word, so a pair with a zero
// operand reads entry 0 or 256; a reserved code with its sign bit set (NaN)
// raises a flag that makes the DOT NaN.
template <typename T> struct lns8_fused_codec {
  // FP64: 16 copies (a half warp per 8-byte wavefront is still conflict-free)
  using table = lane_table<T, sizeof(T) == 8 ? 16 : 32>;
  static constexpr int kS = 8;
  static constexpr int kU = 4;
  static constexpr int kEntry = static_cast<int>(sizeof(T));
  static constexpr int kTableBytes = table::bytes(512);
  static constexpr bool kExactLanes = false;

  // signed entry i of the product table `g` (256 magnitudes)
  __device__ __forceinline__ static T signed_entry(const T *g, int i) {
    const int h = i & 255;
    if (h == 0) return T(0);
    return i >= 256 ? -g[h] : g[h];
  }

  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    const T *g = static_cast<const T *>(p.table);
    T *s = reinterpret_cast<T *>(smem);
    for (int e = threadIdx.x; e < 512 * table::kCopies; e += blockDim.x)
      s[e] = signed_entry(g, e / table::kCopies);
  }

  template <int K> __device__ __forceinline__ static uint32_t permute(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "n"(K));
    return r;
  }

  // table index of pair k: byte k of `sums` | byte k of `signs` << 8 (the
  // upper bytes replicate bit 7 of a sign byte, which is 0)
  template <int K> __device__ __forceinline__ static uint32_t index(uint32_t sums, uint32_t signs) {
    constexpr int c = 8 | (4 + K);
    return permute<(c << 12) | (c << 8) | ((4 + K) << 4) | K>(sums, signs);
  }

  template <class Acc>
  __device__ __forceinline__ static void add(Acc &acc, int slot, const unsigned char *smem,
                                             uint32_t index, uint32_t lane_off) {
    const T p = table::at(smem, index, lane_off);
    if constexpr (sizeof(T) == 4)
      acc.mac(slot, p, 1.0f);
    else
      acc.mac_d(slot, p, 1.0);
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *,
                                                const unsigned char *smem) {
    static_assert(NV % 4 == 0, "four codes per word");
    const uint32_t lane_off = table::lane_offset();
    uint32_t nan = 0;
#pragma unroll
    for (int w = 0; w < NV / 4; ++w) {
      const uint32_t x = xw[w], y = yw[w];
      const uint32_t bx = (x & 0x7f7f7f7fu) ^ 0x40404040u;
      const uint32_t by = (y & 0x7f7f7f7fu) ^ 0x40404040u;
      // bit 7 of each byte: that code is not reserved
      const uint32_t lx = bx + 0x7f7f7f7fu, ly = by + 0x7f7f7f7fu;
      nan |= (x & ~lx) | (y & ~ly);  // reserved with the sign bit set
      // byte k: biased product log of pair k, 0 when an operand is zero
      const uint32_t h = (bx + by) & permute<0xba98>(lx & ly, 0u);
      const uint32_t sg = ((x ^ y) & 0x80808080u) >> 7;  // byte k: sign of pair k
      add(acc, 4 * w + 0, smem, index<0>(h, sg), lane_off);
      add(acc, 4 * w + 1, smem, index<1>(h, sg), lane_off);
      add(acc, 4 * w + 2, smem, index<2>(h, sg), lane_off);
      add(acc, 4 * w + 3, smem, index<3>(h, sg), lane_off);
    }
    if (nan & 0x80808080u) {
      if constexpr (sizeof(T) == 4)
        acc.mac(0, __uint_as_float(0x7fc00000u), 1.0f);
      else
        acc.mac_d(0, __hiloint2double(0x7ff80000, 0), 1.0);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *smem) {
    const uint32_t cx = load_code<8, 8>(xb, i), cy = load_code<8, 8>(yb, j);
    const uint32_t bx = (cx & 0x7fu) ^ 0x40u, by = (cy & 0x7fu) ^ 0x40u;
    double v;
    if ((bx == 0 && (cx & 0x80u)) || (by == 0 && (cy & 0x80u))) {
      v = __hiloint2double(0x7ff80000, 0);
    } else {
      const uint32_t h = (bx == 0 || by == 0) ? 0u : bx + by;
      v = static_cast<double>(
          table::at(smem, h | (((cx ^ cy) & 0x80u) << 1), table::lane_offset()));
    }
    acc.mac_d(0, v, 1.0);
  }
};

// lns16_r11: value = +-2^q * T[f] with log code c = 2048 q + f, T[f] =
// exp2f(f / 2048) (or exp2 for FP64) from a 2048-entry shared table; the
// power of two is an exponent-field add, exact because T[f] is in [1, 2) and
// |q| <= 8.  The reserved code (+: zero, -: NaN) is selected explicitly.
template <typename T> struct lns16_codec {
  static constexpr int kS = 16;
  static constexpr int kU = 4;
  static constexpr int kTableBytes = 2048 * static_cast<int>(sizeof(T));
  static constexpr bool kExactLanes = false;
  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    const void *table = p.table;
    const T *g = static_cast<const T *>(table);
    T *s = reinterpret_cast<T *>(smem);
    for (int e = threadIdx.x; e < 2048; e += blockDim.x) s[e] = g[e];
  }

  __device__ __forceinline__ static T decode(uint32_t c, const T *tab) {
    const int q = static_cast<int>(c << 17) >> 28;
    const uint32_t sign = c & 0x8000u;
    const bool special = (c & 0x7fffu) == 0x4000u;
    if constexpr (sizeof(T) == 4) {
      const uint32_t bits =
          (__float_as_uint(tab[c & 0x7ffu]) + (static_cast<uint32_t>(q) << 23)) |
          (sign << 16);
      const uint32_t out = special ? (sign ? 0x7fc00000u : 0u) : bits;
      return __uint_as_float(out);
    } else {
      const double t = tab[c & 0x7ffu];
      const uint32_t hi =
          (static_cast<uint32_t>(__double2hiint(t)) + (static_cast<uint32_t>(q) << 20)) |
          (sign << 16);
      const uint32_t lo = static_cast<uint32_t>(__double2loint(t));
      const uint32_t ho = special ? (sign ? 0x7ff80000u : 0u) : hi;
      const uint32_t lo2 = special ? 0u : lo;
      return __hiloint2double(static_cast<int>(ho), static_cast<int>(lo2));
    }
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *,
                                                const unsigned char *smem) {
    const T *tab = reinterpret_cast<const T *>(smem);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const T a = decode(field_low<16, 16>(xw, v), tab);
      const T b = decode(field_low<16, 16>(yw, v), tab);
      if constexpr (sizeof(T) == 4)
        acc.mac(v, a, b);
      else
        acc.mac_d(v, a, b);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *smem) {
    const T *tab = reinterpret_cast<const T *>(smem);
    acc.mac_d(0, static_cast<double>(decode(load_code<16, 16>(xb, i), tab)),
              static_cast<double>(decode(load_code<16, 16>(yb, j), tab)));
  }
};

// lns16_r11, FP32, one lookup per code: the 32768 sign-free codes decode
// through a 128 KiB shared table (entry i = host exp2f of code i, entry
// 0x4000 = +0 for the reserved code); the product's sign is applied once per
// pair (sign bits of both words XORed), and the negative reserved code (NaN)
// is made NaN explicitly, since it reads the zero entry.
struct lns16_full_codec {
  static constexpr int kS = 16;
  static constexpr int kU = 4;
  static constexpr int kTableBytes = 32768 * 4;
  static constexpr bool kExactLanes = false;
  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    const void *table = p.table;
    const uint4 *g = static_cast<const uint4 *>(table);
    uint4 *s = reinterpret_cast<uint4 *>(smem);
    for (int e = threadIdx.x; e < 32768 / 4; e += blockDim.x) s[e] = g[e];
  }

  __device__ __forceinline__ static float at(const unsigned char *smem, uint32_t off) {
    return *reinterpret_cast<const float *>(smem + off);
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *,
                                                const unsigned char *smem) {
    static_assert(NV % 2 == 0, "two codes per word");
#pragma unroll
    for (int w = 0; w < NV / 2; ++w) {
      const uint32_t x = xw[w], y = yw[w];
      float xl = at(smem, (x << 2) & 0x1fffcu);
      float xh = at(smem, (x >> 14) & 0x1fffcu);
      const float yl = at(smem, (y << 2) & 0x1fffcu);
      const float yh = at(smem, (y >> 14) & 0x1fffcu);
      const uint32_t sgn = x ^ y;  // product signs at bits 15 and 31
      const uint32_t nan = __vcmpeq2(x, 0xc000c000u) | __vcmpeq2(y, 0xc000c000u);
      xl = __uint_as_float(__float_as_uint(xl) ^ ((sgn << 16) & 0x80000000u) |
                           ((nan << 16) & 0x7fc00000u));
      xh = __uint_as_float((__float_as_uint(xh) ^ (sgn & 0x80000000u)) |
                           (nan & 0x7fc00000u));
      acc.mac(2 * w, xl, yl);
      acc.mac(2 * w + 1, xh, yh);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *smem) {
    const uint32_t cx = load_code<16, 16>(xb, i), cy = load_code<16, 16>(yb, j);
    auto dec = [&](uint32_t c) {
      if (c == 0xc000u) return __uint_as_float(0x7fc00000u);
      const float m = at(smem, (c & 0x7fffu) << 2);
      return (c & 0x8000u) ? -m : m;
    };
    acc.mac_d(0, static_cast<double>(dec(cx)), static_cast<double>(dec(cy)));
  }
};

// lns16_r11 with the fused multiply (lns_decoder_strategies.cuh:353-367): the
// product of two LNS values is 2^((cx + cy) / 2048), so the two log codes are
// added and a single fraction-table lookup serves the pair.  Each 15-bit log
// code is biased by 2^14 (reserved code -> 0, finite codes -> [1, 2^15)), so
// one 32-bit add sums both halfwords of a word pair without a carry crossing
// them: halfword h = cx + cy + 2^15, whose low 11 bits index the fraction
// table and whose top 5 bits are the binary exponent + 16.  The power of two
// and the product's sign go into the accumulating FMA's second operand,
// +-2^(top - 16), so acc += T[f] * +-2^q is one FMA of the looked-up entry
// and the scale: exact, since products lie in [2^-16, 2^16) and are always
// normal, and the same rounding as adding the exact product.  Reserved codes
// follow lns::multiply_codes (lns_benchmark_core.hpp:241-254) without
// branches: adding 0x7fff to a biased halfword sets its top bit exactly when
// the code is not reserved, a sign-replicating byte permute spreads that bit
// into a mask that zeroes the scale of products with a zero operand, and a
// reserved code with its sign bit set (NaN) raises a flag that makes the DOT
// NaN.
template <typename T> struct lns16_fused_codec {
  static constexpr int kS = 16;
  static constexpr int kU = 4;
  static constexpr int kEntry = static_cast<int>(sizeof(T));
  // Interleaved copies of the fraction table: entry f of copy c at element
  // f * kCopies + c, lane l reading copy l % kCopies, so the lanes of a
  // half warp spread their random lookups over more banks.  Two copies of
  // the FP64 table (32 KiB): FP64, N = 2^28, 3755 -> 3936 GB/s (four: 3860,
  // eight: 1693); the FP32 table stays single (two copies: 5047 -> 4834).
  static constexpr int kCopies = sizeof(T) == 8 ? 2 : 1;
  static constexpr int kTableEntryBytes = kEntry * kCopies;
  static constexpr int kTableBytes = 2048 * kTableEntryBytes + 48;  // table + multipliers
  static constexpr bool kExactLanes = false;
  static constexpr int kMant = sizeof(T) == 4 ? 23 : 20;  // exponent shift in the top word
  static constexpr uint32_t kBias = sizeof(T) == 4 ? 127u : 1023u;

  // Field moves done as integer multiplies (x * 2^k for left shifts, the
  // high word of x * 2^k for right shifts, x * 1 + y for adds) run on the
  // FMA pipe instead of the ALU pipe, which the masks, permutes and logic
  // of this decode already fill.  The multipliers are read from shared
  // memory, so the compiler cannot turn them back into shifts.
  struct multipliers {
    uint32_t one;      // 1
    uint32_t k21;      // 2^21: low fraction (bits 0-10) -> bits 21-31, zeros below
    uint32_t off;      // 2^11 * kTableEntryBytes: bits 21-31 -> byte offset (high word)
    uint32_t off_hi;   // 2^16 * kTableEntryBytes: high fraction -> byte offset (high word)
    uint32_t e_lo;     // 2^(kMant - 11): low exponent (bits 11-15) -> exponent field
    uint32_t e_hi;     // 2^(kMant + 5): high exponent (bits 27-31) -> exponent field (high word)
    uint32_t e_bias;   // (kBias - 16) << kMant: exponent + 16 -> biased exponent of 2^q
    uint32_t sign_lo;  // 2^16: bit 15 -> bit 31
    uint32_t mag;      // 0x7fff7fff: both log fields
    uint32_t bias;     // 0x40004000: two's complement -> offset binary
    uint32_t pad[2];
  };
  static_assert(sizeof(multipliers) == kTableBytes - 2048 * kTableEntryBytes, "table layout");
  static constexpr int log2_int(int v) { return v <= 1 ? 0 : 1 + log2_int(v / 2); }

  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    const T *g = static_cast<const T *>(p.table);
    T *s = reinterpret_cast<T *>(smem);
    for (int e = threadIdx.x; e < 2048 * kCopies; e += blockDim.x) s[e] = g[e / kCopies];
    if (threadIdx.x == 0) {
      multipliers m{};
      m.one = 1u;
      m.k21 = 1u << 21;
      m.off = 1u << (11 + log2_int(kTableEntryBytes));
      m.off_hi = 1u << (16 + log2_int(kTableEntryBytes));
      m.e_lo = 1u << (kMant - 11);
      m.e_hi = 1u << (kMant + 5);
      m.e_bias = (kBias - 16u) << kMant;
      m.sign_lo = 1u << 16;
      m.mag = 0x7fff7fffu;
      m.bias = 0x40004000u;
      *reinterpret_cast<multipliers *>(smem + 2048 * kTableEntryBytes) = m;
    }
  }

  // every byte = copies of bit 7 of byte k of v (prmt sign replication)
  template <int K> __device__ __forceinline__ static uint32_t spread(uint32_t v) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(0u), "n"(0x8888 + 0x1111 * K));
    return r;
  }

  // +-2^q as T from the top word of its bit pattern
  __device__ __forceinline__ static T scale_of(uint32_t top) {
    if constexpr (sizeof(T) == 4)
      return __uint_as_float(top);
    else
      return __hiloint2double(static_cast<int>(top), 0);
  }

  // the exact product of two codes, specials included
  __device__ __forceinline__ static T multiply(uint32_t cx, uint32_t cy, const T *tab) {
    const uint32_t bx = (cx & 0x7fffu) ^ 0x4000u, by = (cy & 0x7fffu) ^ 0x4000u;
    const bool nan_x = bx == 0 && (cx & 0x8000u), nan_y = by == 0 && (cy & 0x8000u);
    if (nan_x || nan_y) {
      if constexpr (sizeof(T) == 4) return __uint_as_float(0x7fc00000u);
      else return __hiloint2double(0x7ff80000, 0);
    }
    const uint32_t sign = ((cx ^ cy) & 0x8000u) << 16;
    if (bx == 0 || by == 0) return scale_of(sign);
    const uint32_t h = bx + by;
    return tab[(h & 0x7ffu) * kCopies] * scale_of((((h >> 11) + kBias - 16u) << kMant) | sign);
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *,
                                                const unsigned char *smem) {
    static_assert(NV % 2 == 0, "two codes per word");
    const multipliers m = *reinterpret_cast<const multipliers *>(smem + 2048 * kTableEntryBytes);
    constexpr uint32_t kOff = 2047u * kTableEntryBytes;  // byte-offset mask
    const unsigned char *copy = smem + (threadIdx.x % kCopies) * kEntry;  // this lane's copy
    uint32_t nan = 0;
#pragma unroll
    for (int w = 0; w < NV / 2; ++w) {
      const uint32_t x = xw[w], y = yw[w];
      const uint32_t bx = (x & m.mag) ^ m.bias;  // one three-input logic op each
      const uint32_t by = (y & m.mag) ^ m.bias;
      const uint32_t h = bx * m.one + by;
      // bits 15 / 31: that code is not reserved
      const uint32_t lx = bx * m.one + 0x7fff7fffu, ly = by * m.one + 0x7fff7fffu;
      nan |= (x & ~lx) | (y & ~ly);  // reserved with the sign bit set
      const uint32_t live = lx & ly;
      const uint32_t sg = x ^ y;
      // the high word of (low fraction at bits 21-31, zeros below) * 2^11 *
      // kTableEntryBytes is fraction * kTableEntryBytes, with nothing to mask;
      // the high fraction has the low exponent below it, so it is masked
      const uint32_t off_lo = __umulhi(h * m.k21, m.off);
      const uint32_t off_hi = __umulhi(h, m.off_hi) & kOff;
      // biased exponent fields of 2^q (the exponent bits isolated first)
      const uint32_t e_lo = (h & 0xf800u) * m.e_lo + m.e_bias;
      const uint32_t e_hi = __umulhi(h & 0xf8000000u, m.e_hi) + m.e_bias;
      const uint32_t s_lo = (sg * m.sign_lo) & 0x80000000u;
      const uint32_t s_hi = sg & 0x80000000u;
      const T t_lo = *reinterpret_cast<const T *>(copy + off_lo);
      const T t_hi = *reinterpret_cast<const T *>(copy + off_hi);
      const T k_lo = scale_of((e_lo & spread<1>(live)) | s_lo);
      const T k_hi = scale_of((e_hi & spread<3>(live)) | s_hi);
      if constexpr (sizeof(T) == 4) {
        acc.mac(2 * w, t_lo, k_lo);
        acc.mac(2 * w + 1, t_hi, k_hi);
      } else {
        acc.mac_d(2 * w, t_lo, k_lo);
        acc.mac_d(2 * w + 1, t_hi, k_hi);
      }
    }
    if (nan & 0x80008000u) {
      if constexpr (sizeof(T) == 4)
        acc.mac(0, __uint_as_float(0x7fc00000u), 1.0f);
      else
        acc.mac_d(0, __hiloint2double(0x7ff80000, 0), 1.0);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc,
                                                const unsigned char *smem) {
    const T *tab = reinterpret_cast<const T *>(smem);
    acc.mac_d(0, static_cast<double>(multiply(load_code<16, 16>(xb, i),
                                              load_code<16, 16>(yb, j), tab)),
              1.0);
  }
};

// lns8_r3 / lns16_r11 with the hardware exponential: the reference's
// ex2_approx decoder (ex2.approx.f32, lns_decoder_strategies.cuh:215-224)
// with the fused multiply (:353-367).  The two log codes of a pair are added
// as in the fused table decoders (each biased by 2^(B-2), so one 32-bit add
// sums every lane of a word pair without carries between lanes), the sum is
// placed in the low bits of the FP32 pattern of 2^23 -- an exact integer
// conversion -- and one FMA by 2^-R rebiases it into the exponent argument
// (cx + cy) / 2^R, exactly; one ex2.approx.ftz.f32 per pair then gives the
// product's magnitude.  Zero and NaN codes follow lns::multiply_codes
// (lns_benchmark_core.hpp:241-254) without branches: the accumulating FMA's
// second operand is +-1, or 0 when a code of the pair is zero, and a NaN
// code raises a flag that makes the DOT NaN.  APPROXIMATE: every product
// carries the instruction's relative error (at most 2^-21 on B200, checked
// exhaustively over all log sums by the tests), so the DOT's normalised
// error bound grows by that much; it needs no table.
template <int B, typename T> struct lns_ex2_codec {
  static_assert(B == 8 || B == 16, "lns8_r3 and lns16_r11");
  static constexpr int kS = B;
  static constexpr int kU = 4;
  static constexpr int kTableBytes = 0;
  static constexpr bool kExactLanes = false;
  static constexpr int kR = B == 8 ? 3 : 11;
  static constexpr int kLanes = 32 / B;  // codes per word
  // field of one code, its offset-binary bias, and the bias of a pair's sum
  static constexpr uint32_t kMag = B == 8 ? 0x7f7f7f7fu : 0x7fff7fffu;
  static constexpr uint32_t kHalf = B == 8 ? 0x40404040u : 0x40004000u;
  static constexpr uint32_t kLive = B == 8 ? 0x7f7f7f7fu : 0x7fff7fffu;
  static constexpr uint32_t kTop = B == 8 ? 0x80808080u : 0x80008000u;
  // (2^23 + sum) * 2^-R - (2^23 + 2^(B-1)) * 2^-R = (cx + cy) / 2^R
  static constexpr float kScale = 1.0f / static_cast<float>(1 << kR);
  static constexpr float kShift =
      -static_cast<float>((8388608.0 + static_cast<double>(1u << (B - 1))) / (1 << kR));

  __device__ static void prepare(const dot_params &, unsigned char *) {}

  __device__ __forceinline__ static float ex2(float a) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
  }

  // every byte = copies of bit 7 of byte k of v (prmt sign replication)
  template <int K> __device__ __forceinline__ static uint32_t spread(uint32_t v) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(0u), "n"(0x8888 + 0x1111 * K));
    return r;
  }

  // lane k of the pair sums h as 2^23 + sum, in FP32
  template <int K> __device__ __forceinline__ static float placed(uint32_t h) {
    if constexpr (B == 8)
      return __uint_as_float(__byte_perm(h, 0x4B000000u, 0x7440 + K));
    else
      return __uint_as_float(__byte_perm(h, 0x4B000000u, K == 0 ? 0x7410 : 0x7432));
  }

  // the top bit of code field k, at bit 31
  template <int K> __device__ __forceinline__ static uint32_t top_of(uint32_t v) {
    return (v << (32 - B * (K + 1))) & 0x80000000u;
  }

  template <int K, class Acc>
  __device__ __forceinline__ static void pair(Acc &acc, int slot, uint32_t h, uint32_t live,
                                              uint32_t sg) {
    const float mag = ex2(fmaf(placed<K>(h), kScale, kShift));
    // byte holding the field's top bit: K for bytes, 2K + 1 for halfwords
    constexpr int kByte = B == 8 ? K : 2 * K + 1;
    const uint32_t on = spread<kByte>(live);
    if constexpr (sizeof(T) == 4) {
      acc.mac(slot, mag, __uint_as_float((on & 0x3f800000u) | top_of<K>(sg)));
    } else {
      acc.mac_d(slot, static_cast<double>(mag),
                __hiloint2double(static_cast<int>((on & 0x3ff00000u) | top_of<K>(sg)), 0));
    }
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *, const unsigned char *) {
    static_assert(NV % kLanes == 0, "whole words");
    uint32_t nan = 0;
#pragma unroll
    for (int w = 0; w < NV / kLanes; ++w) {
      const uint32_t x = xw[w], y = yw[w];
      const uint32_t bx = (x & kMag) ^ kHalf, by = (y & kMag) ^ kHalf;
      const uint32_t h = bx + by;  // lane k: cx + cy + 2^(B-1)
      // top bit of each lane: that code is not reserved
      const uint32_t lx = bx + kLive, ly = by + kLive;
      nan |= (x & ~lx) | (y & ~ly);  // reserved with the sign bit set
      const uint32_t live = lx & ly;
      const uint32_t sg = x ^ y;
      pair<0>(acc, kLanes * w, h, live, sg);
      pair<1>(acc, kLanes * w + 1, h, live, sg);
      if constexpr (B == 8) {
        pair<2>(acc, kLanes * w + 2, h, live, sg);
        pair<3>(acc, kLanes * w + 3, h, live, sg);
      }
    }
    if (nan & kTop) {
      if constexpr (sizeof(T) == 4)
        acc.mac(0, __uint_as_float(0x7fc00000u), 1.0f);
      else
        acc.mac_d(0, __hiloint2double(0x7ff80000, 0), 1.0);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc, const unsigned char *) {
    constexpr uint32_t field = (1u << (B - 1)) - 1u, half = 1u << (B - 2);
    const uint32_t cx = load_code<B, B>(xb, i), cy = load_code<B, B>(yb, j);
    const uint32_t bx = (cx & field) ^ half, by = (cy & field) ^ half;
    double v;
    if ((bx == 0 && (cx >> (B - 1))) || (by == 0 && (cy >> (B - 1)))) {
      v = __hiloint2double(0x7ff80000, 0);
    } else if (bx == 0 || by == 0) {
      v = 0.0;
    } else {
      const float a = static_cast<float>(static_cast<int>(bx + by) - (1 << (B - 1))) * kScale;
      v = static_cast<double>(ex2(a));
      if ((cx ^ cy) >> (B - 1)) v = -v;
    }
    acc.mac_d(0, v, 1.0);
  }
};

// Formats with codes of at most 8 bits and no dedicated codec (bit formats
// and LNS alike): the full decode table of the format, built on the host
// from the host decoder, replicated once per lane in shared memory (entry e
// of lane l at element e*32 + l) so a warp's lookups are conflict-free -- the
// reference's full_lut_shared decoder (bitwidth_benchmark_kernels.cuh:166-
// 288).  S is the slot width: the code width when dense, 8 for padded bytes.
// Full-table decode of the 9- to 14-bit E8 codes (decode_with_table with
// full_lut_shared, bitwidth_benchmark_kernels.cuh:166-200): one 32-bit word
// per code, read from a shared copy of the host table -- the FP32 bit pattern
// for the FP32 accumulator, the FP64 value's high word (its low word is zero
// for these codes) for the FP64 accumulator.  The table is not replicated
// (2^W words, up to 64 KiB), so lanes that look up different codes in one
// bank wait for each other.
template <int S, int W, typename T> struct wide_lut_codec {
  static_assert(W >= 9 && W <= 14, "codes of 9 to 14 bits");
  static constexpr int kS = S;
  static constexpr int kU = packet_shape<S>::Q == 1 ? 4 : 1;
  static constexpr int kTableBytes = (1 << W) * 4;
  static constexpr bool kExactLanes = false;

  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    const uint4 *g = static_cast<const uint4 *>(p.table);
    uint4 *s = reinterpret_cast<uint4 *>(smem);
    for (int e = threadIdx.x; e < (1 << W) / 4; e += blockDim.x) s[e] = g[e];
  }

  __device__ __forceinline__ static T value(uint32_t code, const unsigned char *smem) {
    const uint32_t word = reinterpret_cast<const uint32_t *>(smem)[code];
    if constexpr (sizeof(T) == 4)
      return __uint_as_float(word);
    else
      return __hiloint2double(static_cast<int>(word), 0);
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *, const unsigned char *smem) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const T a = value(field_low<S, W>(xw, v), smem);
      const T b = value(field_low<S, W>(yw, v), smem);
      if constexpr (sizeof(T) == 4)
        acc.mac(v, a, b);
      else
        acc.mac_d(v, a, b);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc, const unsigned char *smem) {
    acc.mac_d(0, static_cast<double>(value(load_code<S, W>(xb, i), smem)),
              static_cast<double>(value(load_code<S, W>(yb, j), smem)));
  }
};

// The reference's partial-table decoders of the E8 codes with 1 to 5
// mantissa bits (decode_with_table with prefix_lut_shared /
// subnormal_lut_shared, bitwidth_benchmark_kernels.cuh:229-259; they exist
// for formats of >= 9 bits with >= 2 exponent and >= 1 mantissa bits).
//   PREFIX:    a 512-entry table indexed by sign and exponent holds the
//              target's sign and exponent field (FP32 bits / FP64 high
//              word); the mantissa is ORed below it.  Zero/subnormal and
//              inf/NaN exponents take the direct bit move instead.
//   SUBNORMAL: a 2^M-entry table holds the subnormal values (exponent 0);
//              every other code takes the direct bit move.
// Both select between table and direct decode without branching.  They are
// exact and slower than the bit moves alone (one shared load and a select
// per code), kept for the decoder axis; AUTO never picks them.
template <int S, int W, typename T, bool kPrefix> struct part_lut_codec {
  static constexpr int kS = S;
  static constexpr int kW = W;
  static constexpr int kM = W - 9;
  static_assert(kM >= 1 && kM <= 5, "E8 codes with 1 to 5 mantissa bits");
  static constexpr int kEntries = kPrefix ? 512 : (1 << kM);
  static constexpr int kTableBytes = kEntries * 4 < 16 ? 16 : kEntries * 4;
  static constexpr int kU = packet_shape<S>::Q == 1 ? 4 : 1;
  static constexpr bool kExactLanes = false;
  // mantissa position in the target word (FP32 bits / FP64 high word)
  static constexpr int kShift = (sizeof(T) == 4 ? 23 : 20) - kM;

  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    const uint32_t *g = static_cast<const uint32_t *>(p.table);
    uint32_t *t = reinterpret_cast<uint32_t *>(smem);
    for (int e = threadIdx.x; e < kEntries; e += blockDim.x) t[e] = g[e];
  }

  __device__ __forceinline__ static T decode(uint32_t c, const uint32_t *tab) {
    const uint32_t e = (c >> kM) & 0xffu;
    const uint32_t f = c & ((1u << kM) - 1u);
    const uint32_t direct = c << (32 - W);  // FP32 bits, exact for every code
    uint32_t word;
    bool use_table;
    if constexpr (kPrefix) {
      word = tab[c >> kM] | (f << kShift);
      use_table = e - 1u < 254u;  // a normal exponent
    } else {
      word = tab[f] | ((c >> (W - 1)) << 31);
      use_table = e == 0u;
    }
    if constexpr (sizeof(T) == 4) {
      return __uint_as_float(use_table ? word : direct);
    } else {
      const double d = static_cast<double>(__uint_as_float(direct));
      const double w = __hiloint2double(static_cast<int>(word), 0);
      return use_table ? w : d;
    }
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw, const uint32_t *yw,
                                                Acc &acc, float *, const unsigned char *smem) {
    const uint32_t *tab = reinterpret_cast<const uint32_t *>(smem);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const T a = decode(field_low<S, W>(xw, v), tab);
      const T b = decode(field_low<S, W>(yw, v), tab);
      if constexpr (sizeof(T) == 4)
        acc.mac(v, a, b);
      else
        acc.mac_d(v, a, b);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j, Acc &acc,
                                                const unsigned char *smem) {
    const uint32_t *tab = reinterpret_cast<const uint32_t *>(smem);
    acc.mac_d(0, static_cast<double>(decode(load_code<S, W>(xb, i), tab)),
              static_cast<double>(decode(load_code<S, W>(yb, j), tab)));
  }
};

template <int S, typename T> struct lut_codec {
  static_assert(S >= 2 && S <= 8, "codes of 2 to 8 bits");
  using table = lane_table<T>;
  static constexpr int kS = S;
  static constexpr int kU = packet_shape<S>::Q == 1 ? 4 : 1;
  static constexpr int kEntries = 1 << S;
  static constexpr int kTableBytes = table::bytes(kEntries);
  static constexpr bool kExactLanes = false;

  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    // the format's codes (<= kEntries)
    table::fill(reinterpret_cast<T *>(smem), static_cast<const T *>(p.table), 1 << p.rt.bits);
  }

  __device__ __forceinline__ static uint32_t code(const uint32_t *w, int v) {
    if constexpr (S == 8)
      return __byte_perm(w[v >> 2], 0u, 0x4440u + (v & 3));
    else
      return field_low<S, S>(w, v);
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *, const unsigned char *smem) {
    const uint32_t lane_off = table::lane_offset();
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const T a = table::at(smem, code(xw, v), lane_off);
      const T b = table::at(smem, code(yw, v), lane_off);
      if constexpr (sizeof(T) == 4)
        acc.mac(v, a, b);
      else
        acc.mac_d(v, a, b);
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc, const unsigned char *smem) {
    const uint32_t lane_off = table::lane_offset();
    acc.mac_d(0, static_cast<double>(table::at(smem, load_code<S, S>(xb, i), lane_off)),
              static_cast<double>(table::at(smem, load_code<S, S>(yb, j), lane_off)));
  }
};

// The rest of the registry's bit formats (IEEE-like E/M of any width, E0
// fixed point, FP64 prefixes), decoded by runtime parameters: the code is
// moved to the top of a word (sign at bit 31), its magnitude shifted right
// so that its exponent field lands on the target's exponent field, and one
// multiply by 2^(target bias - format bias) rebiases it -- the half-to-float
// conversion, exact for normals and, through the hardware's denormal
// arithmetic, for subnormals (decode_words_masked,
// decoder_strategy_core.hpp:226-262, computes the same values with integer
// steps).  Formats with inf/NaN whose exponent is narrower than the target's
// build those explicitly.  S is the slot width (dense: the code width B;
// padded: the container, the code in its low B bits).
template <int S, typename T, bool kDense> struct rt_codec {
  static constexpr int kS = S;
  static constexpr int kU = 1;
  static constexpr int kTableBytes = static_cast<int>(sizeof(rt_params));
  static constexpr bool kExactLanes = false;
  __device__ static void prepare(const dot_params &p, unsigned char *smem) {
    if (threadIdx.x == 0) *reinterpret_cast<rt_params *>(smem) = p.rt;
  }

  // t: the code at bits [32 - B, 32); e: E; from: first inf/NaN magnitude
  __device__ __forceinline__ static float dec32(uint32_t t, uint32_t e, uint32_t from,
                                                float scale) {
    const uint32_t mag = t & 0x7fffffffu;
    uint32_t bits = (mag >> (8u - e)) | (t & 0x80000000u);
    if (from != 0u && mag >= from)
      bits = (t & 0x80000000u) | 0x7f800000u | ((t << (e + 1u)) >> 9);
    return __uint_as_float(bits) * scale;
  }
  __device__ __forceinline__ static double dec64(uint32_t t, uint32_t e, uint32_t from,
                                                 double scale) {
    const uint64_t sign = static_cast<uint64_t>(t & 0x80000000u) << 32;
    const uint64_t mag = static_cast<uint64_t>(t & 0x7fffffffu) << 32;
    uint64_t bits = (mag >> (11u - e)) | sign;
    if (from != 0u && (t & 0x7fffffffu) >= from)
      bits = sign | 0x7ff0000000000000ull | ((static_cast<uint64_t>(t << (e + 1u)) << 32) >> 12);
    return __longlong_as_double(static_cast<long long>(bits)) * scale;
  }

  __device__ __forceinline__ static uint32_t top(const uint32_t *w, int v, uint32_t shift) {
    if constexpr (kDense)
      return field_top<S, S>(w, v);
    else
      return field_low<S, S>(w, v) << shift;
  }

  template <int NV, class Acc>
  __device__ __forceinline__ static void values(const uint32_t *xw,
                                                const uint32_t *yw, Acc &acc,
                                                float *, const unsigned char *smem) {
    const rt_params &r = *reinterpret_cast<const rt_params *>(smem);
    const uint32_t shift = 32u - r.bits, e = r.exponent, from = r.special_from;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const uint32_t tx = top(xw, v, shift), ty = top(yw, v, shift);
      if constexpr (sizeof(T) == 4)
        acc.mac(v, dec32(tx, e, from, r.scale32), dec32(ty, e, from, r.scale32));
      else
        acc.mac_d(v, dec64(tx, e, from, r.scale64), dec64(ty, e, from, r.scale64));
    }
  }

  template <class Acc>
  __device__ __forceinline__ static void scalar(const unsigned char *xb, uint64_t i,
                                                const unsigned char *yb, uint64_t j,
                                                Acc &acc, const unsigned char *smem) {
    const rt_params &r = *reinterpret_cast<const rt_params *>(smem);
    const uint32_t shift = 32u - r.bits;
    const uint32_t tx = load_code<S, S>(xb, i) << shift, ty = load_code<S, S>(yb, j) << shift;
    if constexpr (sizeof(T) == 4)
      acc.mac_d(0, static_cast<double>(dec32(tx, r.exponent, r.special_from, r.scale32)),
                static_cast<double>(dec32(ty, r.exponent, r.special_from, r.scale32)));
    else
      acc.mac_d(0, dec64(tx, r.exponent, r.special_from, r.scale64),
                dec64(ty, r.exponent, r.special_from, r.scale64));
  }
};

// Tiles between carries of the FP32 lanes into FP64: at most 32 products per
// FP32 chain (4 chains; the stated error bound), or, for exact lanes, 16 tiles
// (far below the 4096 products an exact FP32 lane holds).
template <class Codec>
constexpr int flush_every(int values_per_tile) {
  if (Codec::kExactLanes) return 16;
  return values_per_tile >= 128 ? 1 : 128 / values_per_tile;
}

template <class Codec, class Acc>
__device__ __forceinline__ void flush_tile(Acc &acc, float *lanes) {
  if constexpr (Codec::kExactLanes) {
    acc.add_exact((static_cast<double>(lanes[0]) + static_cast<double>(lanes[1])) +
                  (static_cast<double>(lanes[2]) + static_cast<double>(lanes[3])));
    lanes[0] = lanes[1] = lanes[2] = lanes[3] = 0.f;
  }
  acc.flush();
}

template <class Codec, class Acc>
__device__ __forceinline__ void ragged_tail(const unsigned char *xb, uint64_t xo,
                                            const unsigned char *yb, uint64_t yo,
                                            uint64_t first, uint64_t n,
                                            Acc &acc, const unsigned char *smem) {
  for (uint64_t i = first + static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    Codec::scalar(xb, xo + i, yb, yo + i, acc, smem);
}

// ---------------------------------------------------------------------------
// COOPERATIVE strategy: the reference's cooperative shuffle loader
// (cooperative_raw / dot_cooperative_kernel, bitwidth_benchmark_kernels.cuh:
// 503-572; geometry bitwidth_benchmark_core.hpp:87-121) for dense streams.
// A group of `consumers` lanes owns one aligned chunk of `values` codes that
// spans `words` words: the first `words` lanes load one word each (a warp's
// loads are consecutive words), every lane then fetches the two words its
// codes lie in by two warp shuffles (the group's spare lanes hold 0 and
// serve as the guard word) and extracts values / consumers codes from the
// 64-bit pair.  Values past the last whole chunk take the per-value path.
// It reads every word once from global memory and never from shared memory;
// it stays behind the bulk-copy ring on B200 (shuffles and per-code shifts),
// kept for the access-method axis, never chosen by AUTO.
// ---------------------------------------------------------------------------
template <int W> struct coop_e8 {  // IEEE-like code with an 8-bit exponent
  __device__ __forceinline__ static float value(uint32_t c) {
    return __uint_as_float(c << (32 - W));
  }
};
struct coop_e2m3 {
  __device__ __forceinline__ static float value(uint32_t c) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e2m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<unsigned short>(c & 0x3fu)));
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h2)));
  }
};

template <int B, class Dec, class Acc>
__global__ void __launch_bounds__(kThreads) dot_coop_kernel(const dot_params p) {
  __shared__ double scratch[kScratchDoubles];
  using geo = aut::bitwidth::cooperative_geometry<B>;
  constexpr int C = geo::consumers;
  constexpr int WORDS = geo::words;
  constexpr int VALS = geo::values;
  constexpr int VPC = geo::values_per_consumer;
  constexpr int GROUPS = 32 / C;  // chunks per warp and step
  static_assert(VPC * B <= 32, "a consumer's codes lie in two words");
  constexpr uint32_t kMask = B == 32 ? 0xffffffffu : (1u << B) - 1u;

  const unsigned int batch = blockIdx.y;
  const unsigned char *xb = p.x + batch * p.x_stride;
  const unsigned char *yb = p.y + batch * p.y_stride;
  const uint64_t xo = p.x_first + batch * p.x_index_stride;
  const uint64_t yo = p.y_first + batch * p.y_index_stride;
  const uint32_t *xw = reinterpret_cast<const uint32_t *>(xb);
  const uint32_t *yw = reinterpret_cast<const uint32_t *>(yb);

  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t g = lane / C, c = lane % C;
  const uint32_t bit0 = c * VPC * B;
  const uint32_t src = g * C + (bit0 >> 5);  // lane holding the first word
  const uint32_t sh = bit0 & 31u;
  const uint64_t chunks = p.vector_ok ? p.n / VALS : 0;
  const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const uint64_t step = (static_cast<uint64_t>(gridDim.x) * kThreads >> 5) * GROUPS;

  pdl_wait();
  pdl_release();
  Acc acc;
  int since_flush = 0;
  // the loop bound is the same for all lanes of a warp (shuffles need them all)
  for (uint64_t base = warp * GROUPS; base < chunks; base += step) {
    const uint64_t chunk = base + g;
    const bool live = chunk < chunks;
    uint32_t wx = 0u, wy = 0u;
    if (live && c < static_cast<uint32_t>(WORDS)) {
      wx = __ldg(xw + chunk * WORDS + c);
      wy = __ldg(yw + chunk * WORDS + c);
    }
    const uint32_t x0 = __shfl_sync(0xffffffffu, wx, src);
    const uint32_t x1 = __shfl_sync(0xffffffffu, wx, src + 1);
    const uint32_t y0 = __shfl_sync(0xffffffffu, wy, src);
    const uint32_t y1 = __shfl_sync(0xffffffffu, wy, src + 1);
    if (live) {
      const uint64_t px = ((static_cast<uint64_t>(x1) << 32) | x0) >> sh;
      const uint64_t py = ((static_cast<uint64_t>(y1) << 32) | y0) >> sh;
#pragma unroll
      for (int v = 0; v < VPC; ++v)
        acc.mac(v, Dec::value(static_cast<uint32_t>(px >> (v * B)) & kMask),
                Dec::value(static_cast<uint32_t>(py >> (v * B)) & kMask));
    }
    if (++since_flush == 32 / VPC) {  // at most 32 products per FP32 chain
      acc.flush();
      since_flush = 0;
    }
  }
  acc.flush();
  // values past the whole chunks (or every value of an unaligned stream)
  for (uint64_t i = chunks * VALS + static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
       i < p.n; i += static_cast<uint64_t>(gridDim.x) * kThreads) {
    const float a = Dec::value(load_code<B, B>(xb, xo + i));
    const float b = Dec::value(load_code<B, B>(yb, yo + i));
    acc.mac_d(0, static_cast<double>(a), static_cast<double>(b));
  }
  const dd s = block_sum_dd(acc.pair(), scratch);
  grid_finish_dd(s, p.partials + 2 * static_cast<uint64_t>(batch) * gridDim.x,
                 p.tickets + batch, p.results + batch, scratch);
}

// ---------------------------------------------------------------------------
// LDG strategy: packets of Q 16-byte vectors straight into registers.
// ---------------------------------------------------------------------------
// Each thread loads its next tile's packets before it decodes the current
// one, so a warp keeps its loads in flight through the decode (N = 2^28 /
// 2^27, GB/s without -> with: lns8_r3 fused sum FP64 4098 -> 4554, e8m0 FP64
// 3605 -> 5236, e2m3 FP32 4982 -> 5833).  The lns16_r11 decoders are bound
// by the shared-memory pipe and lose occupancy to the second set of
// registers (fused, FP64: 3938 -> 3698), so they load one tile at a time.
template <class Codec> struct ldg_prefetch : std::true_type {};
template <typename T> struct ldg_prefetch<lns16_codec<T>> : std::false_type {};
template <typename T> struct ldg_prefetch<lns16_fused_codec<T>> : std::false_type {};
template <> struct ldg_prefetch<lns16_full_codec> : std::false_type {};

template <class Codec, class Acc>
__global__ void __launch_bounds__(kThreads)
    dot_ldg_kernel(const dot_params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ double scratch[kScratchDoubles];
  constexpr int S = Codec::kS;
  constexpr int Q = packet_shape<S>::Q;
  constexpr int P = packet_shape<S>::P;
  constexpr int U = Codec::kU;
  constexpr uint64_t tile_packets = static_cast<uint64_t>(kThreads) * U;

  const unsigned int batch = blockIdx.y;
  const unsigned char *xb = p.x + batch * p.x_stride;
  const unsigned char *yb = p.y + batch * p.y_stride;
  const uint64_t xo = p.x_first + batch * p.x_index_stride;
  const uint64_t yo = p.y_first + batch * p.y_index_stride;

  pdl_wait();
  pdl_release();
  if constexpr (Codec::kTableBytes > 0) {
    Codec::prepare(p, smem);
    __syncthreads();
  }

  Acc acc;
  float lanes[4] = {0.f, 0.f, 0.f, 0.f};
  const uint64_t tiles = p.vector_ok ? (p.n / P) / tile_packets : 0;
  const uint4 *X = reinterpret_cast<const uint4 *>(xb);
  const uint4 *Y = reinterpret_cast<const uint4 *>(yb);
  constexpr int kFlush = flush_every<Codec>(P * U);
  int since_flush = 0;
  constexpr bool kPrefetch = ldg_prefetch<Codec>::value;
  auto load_tile = [&](uint64_t t, uint4 (&a)[U][Q], uint4 (&b)[U][Q]) {
    const uint64_t first = t * tile_packets + threadIdx.x;
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        a[u][q] = __ldg(X + (first + static_cast<uint64_t>(u) * kThreads) * Q + q);
        b[u][q] = __ldg(Y + (first + static_cast<uint64_t>(u) * kThreads) * Q + q);
      }
    }
  };
  uint4 xv[U][Q], yv[U][Q];
  if (kPrefetch && static_cast<uint64_t>(blockIdx.x) < tiles) load_tile(blockIdx.x, xv, yv);
  for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    uint4 nx[kPrefetch ? U : 1][Q], ny[kPrefetch ? U : 1][Q];
    if constexpr (kPrefetch) {
      // the next tile's packets (unused past the last tile)
      if (t + gridDim.x < tiles) load_tile(t + gridDim.x, nx, ny);
    } else {
      load_tile(t, xv, yv);
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      Codec::template values<P>(reinterpret_cast<const uint32_t *>(xv[u]),
                                reinterpret_cast<const uint32_t *>(yv[u]), acc,
                                lanes, smem);
    if (++since_flush == kFlush) {
      flush_tile<Codec>(acc, lanes);
      since_flush = 0;
    }
    if constexpr (kPrefetch) {
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int q = 0; q < Q; ++q) {
          xv[u][q] = nx[u][q];
          yv[u][q] = ny[u][q];
        }
    }
  }
  flush_tile<Codec>(acc, lanes);

  ragged_tail<Codec>(xb, xo, yb, yo, tiles * tile_packets * P, p.n, acc, smem);
  const dd s = block_sum_dd(acc.pair(), scratch);
  grid_finish_dd(s, p.partials + 2 * static_cast<uint64_t>(batch) * gridDim.x,
                 p.tickets + batch, p.results + batch, scratch);
}

// ---------------------------------------------------------------------------
// TMA strategy: a shared-memory ring fed by cp.async.bulk.
// ---------------------------------------------------------------------------
// Geometry of one tile: a unit is UW = S / gcd(S, 32) words holding UV whole
// codes; every thread owns V units per tile, read GROUP consecutive units
// (LW words) per shared load.
// Units read per shared load: 1- and 2-word units four / two at a time (one
// 16-byte load); odd units of 3 words four at a time (12 words: three 16-byte
// loads, lanes 48 bytes apart, so a quarter warp covers 32 distinct banks) and
// of 5, 7 or 9 words two at a time (8-byte loads, lanes 2*UW words apart: a
// half warp covers 32 distinct banks); longer units one at a time.
constexpr int tma_group(int uw) {
  return uw <= 2 ? 4 / uw : (uw == 3 ? 4 : (uw <= 9 ? 2 : 1));
}
constexpr int tma_vpt(int s) {
  const int uw = s / gcd_int(s, 32), uv = s == 64 ? 1 : 32 / gcd_int(s, 32);
  const int base = s >= 24 ? 16 : (s <= 4 ? 128 : (s == 8 ? 64 : 32));
  return base >= tma_group(uw) * uv ? base : tma_group(uw) * uv;
}

template <int S, int RING = 64 * 1024, int VPT_ = tma_vpt(S), int NT_ = kThreads>
struct tma_shape {
  static constexpr int NT = NT_;                   // threads per block
  static constexpr int G = gcd_int(S, 32);
  static constexpr int UW = S / G;                 // words per unit
  static constexpr int UV = S == 64 ? 1 : 32 / G;  // codes per unit
  static constexpr int VPT = VPT_;                 // codes per thread per tile
  static constexpr int V = VPT / UV;               // units per thread per tile
  static constexpr int GROUP = tma_group(UW) < V ? tma_group(UW) : V;  // units per load
  static constexpr int LW = UW * GROUP;            // words per load
  static constexpr int TILE_WORDS = NT * V * UW;
  static constexpr int TILE_BYTES = TILE_WORDS * 4;  // per vector
  static constexpr uint64_t TILE_VALUES = static_cast<uint64_t>(NT) * VPT;
  static constexpr int RING_BYTES = RING;
  static constexpr int STAGES_RAW = RING_BYTES / (2 * TILE_BYTES);
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
  static_assert(TILE_BYTES % 16 == 0, "bulk copies move 16-byte multiples");
  static_assert(V * UV == VPT, "units tile the thread's codes");
  static_assert(V % GROUP == 0, "loads tile the thread's units");
};

// Codecs with a shared decode table get a 32 KiB ring, so that more blocks
// -- more warps to hide the table lookups' latency -- fit an SM beside the
// table (lns8_r3, FP32: 5116 -> 5432 GB/s; 16-bit codes keep two 32 KiB
// stages, since halving their tiles cost 5 %).
// Ring per slot width, from a sweep of 48-200 KiB on B200 (N = 2^27, FP32
// accumulator, GB/s at 64 KiB -> chosen): 9 bits 5773 -> 6118 (160 KiB),
// 10 bits 5882 -> 6328 (128), 12 bits 6182 -> 6418 (128), 14 bits 6414 ->
// 6514 (160), 24 bits 6829 -> 6895 (128); 6 bits keeps 64 KiB (5429; 4266 at
// 128).  The winners hold one block per SM with four to six stages in flight.
// The FP64 accumulator keeps 64 KiB: its longer per-pair work wants more
// warps instead (e8m0 5751 at 64 KiB, 4748 at 160; halving e8m0's tile to 32
// codes per thread: 5457 at 64 KiB, 5104 at 96).
constexpr int tma_ring(int s, bool fp64) {
  if (fp64) return s == 24 ? 128 * 1024 : 64 * 1024;  // 24 bits: e8m15 6368 -> 6649
  return s == 9 || s == 14 ? 160 * 1024 : (s == 10 || s == 12 || s == 24 ? 128 * 1024 : 64 * 1024);
}

// A batch of pairs -- rows of a GEMV among them -- gives every pair a short
// stream that a deep ring with one block per SM starts slowly (E8 GEMV rows,
// 1024 x 2^17: 2377 GB/s at 160 KiB, 3876 at 64 KiB), so batched launches
// run a second instantiation with the 64 KiB ring (`Short`). The ring depth
// stays a compile-time constant: read from the launch parameters instead,
// it cost the 10-bit codes 14 % (6337 -> 5475 GB/s).
// Threads per block of the bulk-copy kernel.  Co-resident blocks of one
// kernel do not stream at equal speed, so fewer, larger blocks per SM finish
// closer together; whether that beats the extra warps of more blocks
// depends on the decode.  From sweeps of 256/512/1024 threads on B200 (N =
// 2^27, GB/s at 256 -> chosen): e2m3 dense 5548 -> 5622 (512), padded 4625
// -> 4685 (512); e8m1 FP32 5915 -> 6295 (512); bf16 FP32 / FP64 6702 / 6411
// -> 6809 / 6654 (512); padded E8 codes e8m0 3747 -> 3822, e8m3 FP64 4821
// -> 4974 (512); raw FP32 6795 -> 7050 (512); e8m3 FP64 6129 -> 6324
// (1024); e8m15 6711 -> 6889 (1024).  The others keep 256 (e8m0 and e8m1
// FP64 lose 1-12 % at 512).
template <class Codec> struct e8_shape {
  static constexpr int S = 0, W = 0;
};
template <int S_, int W_> struct e8_shape<e8_codec<S_, W_>> {
  static constexpr int S = S_, W = W_;
};
template <class Codec, class Acc>
constexpr int tma_threads() {
  constexpr int S = e8_shape<Codec>::S, W = e8_shape<Codec>::W;
  constexpr bool f32 = std::is_same_v<Acc, acc_f32>;
  if constexpr (std::is_same_v<Codec, e2m3_codec<6>> || std::is_same_v<Codec, e2m3_codec<8>>)
    return 512;
  else if constexpr ((S == 24 && W == 24) || (S == 12 && W == 12 && !f32))
    return 1024;
  else if constexpr ((S == 10 && W == 10 && f32) || S == 16 || S == 32)
    return 512;
  else
    return kThreads;
}

template <class Codec, class Acc, bool Short>
constexpr int tma_ring_of() {
  if (Codec::kTableBytes > 1024) return 32 * 1024;
  const int base = Short ? 64 * 1024
                         : tma_ring(Codec::kS, !std::is_same_v<Acc, acc_f32> &&
                                                   !std::is_same_v<Acc, acc_f32c>);
  // blocks of 512 or 1024 threads take twice the ring of their 256-thread
  // configuration, within 192 KiB
  const int ring = tma_threads<Codec, Acc>() > kThreads ? 2 * base : base;
  return ring > 192 * 1024 ? 192 * 1024 : ring;
}

// Codes per thread per tile of the bulk-copy kernel.
template <class Codec, class Acc>
constexpr int tma_vpt_of() {
  return tma_vpt(Codec::kS);
}

template <class Codec, class Acc, bool Short = false>
using tma_shape_of = tma_shape<Codec::kS, tma_ring_of<Codec, Acc, Short>(),
                               tma_vpt_of<Codec, Acc>(), tma_threads<Codec, Acc>()>;

// Whether the codec's single-DOT ring is deeper than the batched one.
template <class Codec, class Acc>
constexpr bool has_short_ring =
    tma_shape_of<Codec, Acc, false>::STAGES != tma_shape_of<Codec, Acc, true>::STAGES;

constexpr long long kWaitCycles = aut::kWaitCyclesDefault;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Returns false when the phase did not complete within `limit` cycles.
__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

// The common case (the tile has landed) costs one try_wait; the clock is
// read only once the first try fails, and then every 32 tries.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          long long limit = kWaitCycles) {
  const uint32_t addr = smem_addr(bar);
  if (mbar_try(addr, parity)) return true;
  const long long start = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(addr, parity)) return true;
    if ((i & 31u) == 0u && clock64() - start > limit) return false;
  }
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src,
                                          uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

template <class Codec, class Acc, bool Short = false>
__global__ void __launch_bounds__(tma_shape_of<Codec, Acc, Short>::NT)
    dot_tma_kernel(const dot_params p) {
  using shape = tma_shape_of<Codec, Acc, Short>;
  constexpr int NT = shape::NT;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ double scratch[scratch_doubles<NT>];
  constexpr int UV = shape::UV;
  constexpr int V = shape::V;
  constexpr int GROUP = shape::GROUP;
  constexpr int LW = shape::LW;
  constexpr int STAGES = shape::STAGES;
  constexpr int TILE_BYTES = shape::TILE_BYTES;
  __shared__ __align__(8) uint64_t full[STAGES];

  const unsigned int batch = blockIdx.y;
  const unsigned char *xb = p.x + batch * p.x_stride;
  const unsigned char *yb = p.y + batch * p.y_stride;
  const uint64_t xo = p.x_first + batch * p.x_index_stride;
  const uint64_t yo = p.y_first + batch * p.y_index_stride;
  unsigned char *ring = smem + Codec::kTableBytes;

  // Tiles are dealt round-robin: block b takes tiles b, b + G, ... (G =
  // gridDim.x).  Co-resident blocks do not stream at equal speed (the SM's
  // warp scheduler favours some), so with equal static shares the last
  // blocks of a launch finish several microseconds after the median one.
  // For codecs whose DOT is exact (kExactLanes: every partial sum is exact,
  // so the summation order cannot change the result) the last kClaimRounds
  // rounds of tiles are instead claimed one at a time from a counter
  // (p.claims) by whichever block is free, which evens the finish out and
  // keeps the result bit-identical.  The block holding the last ticket
  // resets the counter.
  constexpr uint64_t kNoTile = ~0ull;
  constexpr uint64_t kClaimRounds = 2;
  constexpr bool kMayClaim = Codec::kExactLanes;
  const uint64_t G = gridDim.x;
  const uint64_t tiles = p.vector_ok ? p.n / shape::TILE_VALUES : 0;
  const bool claiming = kMayClaim && p.claims != nullptr && tiles / G > kClaimRounds;
  const uint64_t fixed_rounds = claiming ? tiles / G - kClaimRounds : 0;
  const uint64_t mine =  // statically dealt tiles of this block
      claiming ? fixed_rounds
               : (tiles > blockIdx.x ? (tiles - blockIdx.x + G - 1) / G : 0);
  __shared__ uint64_t stage_tile[kMayClaim ? STAGES : 1];

  // Tile of the block's k-th stage fill (thread 0 only, in increasing k):
  // dealt, claimed, or kNoTile once none is left (then every later k too).
  auto tile_of = [&](uint64_t k) -> uint64_t {
    if (k < mine) return blockIdx.x + k * G;
    if (!claiming) return kNoTile;
    const uint64_t t = fixed_rounds * G + atomicAdd(p.claims + batch, 1u);
    return t < tiles ? t : kNoTile;
  };
  auto issue = [&](uint64_t t, uint32_t stage) {
    unsigned char *dst = ring + stage * (2 * TILE_BYTES);
    uint64_t *bar = &full[stage];
    if constexpr (kMayClaim) stage_tile[stage] = t;  // ordered by the arrive below
    mbar_expect_tx(bar, t == kNoTile ? 0u : 2u * TILE_BYTES);
    if (t == kNoTile || t == p.stall_tile) return;  // stall: failure-detection test
    bulk_load(dst, xb + t * TILE_BYTES, TILE_BYTES, bar);
    bulk_load(dst + TILE_BYTES, yb + t * TILE_BYTES, TILE_BYTES, bar);
  };
  // Fills k = 0 .. in flight after the loop stopped at k (claiming: every
  // stage is refilled each round, with kNoTile at the end).
  auto armed = [&](uint64_t j) { return claiming || j < mine; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  pdl_wait();
  pdl_release();
  if constexpr (Codec::kTableBytes > 0) Codec::prepare(p, smem);
  __syncthreads();
  if (threadIdx.x == 0)
    for (uint32_t k = 0; k < static_cast<uint32_t>(STAGES) && armed(k); ++k)
      issue(tile_of(k), k);

  Acc acc;
  float lanes[4] = {0.f, 0.f, 0.f, 0.f};
  bool failed = false;
  constexpr int kFlush = flush_every<Codec>(shape::VPT);
  int since_flush = 0;
  uint32_t stage = 0, phase = 0;  // k % STAGES and (k / STAGES) & 1
  uint64_t k = 0;
  for (; claiming || k < mine; ++k) {
    const bool ok = mbar_wait(&full[stage], phase, p.wait_cycles);
    if constexpr (kMayClaim)
      if (claiming && stage_tile[stage] == kNoTile) break;  // the same for all threads
    const uint32_t *xs = reinterpret_cast<const uint32_t *>(ring + stage * (2 * TILE_BYTES));
    const uint32_t *ys = xs + shape::TILE_WORDS;
#pragma unroll
    for (int v = 0; v < V / GROUP; ++v) {
      const int u = threadIdx.x + v * NT;  // load index
      uint32_t xw[LW], yw[LW];
      if constexpr (LW % 4 == 0) {
#pragma unroll
        for (int q = 0; q < LW / 4; ++q) {
          const uint4 a = reinterpret_cast<const uint4 *>(xs)[u * (LW / 4) + q];
          const uint4 b = reinterpret_cast<const uint4 *>(ys)[u * (LW / 4) + q];
          xw[4 * q] = a.x; xw[4 * q + 1] = a.y; xw[4 * q + 2] = a.z; xw[4 * q + 3] = a.w;
          yw[4 * q] = b.x; yw[4 * q + 1] = b.y; yw[4 * q + 2] = b.z; yw[4 * q + 3] = b.w;
        }
      } else if constexpr (LW % 2 == 0) {
#pragma unroll
        for (int q = 0; q < LW / 2; ++q) {
          const uint2 a = reinterpret_cast<const uint2 *>(xs)[u * (LW / 2) + q];
          const uint2 b = reinterpret_cast<const uint2 *>(ys)[u * (LW / 2) + q];
          xw[2 * q] = a.x; xw[2 * q + 1] = a.y;
          yw[2 * q] = b.x; yw[2 * q + 1] = b.y;
        }
      } else {
#pragma unroll
        for (int w = 0; w < LW; ++w) {
          xw[w] = xs[u * LW + w];
          yw[w] = ys[u * LW + w];
        }
      }
      Codec::template values<UV * GROUP>(xw, yw, acc, lanes, smem);
    }
    if (++since_flush == kFlush) {
      flush_tile<Codec>(acc, lanes);
      since_flush = 0;
    }
    // Every thread is done with this stage (and the exit decision is the
    // same for all threads) before it is refilled.
    if (__syncthreads_or(ok ? 0 : 1)) {
      failed = true;
      break;
    }
    if (threadIdx.x == 0 && (claiming || k + STAGES < mine)) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(tile_of(k + STAGES), stage);
    }
    if (++stage == static_cast<uint32_t>(STAGES)) {
      stage = 0;
      phase ^= 1u;
    }
  }
  flush_tile<Codec>(acc, lanes);
  if (failed) {
    // Let the copies this block still has in flight land before it exits.
    if (threadIdx.x == 0) {
      for (uint64_t j = k; armed(j) && j < k + STAGES; ++j)
        mbar_wait(&full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1),
                  p.wait_cycles);
      atomicOr(p.status, static_cast<unsigned int>(AUT_STATUS_WAIT_TIMEOUT));
    }
    __syncthreads();
  } else {
    ragged_tail<Codec>(xb, xo, yb, yo, tiles * shape::TILE_VALUES, p.n, acc, smem);
  }
  const dd mine_sum = failed ? dd{__longlong_as_double(0x7ff8000000000000ll), 0.0} : acc.pair();
  const dd s = block_sum_dd<NT>(mine_sum, scratch);
  grid_finish_dd<NT>(s, p.partials + 2 * static_cast<uint64_t>(batch) * gridDim.x,
                     p.tickets + batch, p.results + batch, scratch,
                     claiming ? p.claims + batch : nullptr);
}


// ---------------------------------------------------------------------------
// GEMV with the vector decoded once per block (FP32 accumulation of the E8
// codes and raw FP32; e2m3, exact, with either accumulator).  Block (s, b) owns column segment s -- one tile of the DOT
// kernels' shape, so one bulk copy per row -- and the contiguous rows of
// groups [b * groups_per_block, (b + 1) * groups_per_block).  It decodes its
// vector segment into registers once, streams its rows' tiles through the
// bulk-copy ring, and multiplies each row tile by the register-resident
// vector: one decode per matrix element instead of two.  Every thread's row
// partial (two FP32 chains of at most 32 products, summed in FP64) is staged
// in shared memory; after each group of eight rows one warp per row sums its
// 256 partials in a fixed order into the row's segment partial; a second
// kernel sums each row's segment partials in segment order, so results do
// not depend on scheduling (and the streaming kernel issues no fences or
// atomics).
// ---------------------------------------------------------------------------
struct gemv_params {
  const unsigned char *matrix;  // row r at matrix + r * row_bytes
  const unsigned char *vector;
  uint64_t row_bytes;
  uint32_t rows;               // rows of this launch
  uint32_t groups_per_block;   // groups of gemv_rows<Codec>() rows
  double *partials;            // [rows][gridDim.x]
  unsigned int *status;
  const void *table;           // decode table (lns8_r3)
};

template <class Codec> struct is_e2m3 : std::false_type {};
template <int S> struct is_e2m3<e2m3_codec<S>> : std::true_type {};

// Rows per group (at most one warp per row): 4 for 9-bit codes, whose
// 18 KiB tiles leave room for a third ring stage when the row staging
// halves (e8m0 4590 -> 4859 GB/s), and for dense e2m3, which fits another
// block per SM (3038 -> 3348); 8 for the others (e8m5 5685 at 8 rows, 5443
// at 4).
template <class Codec> constexpr int gemv_rows() {
  return Codec::kS == 9 || Codec::kS == 6 ? 4 : kThreads / 32;
}

// c + a * b for two bf16 values, exact product, one rounding (the sm_100
// mixed-precision FMA): `a_top` holds a in its high half (FP32 bits whose low
// half is zero), `pair` holds b in its low (H = false) or high (H = true) half.
template <bool H>
__device__ __forceinline__ float fma_bf16(uint32_t a_top, uint32_t pair, float c) {
  if constexpr (H)
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, ah, bh, %0;\n\t}"
        : "+f"(c)
        : "r"(a_top), "r"(pair));
  else
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, ah, bl, %0;\n\t}"
        : "+f"(c)
        : "r"(a_top), "r"(pair));
  return c;
}

// One operand per stage (tma_shape's ring counts two, so the ring is half the
// figure).  From sweeps of 64-256 on B200 (1024 x 2^17, FP32, GB/s at 96 /
// 128): e8m0 4590 / 4322, e8m1 5107 / 4480, e8m3 5408 / 5224, e8m5 5651 /
// 5477, bf16 5829 / 5934, e8m15 6284 / 6282: beside the 16 KiB row staging a
// bigger ring costs a block per SM, except for 16-bit codes; 9-bit codes
// stage 8 KiB of rows and take the third stage (see gemv_rows).
constexpr int gemv_ring(int s) { return (s == 16 || s == 9 ? 128 : 96) * 1024; }

// FP64 rows of lns8_r3 (the vector held as FP64 values): 32 codes per
// thread and a 32 KiB stage ring beside the 32 KiB table, two blocks per SM.
template <class Codec> constexpr bool is_lns8_f64 = std::is_same_v<Codec, lns8_codec<double, 16>>;

template <class Codec>
using gemv_shape = tma_shape<Codec::kS, is_lns8_f64<Codec> ? 64 * 1024 : gemv_ring(Codec::kS),
                             is_lns8_f64<Codec> ? 32
                                                : (tma_vpt(Codec::kS) > 32 ? tma_vpt(Codec::kS) : 32)>;

__device__ __forceinline__ void gemv_publish(const gemv_params &g, uint32_t r, double v) {
  g.partials[static_cast<uint64_t>(r) * gridDim.x + blockIdx.x] = v;
}

// results[r] = the sum of row r's segment partials: one warp per row, lane l
// taking segments l, l + 32, ... in order, then the warp's fixed tree.
__global__ void __launch_bounds__(kThreads)
    gemv_rows_kernel(const double *partials, uint32_t segments, uint32_t rows,
                     double *results) {
  pdl_wait();  // the streaming kernel's partials
  pdl_release();
  const uint32_t r = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  const uint32_t lane = threadIdx.x & 31;
  if (r >= rows) return;
  const double *row = partials + static_cast<uint64_t>(r) * segments;
  double s = 0.0;
  for (uint32_t j = lane; j < segments; j += 32) s += row[j];
  s = warp_sum(s);
  if (lane == 0) results[r] = s;
}

// Three blocks per SM for the 12-bit codes (e8m3 4895 -> 5228 GB/s); the
// 9-bit kernel's register-resident 64-value vector spills under that bound
// (4330 -> 3873), the other widths do not change.  The FP64 rows take the
// bound too: unbounded, the compiler spends 200-255 registers on them.
//
// F64 (FP64 accumulator): 24- and 32-bit codes multiply both operands
// widened to FP64 (exact products).  For E8 codes of at most 16 bits the product of a
// matrix code and a vector value -- two bf16 values -- is exact in FP32
// unless it falls below 2^-126 or overflows, so each product is widened to
// FP64 once and summed in FP64 (as the DOT's e8_codec does); a chunk of 16
// values whose smallest |product| is below 2^-126 (zeros included) or whose
// sum is not finite is summed again from both operands widened, so every
// row is an FP64 sum of exact products either way.
template <class Codec, bool F64 = false>
__global__ void __launch_bounds__(kThreads, Codec::kS == 12 || F64 ? 3 : 1)
    gemv_tma_kernel(const gemv_params g) {
  extern __shared__ __align__(128) unsigned char smem[];
  using shape = gemv_shape<Codec>;
  constexpr int S = Codec::kS;
  constexpr int W = Codec::kW;
  constexpr int UV = shape::UV;
  constexpr int V = shape::V;
  constexpr int GROUP = shape::GROUP;
  constexpr int LW = shape::LW;
  constexpr int VPT = shape::VPT;
  constexpr int STAGES = shape::STAGES;
  constexpr int TILE_BYTES = shape::TILE_BYTES;
  static_assert(VPT <= 64, "two chains of at most 32 products per row tile");
  static_assert(!F64 || (!is_e2m3<Codec>::value && Codec::kTableBytes == 0),
                "FP64 rows for the E8 codes and raw FP32");
  __shared__ __align__(8) uint64_t full[STAGES];
  unsigned char *ring = smem + Codec::kTableBytes;
  constexpr int kRows = gemv_rows<Codec>();
  double *red = reinterpret_cast<double *>(ring + STAGES * TILE_BYTES);  // [kRows][kThreads]
  constexpr bool kE2m3 = is_e2m3<Codec>::value;

  const uint32_t first_row = blockIdx.y * g.groups_per_block * kRows;
  const uint32_t end_row = min(g.rows, first_row + g.groups_per_block * kRows);
  const uint32_t tiles = end_row > first_row ? end_row - first_row : 0;
  const unsigned char *seg = g.matrix + static_cast<uint64_t>(blockIdx.x) * TILE_BYTES;

  auto issue = [&](uint32_t t, uint32_t stage) {
    uint64_t *bar = &full[stage];
    mbar_expect_tx(bar, TILE_BYTES);
    bulk_load(ring + stage * TILE_BYTES, seg + static_cast<uint64_t>(first_row + t) * g.row_bytes,
              TILE_BYTES, bar);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  pdl_wait();
  pdl_release();
  if constexpr (Codec::kTableBytes > 0) {
    dot_params tp{};
    tp.table = g.table;
    Codec::prepare(tp, smem);
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (uint32_t t = 0; t < tiles && t < static_cast<uint32_t>(STAGES); ++t) issue(t, t);

  // this thread's codes of the vector segment, decoded once: codes of up to
  // 16 bits are bf16 values exactly and are kept as bf16 pairs (half the
  // registers, so more blocks fit an SM); wider ones as FP32; e2m3 codes as
  // the f16 pairs of the hardware conversion; lns8_r3 codes as the FP32 (or,
  // for FP64 rows, FP64) values of their per-lane table
  constexpr bool kLns = std::is_same_v<Codec, lns8_codec<float>>;
  constexpr bool kLns64 = is_lns8_f64<Codec>;
  constexpr bool kPairs = W <= 16 && !kLns && !kLns64;
  float vec[kPairs || kLns64 ? 1 : VPT];
  double vecd[kLns64 ? VPT : 1];
  uint32_t vec2[kPairs ? VPT / 2 : 1];
  {
    const uint32_t *vw = reinterpret_cast<const uint32_t *>(
        g.vector + static_cast<uint64_t>(blockIdx.x) * TILE_BYTES);
#pragma unroll
    for (int v = 0; v < V / GROUP; ++v) {
      const int u = threadIdx.x + v * kThreads;
      uint32_t w[LW];
#pragma unroll
      for (int q = 0; q < LW; ++q) w[q] = __ldg(vw + u * LW + q);
      if constexpr (kE2m3) {
#pragma unroll
        for (int q = 0; q < UV * GROUP / 4; ++q) {
          const int j = (v * UV * GROUP) / 2 + 2 * q;  // f16 pair index
          Codec::to_f16x2x2(Codec::bytes4(w, q, smem), vec2[j], vec2[j + 1]);
        }
        continue;
      }
      if constexpr (kLns || kLns64) {
        const uint32_t lane_off = Codec::table::lane_offset();
#pragma unroll
        for (int i = 0; i < UV * GROUP; ++i) {
          const auto dv =
              Codec::table::at(smem, __byte_perm(w[i >> 2], 0u, 0x4440u + (i & 3)), lane_off);
          if constexpr (kLns64)
            vecd[v * UV * GROUP + i] = dv;
          else
            vec[v * UV * GROUP + i] = dv;
        }
        continue;
      }
#pragma unroll
      for (int i = 0; i < UV * GROUP; ++i) {
        const uint32_t bits = field_top<S, W>(w, i);
        const int j = v * UV * GROUP + i;
        if constexpr (kPairs) {
          if (j & 1)
            vec2[j >> 1] = __byte_perm(vec2[j >> 1], bits, 0x7610);
          else
            vec2[j >> 1] = bits >> 16;
        } else {
          vec[j] = __uint_as_float(bits);
        }
      }
    }
  }

  // Rings of four or more stages consume two row tiles per block barrier.
  constexpr uint32_t kPerSync = STAGES >= 4 ? 2 : 1;
  bool failed = false;
  uint32_t stage = 0, phase = 0, k = 0, done = 0;  // done: rows finished
  for (uint32_t t = 0; t < tiles; t += kPerSync) {
    const uint32_t n = tiles - t < kPerSync ? tiles - t : kPerSync;  // same in every thread
    bool ok = true;
#pragma unroll
    for (uint32_t h = 0; h < kPerSync; ++h) {
      if (h >= n) break;
      uint32_t st = stage + h, ph = phase;
      if (st >= static_cast<uint32_t>(STAGES)) {
        st -= STAGES;
        ph ^= 1u;
      }
      ok = mbar_wait(&full[st], ph) && ok;
      const uint32_t *ws = reinterpret_cast<const uint32_t *>(ring + st * TILE_BYTES);
      float c0 = 0.f, c1 = 0.f;
      double d0 = 0.0, d1 = 0.0;  // F64, kLns64
#pragma unroll
      for (int v = 0; v < V / GROUP; ++v) {
        const int u = threadIdx.x + v * kThreads;
        uint32_t w[LW];
        if constexpr (LW % 4 == 0) {
#pragma unroll
          for (int q = 0; q < LW / 4; ++q) {
            const uint4 a = reinterpret_cast<const uint4 *>(ws)[u * (LW / 4) + q];
            w[4 * q] = a.x; w[4 * q + 1] = a.y; w[4 * q + 2] = a.z; w[4 * q + 3] = a.w;
          }
        } else if constexpr (LW % 2 == 0) {
#pragma unroll
          for (int q = 0; q < LW / 2; ++q) {
            const uint2 a = reinterpret_cast<const uint2 *>(ws)[u * (LW / 2) + q];
            w[2 * q] = a.x; w[2 * q + 1] = a.y;
          }
        } else {
#pragma unroll
          for (int q = 0; q < LW; ++q) w[q] = ws[u * LW + q];
        }
        if constexpr (kLns) {
          const uint32_t lane_off = Codec::table::lane_offset();
#pragma unroll
          for (int i = 0; i < UV * GROUP; ++i) {
            const int j = v * UV * GROUP + i;
            const float mv =
                Codec::table::at(smem, __byte_perm(w[i >> 2], 0u, 0x4440u + (i & 3)), lane_off);
            if (i & 1)
              c1 = fmaf(mv, vec[j], c1);
            else
              c0 = fmaf(mv, vec[j], c0);
          }
          continue;
        }
        if constexpr (kLns64) {
          // exact products of the decoded FP64 values, values 2k and 2k + 1
          // on one chain (as the DOT's FP64 accumulator)
          const uint32_t lane_off = Codec::table::lane_offset();
#pragma unroll
          for (int i = 0; i < UV * GROUP; ++i) {
            const int j = v * UV * GROUP + i;
            const double mv =
                Codec::table::at(smem, __byte_perm(w[i >> 2], 0u, 0x4440u + (i & 3)), lane_off);
            if ((i >> 1) & 1)
              d1 = fma(mv, vecd[j], d1);
            else
              d0 = fma(mv, vecd[j], d0);
          }
          continue;
        }
        if constexpr (F64 && W > 16) {
          // 24- and 32-bit codes: both operands widened, exact products
#pragma unroll
          for (int i = 0; i < UV * GROUP; ++i) {
            const int j = v * UV * GROUP + i;
            d0 = fma(static_cast<double>(__uint_as_float(field_top<S, W>(w, i))),
                     static_cast<double>(vec[j]), d0);
          }
          continue;
        }
        if constexpr (F64) {
          constexpr int C = UV * GROUP < 16 ? UV * GROUP : 16;  // values per check
          static_assert((UV * GROUP) % C == 0, "whole chunks");
#pragma unroll
          for (int i0 = 0; i0 < UV * GROUP; i0 += C) {
            double s0 = 0.0, s1 = 0.0;
            float smallest = __int_as_float(0x7f800000);
#pragma unroll
            for (int i = i0; i < i0 + C; ++i) {
              const int j = v * UV * GROUP + i;
              const uint32_t m = field_top<S, W>(w, i);
              const float pr = (j & 1) ? fma_bf16<true>(m, vec2[j >> 1], 0.f)
                                       : fma_bf16<false>(m, vec2[j >> 1], 0.f);
              smallest = fminf(smallest, fabsf(pr));
              if (j & 1)
                s1 += static_cast<double>(pr);
              else
                s0 += static_cast<double>(pr);
            }
            const double sc = s0 + s1;
            if (smallest >= 1.17549435e-38f && fabs(sc) <= 1.7976931348623157e308) {
              d0 += sc;
            } else {
#pragma unroll
              for (int i = i0; i < i0 + C; ++i) {
                const int j = v * UV * GROUP + i;
                const uint32_t vb = (j & 1) ? (vec2[j >> 1] & 0xffff0000u) : (vec2[j >> 1] << 16);
                d0 = fma(static_cast<double>(__uint_as_float(field_top<S, W>(w, i))),
                         static_cast<double>(__uint_as_float(vb)), d0);
              }
            }
          }
          continue;
        }
        if constexpr (kE2m3) {
          // products of two f16 values into FP32, exactly (e2m3_codec::fma2):
          // c0 takes the even codes, c1 the odd ones
#pragma unroll
          for (int q = 0; q < UV * GROUP / 4; ++q) {
            const int j = (v * UV * GROUP) / 2 + 2 * q;
            uint32_t lo, hi;
            Codec::to_f16x2x2(Codec::bytes4(w, q, smem), lo, hi);
            Codec::fma2(c0, c1, lo, vec2[j]);
            Codec::fma2(c0, c1, hi, vec2[j + 1]);
          }
          continue;
        }
#pragma unroll
        for (int i = 0; i < UV * GROUP; ++i) {
          const uint32_t m = field_top<S, W>(w, i);
          const int j = v * UV * GROUP + i;
          if constexpr (kPairs) {
            if (j & 1)
              c1 = fma_bf16<true>(m, vec2[j >> 1], c1);
            else
              c0 = fma_bf16<false>(m, vec2[j >> 1], c0);
          } else if (i & 1) {
            c1 = fmaf(__uint_as_float(m), vec[j], c1);
          } else {
            c0 = fmaf(__uint_as_float(m), vec[j], c0);
          }
        }
      }
      if constexpr (F64) {
        red[(k + h) * kThreads + threadIdx.x] = d0;
      } else if constexpr (kLns64) {
        red[(k + h) * kThreads + threadIdx.x] = d0 + d1;
      } else {
        red[(k + h) * kThreads + threadIdx.x] =
            static_cast<double>(c0) + static_cast<double>(c1);
      }
    }
    // every thread is done with these stages, and their rows of red are
    // complete, before the stages are refilled or the group reduced
    if (__syncthreads_or(ok ? 0 : 1)) {
      failed = true;
      break;
    }
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (uint32_t h = 0; h < n; ++h) {
        uint32_t st = stage + h;
        if (st >= static_cast<uint32_t>(STAGES)) st -= STAGES;
        if (t + h + STAGES < tiles) issue(t + h + STAGES, st);
      }
    }
    stage += n;
    if (stage >= static_cast<uint32_t>(STAGES)) {
      stage -= STAGES;
      phase ^= 1u;
    }
    k += n;
    if (k == static_cast<uint32_t>(kRows) || t + n == tiles) {
      // one warp per row of the group: lane l adds partials l, l + 32, ...
      // (conflict-free), then the warp's fixed tree
      const uint32_t row = threadIdx.x >> 5, lane = threadIdx.x & 31;
      if (row < k) {
        const double *p = red + row * kThreads + lane;
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < kThreads / 32; ++j) s += p[32 * j];
        s = warp_sum(s);
        if (lane == 0) gemv_publish(g, first_row + done + row, s);
      }
      done += k;
      k = 0;
      __syncthreads();  // red is read before the next group writes it
    }
  }
  if (failed) {
    // Let the copies still in flight land, then give every unfinished row of
    // this block a NaN partial.
    if (threadIdx.x == 0) {
      const uint32_t t0 = done + k;
      for (uint32_t j = t0; j < tiles && j < t0 + STAGES; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1u);
      atomicOr(g.status, static_cast<unsigned int>(AUT_STATUS_WAIT_TIMEOUT));
    }
    __syncthreads();
    for (uint32_t r = done + threadIdx.x; r < tiles; r += kThreads)
      gemv_publish(g, first_row + r, __longlong_as_double(0x7ff8000000000000ll));
  }
}

} // namespace aut::dev

// ---------------------------------------------------------------------------
// Host-side dispatch.
// ---------------------------------------------------------------------------
namespace aut::lib {
namespace {

using kernel_fn = void (*)(aut::dev::dot_params);

struct kernel_entry {
  kernel_fn fn = nullptr;
  int smem = 0;
  int stride = 0;       // bits per stored slot
  int table_kind = 0;   // 0 none, 1/2 full f32/f64, 3/4 frac f32/f64, 5/6 product f32/f64,
                        // 7 full FP64 high words
  uint64_t tile_values = 0;  // codes per block-tile of the vector path
  int blocks_per_sm = 0;
  int runtime = 0;      // rt_codec: dot_params::rt carries the format
  kernel_fn batch_fn = nullptr;  // TMA: the short-ring kernel for batches
  int batch_smem = 0;
  int threads = aut::dev::kThreads;  // per block
};

template <class Codec, class Acc>
void set_tma_kernels(kernel_entry &e) {
  using shape = aut::dev::tma_shape_of<Codec, Acc>;
  e.fn = aut::dev::dot_tma_kernel<Codec, Acc>;
  e.smem = Codec::kTableBytes + shape::STAGES * 2 * shape::TILE_BYTES;
  e.tile_values = shape::TILE_VALUES;
  e.threads = shape::NT;
  if constexpr (aut::dev::has_short_ring<Codec, Acc>) {
    using batch_shape = aut::dev::tma_shape_of<Codec, Acc, true>;
    static_assert(batch_shape::TILE_VALUES == shape::TILE_VALUES, "same tiles");
    e.batch_fn = aut::dev::dot_tma_kernel<Codec, Acc, true>;
    e.batch_smem = Codec::kTableBytes + batch_shape::STAGES * 2 * batch_shape::TILE_BYTES;
  }
}

template <class Codec, class Acc>
kernel_entry make_entry(int strategy, int table_kind) {
  kernel_entry e;
  e.stride = Codec::kS;
  e.table_kind = table_kind;
  if (strategy == AUT_STRATEGY_TMA) {
    set_tma_kernels<Codec, Acc>(e);
  } else {
    e.fn = aut::dev::dot_ldg_kernel<Codec, Acc>;
    e.smem = Codec::kTableBytes;
    e.tile_values = static_cast<uint64_t>(aut::dev::packet_shape<Codec::kS>::P) *
                    aut::dev::kThreads * Codec::kU;
  }
  return e;
}

// TMA-only entry (rt_codec: packets of up to 17 vectors would not fit an
// LDG thread's registers).
template <class Codec, class Acc>
kernel_entry make_tma_entry() {
  kernel_entry e;
  e.stride = Codec::kS;
  set_tma_kernels<Codec, Acc>(e);
  e.runtime = 1;
  return e;
}

template <int S, bool kDense>
kernel_entry rt_entry(int32_t accum) {
  using namespace aut::dev;
  return accum == AUT_ACCUM_FP32 ? make_tma_entry<rt_codec<S, float, kDense>, acc_f32>()
                                 : make_tma_entry<rt_codec<S, double, kDense>, acc_f64>();
}

// Bit formats without a dedicated codec: the rt_codec TMA kernel of their
// slot width (the registry's widths; padded containers of 8, 16, 32 bits).
kernel_entry rt_lookup(int32_t format, int32_t layout, int32_t accum) {
  const format_desc *f = find_format(format);
  if (f == nullptr || !generic_dot_ok(*f, accum)) return {};
  if (f->family != AUT_FAMILY_BINARY && f->family != AUT_FAMILY_FP64_PREFIX) return {};
  if (layout == AUT_LAYOUT_PADDED) {
    switch (container_bits(*f)) {
    case 8: return rt_entry<8, false>(accum);
    case 16: return rt_entry<16, false>(accum);
    case 32: return rt_entry<32, false>(accum);
    default: return {};
    }
  }
  switch (f->total_bits) {
  case 2: return rt_entry<2, true>(accum);
  case 3: return rt_entry<3, true>(accum);
  case 4: return rt_entry<4, true>(accum);
  case 5: return rt_entry<5, true>(accum);
  case 6: return rt_entry<6, true>(accum);
  case 7: return rt_entry<7, true>(accum);
  case 8: return rt_entry<8, true>(accum);
  case 9: return rt_entry<9, true>(accum);
  case 10: return rt_entry<10, true>(accum);
  case 12: return rt_entry<12, true>(accum);
  case 14: return rt_entry<14, true>(accum);
  case 16: return rt_entry<16, true>(accum);
  case 17: return rt_entry<17, true>(accum);
  case 20: return rt_entry<20, true>(accum);
  case 24: return rt_entry<24, true>(accum);
  case 28: return rt_entry<28, true>(accum);
  case 32: return rt_entry<32, true>(accum);
  default: return {};
  }
}

// Runtime decode parameters of a bit format for rt_codec.
aut::dev::rt_params rt_params_for(const format_desc &f, int32_t accum) {
  aut::dev::rt_params r{};
  const int E = f.family == AUT_FAMILY_FP64_PREFIX ? 11 : f.exponent_bits;
  const bool finite = f.family == AUT_FAMILY_BINARY && f.finite != 0;
  const int bias = E == 0 ? 1 : (1 << (E - 1)) - 1;  // fixed point: value = m 2^-M
  r.bits = static_cast<uint32_t>(f.total_bits);
  r.exponent = static_cast<uint32_t>(E);
  const int target_e = accum == AUT_ACCUM_FP32 ? 8 : 11;
  r.special_from = (!finite && E > 0 && E < target_e)
                       ? ((1u << E) - 1u) << (31 - E)
                       : 0u;
  r.scale32 = std::ldexp(1.0f, 127 - bias);
  r.scale64 = std::ldexp(1.0, 1023 - bias);
  return r;
}

template <int S>
kernel_entry lut_entry(int32_t accum, int strategy) {
  using namespace aut::dev;
  kernel_entry e = accum == AUT_ACCUM_FP32
                       ? make_entry<lut_codec<S, float>, acc_f32>(strategy, 1)
                       : make_entry<lut_codec<S, double>, acc_f64>(strategy, 2);
  e.runtime = 1;  // prepare() reads the code width from dot_params::rt
  return e;
}

// Codes of at most 8 bits: the table-decoded kernels of their slot width.
kernel_entry lut_lookup(const format_desc &f, int32_t layout, int32_t accum, int strategy) {
  if (strategy != AUT_STRATEGY_LDG && strategy != AUT_STRATEGY_TMA) return {};
  switch (layout == AUT_LAYOUT_PADDED ? 8 : f.total_bits) {
  case 2: return lut_entry<2>(accum, strategy);
  case 3: return lut_entry<3>(accum, strategy);
  case 4: return lut_entry<4>(accum, strategy);
  case 5: return lut_entry<5>(accum, strategy);
  case 6: return lut_entry<6>(accum, strategy);
  case 7: return lut_entry<7>(accum, strategy);
  case 8: return lut_entry<8>(accum, strategy);
  default: return {};
  }
}

template <class Codec>
kernel_entry pick(int strategy, int accum, int table_kind) {
  return accum == AUT_ACCUM_FP32
             ? make_entry<Codec, aut::dev::acc_f32>(strategy, table_kind)
             : make_entry<Codec, aut::dev::acc_f64>(strategy, table_kind);
}

// table kinds 8-11: prefix (FP32 bits / FP64 high word), subnormal (same)
template <int S, int W, bool kPrefix>
kernel_entry part_pick(int strategy, int accum) {
  using namespace aut::dev;
  const int kind = (kPrefix ? 8 : 10) + (accum == AUT_ACCUM_FP32 ? 0 : 1);
  return accum == AUT_ACCUM_FP32
             ? make_entry<part_lut_codec<S, W, float, kPrefix>, acc_f32>(strategy, kind)
             : make_entry<part_lut_codec<S, W, double, kPrefix>, acc_f64>(strategy, kind);
}

template <int S, int W>
kernel_entry wide_pick(int strategy, int accum) {
  using namespace aut::dev;
  return accum == AUT_ACCUM_FP32 ? make_entry<wide_lut_codec<S, W, float>, acc_f32>(strategy, 1)
                                 : make_entry<wide_lut_codec<S, W, double>, acc_f64>(strategy, 7);
}

// The strategy AUTO resolves to per format and accumulator, chosen from
// CUDA-event timings of both strategies at N = 2^27 on B200 (packed GB/s,
// LDG / TMA, FP32 accumulator):
//   fp32 7037 / 6776     fp64  7185 / 7312     e2m3 5414 / 5422
//   e8m0 3886 / 6122     e8m1 5272 / 6333     e8m3 5995 / 6474
//   e8m5 5366 / 6525     bf16 6651 / 6545     e8m15 6532 / 6874
//   lns8_r3 4756 / 5567 (FP64 accumulator: 3677 / 2444)
//   lns16_r11 (fused multiply) 4321 / 4540 (FP64: 3710 / 3631)
// Packets of several 16-byte vectors (S = 6, 9, 10, 14, 24) load strided per
// thread and stall on the LSU queue; the bulk-copy ring removes that.  lns8
// with FP64 has a 64 KiB table, and beside the ring only one block fits an SM.
int auto_strategy(int32_t format, int32_t layout, int32_t accum) {
  (void)layout;
  switch (format) {
  case AUT_FMT_LNS8_R3:
  case AUT_FMT_LNS16_R11:
    return accum == AUT_ACCUM_FP32 ? AUT_STRATEGY_TMA : AUT_STRATEGY_LDG;
  default: return AUT_STRATEGY_TMA;
  }
}

template <int B, class Dec>
kernel_entry coop_entry(int32_t accum) {
  using namespace aut::dev;
  kernel_entry e;
  e.stride = B;
  e.fn = accum == AUT_ACCUM_FP32 ? dot_coop_kernel<B, Dec, acc_f32> : dot_coop_kernel<B, Dec, acc_f64>;
  e.smem = 0;
  using geo = aut::bitwidth::cooperative_geometry<B>;
  e.tile_values = static_cast<uint64_t>(kThreads / geo::consumers) * geo::values;
  return e;
}

// The cooperative shuffle loader: dense E8 and e2m3 streams, decoded by
// bit moves / the hardware conversion.
kernel_entry coop_lookup(int32_t format, int32_t layout, int32_t accum) {
  using namespace aut::dev;
  if (layout != AUT_LAYOUT_DENSE) return {};
  switch (format) {
  case AUT_FMT_E2M3: return coop_entry<6, coop_e2m3>(accum);
  case AUT_FMT_E8M0: return coop_entry<9, coop_e8<9>>(accum);
  case AUT_FMT_E8M1: return coop_entry<10, coop_e8<10>>(accum);
  case AUT_FMT_E8M3: return coop_entry<12, coop_e8<12>>(accum);
  case AUT_FMT_E8M5: return coop_entry<14, coop_e8<14>>(accum);
  case AUT_FMT_BF16_E8M7: return coop_entry<16, coop_e8<16>>(accum);
  case AUT_FMT_E8M15: return coop_entry<24, coop_e8<24>>(accum);
  default: return {};
  }
}

// Decoders per format (the reference's decoder_kind axis): the E8 formats,
// raw storage and e2m3 decode DIRECT (bit moves / hardware conversion);
// lns8_r3 has FULL_LUT and FUSED_SUM_LUT; lns16_r11 has FULL_LUT (FP32
// only: the table is 128 KiB of FP32), FRACTION_LUT and FRACTION_LUT_FUSED;
// both have EX2_APPROX.  AUTO picks the fastest measured exact one.
kernel_entry lookup(int32_t format, int32_t layout, int32_t accum, int strategy,
                    int decoder = AUT_DECODER_AUTO) {
  using namespace aut::dev;
  if (format > AUT_FMT_LNS16_R11) {
    const format_desc *f = find_format(format);
    if (f == nullptr || !generic_dot_ok(*f, accum)) return {};
    if (f->total_bits <= 8 && (decoder == AUT_DECODER_AUTO || decoder == AUT_DECODER_FULL_LUT))
      return lut_lookup(*f, layout, accum, strategy == AUT_STRATEGY_AUTO ? AUT_STRATEGY_TMA
                                                                         : strategy);
    if (f->family == AUT_FAMILY_LNS) return {};
    if (strategy != AUT_STRATEGY_AUTO && strategy != AUT_STRATEGY_TMA) return {};
    if (decoder != AUT_DECODER_AUTO && decoder != AUT_DECODER_DIRECT) return {};
    return rt_lookup(format, layout, accum);
  }
  if (strategy == AUT_STRATEGY_AUTO) strategy = auto_strategy(format, layout, accum);
  const bool dense = layout == AUT_LAYOUT_DENSE;
  const int s = strategy;
  const bool lns = format == AUT_FMT_LNS8_R3 || format == AUT_FMT_LNS16_R11;
  if (decoder == AUT_DECODER_FULL_LUT && !lns) {
    // the full-table decoder of the bit formats (decode_with_table)
    switch (format) {
    case AUT_FMT_E2M3: return lut_lookup(*find_format(format), layout, accum, s);
    case AUT_FMT_E8M0: return dense ? wide_pick<9, 9>(s, accum) : wide_pick<16, 9>(s, accum);
    case AUT_FMT_E8M1: return dense ? wide_pick<10, 10>(s, accum) : wide_pick<16, 10>(s, accum);
    case AUT_FMT_E8M3: return dense ? wide_pick<12, 12>(s, accum) : wide_pick<16, 12>(s, accum);
    case AUT_FMT_E8M5: return dense ? wide_pick<14, 14>(s, accum) : wide_pick<16, 14>(s, accum);
    default: return {};
    }
  }
  if (decoder == AUT_DECODER_PREFIX_LUT || decoder == AUT_DECODER_SUBNORMAL_LUT) {
    // the partial-table decoders of the E8 codes with 1 to 5 mantissa bits
    const bool pre = decoder == AUT_DECODER_PREFIX_LUT;
    switch (format) {
    case AUT_FMT_E8M1:
      return dense ? (pre ? part_pick<10, 10, true>(s, accum) : part_pick<10, 10, false>(s, accum))
                   : (pre ? part_pick<16, 10, true>(s, accum) : part_pick<16, 10, false>(s, accum));
    case AUT_FMT_E8M3:
      return dense ? (pre ? part_pick<12, 12, true>(s, accum) : part_pick<12, 12, false>(s, accum))
                   : (pre ? part_pick<16, 12, true>(s, accum) : part_pick<16, 12, false>(s, accum));
    case AUT_FMT_E8M5:
      return dense ? (pre ? part_pick<14, 14, true>(s, accum) : part_pick<14, 14, false>(s, accum))
                   : (pre ? part_pick<16, 14, true>(s, accum) : part_pick<16, 14, false>(s, accum));
    default: return {};
    }
  }
  if (decoder != AUT_DECODER_AUTO) {
    if (!lns && decoder != AUT_DECODER_DIRECT) return {};
    if (lns && decoder == AUT_DECODER_DIRECT) return {};
    if (format == AUT_FMT_LNS8_R3 && decoder != AUT_DECODER_FULL_LUT &&
        decoder != AUT_DECODER_FUSED_SUM_LUT && decoder != AUT_DECODER_EX2_APPROX)
      return {};
    if (format == AUT_FMT_LNS16_R11 && decoder == AUT_DECODER_FUSED_SUM_LUT) return {};
  }
  if (decoder == AUT_DECODER_EX2_APPROX) {
    // never chosen by AUTO: approximate
    if (format == AUT_FMT_LNS8_R3)
      return accum == AUT_ACCUM_FP32 ? make_entry<lns_ex2_codec<8, float>, acc_f32>(s, 0)
                                     : make_entry<lns_ex2_codec<8, double>, acc_f64>(s, 0);
    return accum == AUT_ACCUM_FP32 ? make_entry<lns_ex2_codec<16, float>, acc_f32>(s, 0)
                                   : make_entry<lns_ex2_codec<16, double>, acc_f64>(s, 0);
  }
  if (format == AUT_FMT_LNS16_R11) {
    const bool f32 = accum == AUT_ACCUM_FP32;
    switch (decoder) {
    case AUT_DECODER_FULL_LUT:
      if (!f32) return {};
      return make_entry<lns16_full_codec, acc_f32>(s, 1);
    case AUT_DECODER_FRACTION_LUT:
      return f32 ? make_entry<lns16_codec<float>, acc_f32>(s, 3)
                 : make_entry<lns16_codec<double>, acc_f64>(s, 4);
    default:  // AUTO, FRACTION_LUT_FUSED
      return f32 ? make_entry<lns16_fused_codec<float>, acc_f32>(s, 3)
                 : make_entry<lns16_fused_codec<double>, acc_f64>(s, 4);
    }
  }
  switch (format) {
  // raw storage: accumulation compensated per product (acc_f32c, acc_f64c)
  case AUT_FMT_FP32:
    return accum == AUT_ACCUM_FP32 ? make_entry<e8_codec<32, 32>, acc_f32c>(s, 0)
                                   : make_entry<e8_codec<32, 32>, acc_f64c>(s, 0);
  case AUT_FMT_FP64:
    if (accum != AUT_ACCUM_FP64) return {};
    return make_entry<f64_codec, acc_f64c>(s, 0);
  case AUT_FMT_E2M3:
    return dense ? pick<e2m3_codec<6>>(s, accum, 0) : pick<e2m3_codec<8>>(s, accum, 0);
  case AUT_FMT_E8M0:
    return dense ? pick<e8_codec<9, 9>>(s, accum, 0) : pick<e8_codec<16, 9>>(s, accum, 0);
  case AUT_FMT_E8M1:
    return dense ? pick<e8_codec<10, 10>>(s, accum, 0) : pick<e8_codec<16, 10>>(s, accum, 0);
  case AUT_FMT_E8M3:
    return dense ? pick<e8_codec<12, 12>>(s, accum, 0) : pick<e8_codec<16, 12>>(s, accum, 0);
  case AUT_FMT_E8M5:
    return dense ? pick<e8_codec<14, 14>>(s, accum, 0) : pick<e8_codec<16, 14>>(s, accum, 0);
  case AUT_FMT_BF16_E8M7: return pick<e8_codec<16, 16>>(s, accum, 0);
  case AUT_FMT_E8M15:
    // 16-bit significands: an FP32 product rounds, so both accumulators
    // widen the operands and sum the exact products in FP64 (FP32 chains:
    // normalised error 7.7e-12 at 2^27; FP64: 2.8e-21, and the bulk-copy
    // kernel stays HBM-bound either way, 6644 GB/s against 6802 for FP32)
    return dense ? make_entry<e8_codec<24, 24>, acc_f64>(s, 0)
                 : make_entry<e8_codec<32, 24>, acc_f64>(s, 0);
  case AUT_FMT_LNS8_R3:
    // AUTO: the full table for FP32 (N = 2^28: 5863 GB/s against 3679 for
    // the fused sum), the fused sum for FP64 (4093 against 3712; the same
    // normalised error on the cancellation pair, 4.8e-20)
    if (decoder == AUT_DECODER_FUSED_SUM_LUT ||
        (decoder == AUT_DECODER_AUTO && accum != AUT_ACCUM_FP32))
      return accum == AUT_ACCUM_FP32 ? make_entry<lns8_fused_codec<float>, acc_f32>(s, 5)
                                     : make_entry<lns8_fused_codec<double>, acc_f64>(s, 6);
    return accum == AUT_ACCUM_FP32 ? make_entry<lns8_codec<float>, acc_f32>(s, 1)
                                   : make_entry<lns8_codec<double>, acc_f64>(s, 2);
  default: return {};
  }
}

// Occupancy of each kernel, cached per function pointer.
struct occupancy_cache {
  std::mutex mutex;
  kernel_fn fns[256] = {};
  int blocks[256] = {};
  int count = 0;
};
occupancy_cache &cache() {
  static occupancy_cache c;
  return c;
}

aut_status blocks_per_sm(kernel_entry &e) {
  auto &c = cache();
  std::lock_guard<std::mutex> lock(c.mutex);
  for (int k = 0; k < c.count; ++k)
    if (c.fns[k] == e.fn) {
      e.blocks_per_sm = c.blocks[k];
      return AUT_OK;
    }
  // Dynamic shared memory plus the kernel's static barriers may pass the
  // 48 KB default even when the dynamic part alone does not.
  if (e.smem > 0)
    AUT_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void *>(e.fn),
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      e.smem));
  int b = 0;
  AUT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &b, reinterpret_cast<const void *>(e.fn), e.threads, e.smem));
  if (b < 1) return fail(AUT_ERR_UNSUPPORTED, "kernel does not fit on an SM");
  if (c.count < 256) {
    c.fns[c.count] = e.fn;
    c.blocks[c.count] = b;
    ++c.count;
  }
  e.blocks_per_sm = b;
  return AUT_OK;
}

} // namespace

aut_status generic_dot_launch(aut_workspace *ws, const format_desc &f, int32_t format,
                              int32_t layout, int32_t accum, const void *x, const void *y,
                              uint64_t n, uint32_t batch, const batch_layout &bl,
                              double *results, cudaStream_t stream, double *partials,
                              unsigned int *tickets, int max_blocks_total);

// Formats with fused kernels (ids 0..10) never fall back to the generic DOT;
// every other registered format runs it when it decodes exactly.
static bool has_fused_kernel(int32_t format, int32_t layout, int32_t accum) {
  return lookup(format, layout, accum, AUT_STRATEGY_AUTO).fn != nullptr;
}

static bool generic_format(int32_t format) {
  return format > AUT_FMT_LNS16_R11 && find_format(format) != nullptr;
}

int32_t dot_supported(int32_t format, int32_t layout, int32_t accum) {
  if (layout != AUT_LAYOUT_DENSE && layout != AUT_LAYOUT_PADDED) return 0;
  if (accum != AUT_ACCUM_FP32 && accum != AUT_ACCUM_FP64) return 0;
  if (has_fused_kernel(format, layout, accum)) return 1;
  return generic_format(format) && generic_dot_ok(*find_format(format), accum) ? 1 : 0;
}

// The vector paths need 16-byte aligned streams for every pair of the batch.
static bool vector_path_ok(const void *x, const void *y, uint32_t batch, const batch_layout &bl) {
  const bool bases = reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(y) % 16 == 0;
  if (batch <= 1) return bases;
  return bases && bl.x_stride % 16 == 0 && bl.y_stride % 16 == 0 &&
         bl.x_index_stride == 0 && bl.y_index_stride == 0;
}

// Kernel parameters for the pairs b0, b0 + 1, ... of a batch.
static aut::dev::dot_params params_for(const void *x, const void *y, uint64_t n, uint32_t b0,
                                const batch_layout &bl, bool aligned) {
  aut::dev::dot_params p{};
  p.x = static_cast<const unsigned char *>(x) + static_cast<uint64_t>(b0) * bl.x_stride;
  p.y = static_cast<const unsigned char *>(y) + static_cast<uint64_t>(b0) * bl.y_stride;
  p.x_stride = bl.x_stride;
  p.y_stride = bl.y_stride;
  p.x_first = static_cast<uint64_t>(b0) * bl.x_index_stride;
  p.y_first = static_cast<uint64_t>(b0) * bl.y_index_stride;
  p.x_index_stride = bl.x_index_stride;
  p.y_index_stride = bl.y_index_stride;
  p.n = n;
  p.vector_ok = aligned ? 1 : 0;
  p.wait_cycles = aut::kWaitCyclesDefault;
  p.stall_tile = ~0ull;
  return p;
}

// Launches a DOT kernel with programmatic stream serialisation: it may be
// scheduled while the kernel before it on the stream finishes (the kernels
// call pdl_wait before their first global access, so they still see all
// of that kernel's writes), which hides the launch gap between consecutive
// DOTs.
template <class... P, class... A>
static cudaError_t launch_pdl(void (*fn)(P...), dim3 grid, unsigned threads, size_t smem,
                              cudaStream_t stream, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, args...);
}

static cudaError_t launch_dependent(const kernel_entry &e, dim3 grid, cudaStream_t stream,
                                    const aut::dev::dot_params &p) {
  return launch_pdl(e.fn, grid, static_cast<unsigned>(e.threads),
                    static_cast<size_t>(e.smem), stream, p);
}

aut_status dot_launch(aut_workspace *ws, int32_t format, int32_t layout,
                      int32_t accum, int32_t strategy, int32_t decoder,
                      const void *x, const void *y, uint64_t n, uint32_t batch,
                      const batch_layout &bl, double *results, void *stream,
                      double *partials, unsigned int *tickets,
                      unsigned int *status, int max_blocks_total) {
  // SCALAR runs the LDG kernel with the vector path switched off, so every
  // code goes through the per-value load and decode.
  const bool scalar_only = strategy == AUT_STRATEGY_SCALAR;
  if (generic_format(format) &&
      ((find_format(format)->family == AUT_FAMILY_LNS && find_format(format)->total_bits > 8) ||
       scalar_only)) {
    // the generic DOT reads one value per thread: LNS formats other than
    // lns8_r3 / lns16_r11 (decoder AUTO or FULL_LUT: the host-built table),
    // and the per-value (SCALAR) strategy of the other bit formats
    const format_desc &f = *find_format(format);
    const int direct = f.family == AUT_FAMILY_LNS ? AUT_DECODER_FULL_LUT : AUT_DECODER_DIRECT;
    if ((strategy != AUT_STRATEGY_AUTO && !scalar_only) ||
        (decoder != AUT_DECODER_AUTO && decoder != direct))
      return fail(AUT_ERR_UNSUPPORTED,
                  "this format takes strategy AUTO/SCALAR and its full-table decoder");
    return generic_dot_launch(ws, f, format, layout, accum, x, y, n, batch, bl, results,
                              static_cast<cudaStream_t>(stream), partials, tickets,
                              max_blocks_total);
  }
  const bool coop = strategy == AUT_STRATEGY_COOPERATIVE;
  if (coop && decoder != AUT_DECODER_AUTO && decoder != AUT_DECODER_DIRECT)
    return fail(AUT_ERR_UNSUPPORTED, "the cooperative loader decodes by bit moves (DIRECT)");
  kernel_entry e = coop ? coop_lookup(format, layout, accum)
                        : lookup(format, layout, accum,
                                 scalar_only ? AUT_STRATEGY_LDG : strategy, decoder);
  if (e.fn == nullptr)
    return fail(AUT_ERR_UNSUPPORTED,
                "no fused DOT kernel for this format/layout/accumulator/decoder");
  if (batch > 1 && e.batch_fn != nullptr) {
    e.fn = e.batch_fn;
    e.smem = e.batch_smem;
  }
  aut_status st = blocks_per_sm(e);
  if (st != AUT_OK) return st;

  const void *table = nullptr;
  if (e.table_kind != 0) {
    const code_tables *t = nullptr;
    st = code_tables_for(ws, format, &t);
    if (st != AUT_OK) return st;
    if ((e.table_kind == 3 && !t->split_f32) || (e.table_kind == 4 && !t->split_f64))
      return fail(AUT_ERR_UNSUPPORTED,
                  "this host's exp2/exp2f break the split LNS decode identity that the "
                  "fraction-table kernels rely on");
    if ((e.table_kind == 7 && t->full_hi == nullptr) ||
        ((e.table_kind == 5 || e.table_kind == 6) && t->prod_f32 == nullptr) ||
        (e.table_kind >= 8 && t->part == nullptr))
      return fail(AUT_ERR_UNSUPPORTED, "no decode table of this kind for this format");
    const uint32_t sub_entries = t->part_sub_entries;
    table = e.table_kind >= 8
                ? static_cast<const void *>(
                      t->part + (e.table_kind == 8   ? 0
                                 : e.table_kind == 9 ? 512
                                 : e.table_kind == 10 ? 1024
                                                      : 1024 + sub_entries))
            : e.table_kind == 1 ? static_cast<const void *>(t->full_f32)
            : e.table_kind == 2 ? static_cast<const void *>(t->full_f64)
            : e.table_kind == 5 ? static_cast<const void *>(t->prod_f32)
            : e.table_kind == 6 ? static_cast<const void *>(t->prod_f64)
            : e.table_kind == 7 ? static_cast<const void *>(t->full_hi)
            : e.table_kind == 3 ? static_cast<const void *>(t->frac_f32)
                                : static_cast<const void *>(t->frac_f64);
  }

  const bool aligned = !scalar_only && vector_path_ok(x, y, batch, bl);
  const int cap = ws->sm_count * e.blocks_per_sm;
  uint64_t wanted = aligned ? (n / e.tile_values) : 0;
  if (wanted == 0) wanted = (n + aut::dev::kThreads - 1) / aut::dev::kThreads;
  if (wanted == 0) wanted = 1;
  for (uint32_t b0 = 0; b0 < batch; b0 += kMaxBatchPerLaunch) {
    const uint32_t nb = batch - b0 < static_cast<uint32_t>(kMaxBatchPerLaunch)
                            ? batch - b0
                            : static_cast<uint32_t>(kMaxBatchPerLaunch);
    int per_pair = static_cast<int>((cap + nb - 1) / nb);
    if (per_pair < 1) per_pair = 1;
    if (static_cast<uint64_t>(per_pair) > wanted) per_pair = static_cast<int>(wanted);
    if (per_pair > max_blocks_total) per_pair = max_blocks_total;
    aut::dev::dot_params p = params_for(x, y, n, b0, bl, aligned);
    if (e.runtime) p.rt = rt_params_for(*find_format(format), accum);
    p.table = table;
    p.partials = partials;
    p.tickets = tickets;
    p.results = results + b0;
    p.status = status;
    p.wait_cycles = ws->wait_cycles;
    p.stall_tile = ws->stall_tile;
    p.claims = ws->claims;
    dim3 grid(static_cast<unsigned>(per_pair), nb);
    AUT_CUDA_TRY(launch_dependent(e, grid, static_cast<cudaStream_t>(stream), p));
  }
  return AUT_OK;
}

// ---- GEMV with the vector decoded once per block ----------------------------
struct gemv_entry {
  void (*fn)(aut::dev::gemv_params) = nullptr;
  int smem = 0;
  uint64_t tile_values = 0;
  uint64_t tile_bytes = 0;
  int group_rows = 0;
};

template <class Codec, bool F64 = false>
gemv_entry make_gemv_entry() {
  using shape = aut::dev::gemv_shape<Codec>;
  gemv_entry e;
  e.fn = aut::dev::gemv_tma_kernel<Codec, F64>;
  e.smem = Codec::kTableBytes + shape::STAGES * shape::TILE_BYTES +
           aut::dev::gemv_rows<Codec>() * aut::dev::kThreads * 8;
  e.group_rows = aut::dev::gemv_rows<Codec>();
  e.tile_values = shape::TILE_VALUES;
  e.tile_bytes = shape::TILE_BYTES;
  return e;
}

// The vector-once kernels: FP32 rows of the E8 codes, raw FP32 and
// lns8_r3 (its per-lane table); FP64 rows of the E8 codes, raw FP32 and
// lns8_r3 (the FP64 table); e2m3 rows (exact) for both.
static gemv_entry gemv_lookup(int32_t format, int32_t layout, int32_t accum) {
  using namespace aut::dev;
  const bool dense = layout == AUT_LAYOUT_DENSE;
  if (accum == AUT_ACCUM_FP64) {
    switch (format) {
    case AUT_FMT_E8M0:
      return dense ? make_gemv_entry<e8_codec<9, 9>, true>() : make_gemv_entry<e8_codec<16, 9>, true>();
    case AUT_FMT_E8M1:
      return dense ? make_gemv_entry<e8_codec<10, 10>, true>() : make_gemv_entry<e8_codec<16, 10>, true>();
    case AUT_FMT_E8M3:
      return dense ? make_gemv_entry<e8_codec<12, 12>, true>() : make_gemv_entry<e8_codec<16, 12>, true>();
    case AUT_FMT_E8M5:
      return dense ? make_gemv_entry<e8_codec<14, 14>, true>() : make_gemv_entry<e8_codec<16, 14>, true>();
    case AUT_FMT_BF16_E8M7: return make_gemv_entry<e8_codec<16, 16>, true>();
    case AUT_FMT_E8M15:
      return dense ? make_gemv_entry<e8_codec<24, 24>, true>() : make_gemv_entry<e8_codec<32, 24>, true>();
    case AUT_FMT_FP32: return make_gemv_entry<e8_codec<32, 32>, true>();
    case AUT_FMT_LNS8_R3: return make_gemv_entry<lns8_codec<double, 16>>();
    case AUT_FMT_E2M3: break;
    default: return {};
    }
  }
  switch (format) {
  case AUT_FMT_FP32: return make_gemv_entry<e8_codec<32, 32>>();
  case AUT_FMT_E8M0: return dense ? make_gemv_entry<e8_codec<9, 9>>() : make_gemv_entry<e8_codec<16, 9>>();
  case AUT_FMT_E8M1: return dense ? make_gemv_entry<e8_codec<10, 10>>() : make_gemv_entry<e8_codec<16, 10>>();
  case AUT_FMT_E8M3: return dense ? make_gemv_entry<e8_codec<12, 12>>() : make_gemv_entry<e8_codec<16, 12>>();
  case AUT_FMT_E8M5: return dense ? make_gemv_entry<e8_codec<14, 14>>() : make_gemv_entry<e8_codec<16, 14>>();
  case AUT_FMT_BF16_E8M7: return make_gemv_entry<e8_codec<16, 16>>();
  case AUT_FMT_E8M15: return dense ? make_gemv_entry<e8_codec<24, 24>>() : make_gemv_entry<e8_codec<32, 24>>();
  case AUT_FMT_E2M3: return dense ? make_gemv_entry<e2m3_codec<6>>() : make_gemv_entry<e2m3_codec<8>>();
  case AUT_FMT_LNS8_R3: return make_gemv_entry<lns8_codec<float>>();  // one code per byte
  default: return {};
  }
}

static aut_status gemv_blocks_per_sm(const gemv_entry &e, int *out) {
  static std::mutex mutex;
  static void (*fns[64])(aut::dev::gemv_params) = {};
  static int blocks[64] = {};
  static int count = 0;
  std::lock_guard<std::mutex> lock(mutex);
  for (int k = 0; k < count; ++k)
    if (fns[k] == e.fn) {
      *out = blocks[k];
      return AUT_OK;
    }
  AUT_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void *>(e.fn),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, e.smem));
  int b = 0;
  AUT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &b, reinterpret_cast<const void *>(e.fn), aut::dev::kThreads, e.smem));
  if (b < 1) return fail(AUT_ERR_UNSUPPORTED, "GEMV kernel does not fit on an SM");
  if (count < 64) {
    fns[count] = e.fn;
    blocks[count] = b;
    ++count;
  }
  *out = b;
  return AUT_OK;
}

// The GEMV path that decodes the vector once per block: FP32 accumulation
// of the E8 codes and raw FP32, either accumulator for e2m3 (exact), decoder
// AUTO/DIRECT, strategy AUTO/TMA, whole
// segments (columns a multiple of one tile) and 16-byte aligned operands.
// *handled is false when the call does not qualify; aut_gemv then runs the
// rows as a batch of DOTs.
aut_status gemv_launch(aut_workspace *ws, int32_t format, int32_t layout, int32_t accum,
                       int32_t strategy, int32_t decoder, const void *matrix,
                       const void *vector, uint64_t rows, uint64_t columns,
                       double *results, void *stream, bool *handled) {
  *handled = false;
  if (accum != AUT_ACCUM_FP32 && accum != AUT_ACCUM_FP64) return AUT_OK;
  if (strategy != AUT_STRATEGY_AUTO && strategy != AUT_STRATEGY_TMA) return AUT_OK;
  if (decoder != AUT_DECODER_AUTO && decoder != AUT_DECODER_DIRECT) return AUT_OK;
  const gemv_entry e = gemv_lookup(format, layout, accum);
  if (e.fn == nullptr || columns == 0 || rows == 0 || columns % e.tile_values != 0) return AUT_OK;
  if ((reinterpret_cast<uintptr_t>(matrix) | reinterpret_cast<uintptr_t>(vector)) & 15u)
    return AUT_OK;
  const uint64_t segments = columns / e.tile_values;
  if (segments > static_cast<uint64_t>(ws->max_blocks) || segments > 65535u) return AUT_OK;
  int per_sm = 0;
  aut_status st = gemv_blocks_per_sm(e, &per_sm);
  if (st != AUT_OK) return st;
  const void *table = nullptr;
  if (format == AUT_FMT_LNS8_R3) {
    const code_tables *t = nullptr;
    st = code_tables_for(ws, format, &t);
    if (st != AUT_OK) return st;
    table = accum == AUT_ACCUM_FP64 ? static_cast<const void *>(t->full_f64)
                                    : static_cast<const void *>(t->full_f32);
  }
  const uint64_t row_bytes = segments * e.tile_bytes;
  const uint64_t cap = static_cast<uint64_t>(ws->sm_count) * per_sm;
  const uint64_t group_rows = static_cast<uint64_t>(e.group_rows);
  for (uint64_t r0 = 0; r0 < rows; r0 += kMaxBatchPerLaunch) {
    const uint64_t rc = rows - r0 < static_cast<uint64_t>(kMaxBatchPerLaunch)
                            ? rows - r0
                            : static_cast<uint64_t>(kMaxBatchPerLaunch);
    // about one block per resident slot: each block takes an equal run of
    // row groups for its segment
    const uint64_t groups = (rc + group_rows - 1) / group_rows;
    uint64_t per_segment = cap / segments;
    if (per_segment < 1) per_segment = 1;
    const uint64_t groups_per_block = (groups + per_segment - 1) / per_segment;
    const uint64_t blocks_y = (groups + groups_per_block - 1) / groups_per_block;
    aut::dev::gemv_params g{};
    g.matrix = static_cast<const unsigned char *>(matrix) + r0 * row_bytes;
    g.vector = static_cast<const unsigned char *>(vector);
    g.row_bytes = row_bytes;
    g.rows = static_cast<uint32_t>(rc);
    g.groups_per_block = static_cast<uint32_t>(groups_per_block);
    g.partials = ws->partials;
    g.status = ws->tickets + kMaxBatchPerLaunch;
    g.table = table;
    dim3 grid(static_cast<unsigned>(segments), static_cast<unsigned>(blocks_y));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    AUT_CUDA_TRY(launch_pdl(e.fn, grid, aut::dev::kThreads, static_cast<size_t>(e.smem), s, g));
    constexpr uint64_t rows_per_block = aut::dev::kThreads / 32;
    AUT_CUDA_TRY(launch_pdl(aut::dev::gemv_rows_kernel,
                            dim3(static_cast<unsigned>((rc + rows_per_block - 1) / rows_per_block)),
                            aut::dev::kThreads, 0, s, static_cast<const double *>(ws->partials),
                            static_cast<uint32_t>(segments), static_cast<uint32_t>(rc),
                            results + r0));
  }
  *handled = true;
  return AUT_OK;
}

// Same launch as dot_launch for callers that bring their own reduction
// scratch and have no workspace: formats that need decode tables (LNS) are
// refused, the grid never uses more than `slots` partial slots in total, and
// nothing is allocated.  Once the format is accepted, `clear_bytes` bytes at
// `clear` (the counters) are zeroed on the stream before the launch; a
// refused call enqueues nothing.
aut_status dot_launch_scratch(int sm_count, int32_t format, int32_t layout,
                              int32_t accum, const void *x, const void *y,
                              uint64_t n, uint32_t batch, const batch_layout &bl,
                              double *results, void *stream, double *partials,
                              unsigned int *tickets, unsigned int *status,
                              int slots, void *clear, size_t clear_bytes) {
  kernel_entry e = lookup(format, layout, accum, AUT_STRATEGY_AUTO);
  if (e.fn == nullptr)
    return fail(AUT_ERR_UNSUPPORTED,
                "no fused DOT kernel for this format/layout/accumulator");
  if (e.table_kind != 0)
    return fail(AUT_ERR_UNSUPPORTED,
                "this format decodes through tables kept in a workspace; use aut_dot");
  if (batch > 1 && e.batch_fn != nullptr) {
    e.fn = e.batch_fn;
    e.smem = e.batch_smem;
  }
  aut_status st = blocks_per_sm(e);
  if (st != AUT_OK) return st;
  const bool aligned = vector_path_ok(x, y, batch, bl);
  uint64_t wanted = aligned ? (n / e.tile_values) : 0;
  if (wanted == 0) wanted = (n + aut::dev::kThreads - 1) / aut::dev::kThreads;
  if (wanted == 0) wanted = 1;
  int per_pair = (sm_count * e.blocks_per_sm + static_cast<int>(batch) - 1) /
                 static_cast<int>(batch);
  const int cap = slots / (2 * static_cast<int>(batch));  // two slots per block
  if (per_pair > cap) per_pair = cap;
  if (static_cast<uint64_t>(per_pair) > wanted) per_pair = static_cast<int>(wanted);
  if (per_pair < 1) per_pair = 1;
  aut::dev::dot_params p = params_for(x, y, n, 0, bl, aligned);
  if (e.runtime) p.rt = rt_params_for(*find_format(format), accum);
  p.table = nullptr;
  p.partials = partials;
  p.tickets = tickets;
  p.results = results;
  p.status = status;
  if (clear_bytes > 0)
    AUT_CUDA_TRY(cudaMemsetAsync(clear, 0, clear_bytes, static_cast<cudaStream_t>(stream)));
  dim3 grid(static_cast<unsigned>(per_pair), batch);
  e.fn<<<grid, e.threads, e.smem, static_cast<cudaStream_t>(stream)>>>(p);
  AUT_CUDA_TRY(cudaGetLastError());
  return AUT_OK;
}

} // namespace aut::lib

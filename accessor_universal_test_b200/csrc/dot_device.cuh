// dot_device.cuh -- building blocks of the decode-fused DOT kernels (sm_100a).
//
// Stream layout: a B-bit code stream (dense or padded) is read as "packets"
// of Q 16-byte vectors holding exactly P = 128*Q/S codes (S = bits per
// stored slot), so no code straddles a packet edge and every field offset is
// a compile-time constant once the packet loop is unrolled:
//   S =  6 -> Q=3, P=64     S =  9 -> Q=9, P=128    S = 10 -> Q=5, P=64
//   S = 12 -> Q=3, P=32     S = 14 -> Q=7, P=64     S = 16 -> Q=1, P=8
//   S = 24 -> Q=3, P=16     S =  8 -> Q=1, P=16     S = 32 -> Q=1, P=4
// Field extraction is one funnel shift (fields crossing a 32-bit word) or
// one shift, plus one mask.
#ifndef AUT_DOT_DEVICE_CUH_
#define AUT_DOT_DEVICE_CUH_

#include <cuda_runtime.h>

#include <cstdint>

namespace aut::dev {

constexpr int kThreads = 256;

constexpr int gcd_int(int a, int b) { return b == 0 ? a : gcd_int(b, a % b); }
template <int S> struct packet_shape {
  static constexpr int Q = S / gcd_int(S, 128);  // 16-byte vectors per packet
  static constexpr int P = 128 * Q / S;          // codes per packet
};

template <int W> __device__ __forceinline__ constexpr uint32_t top_mask() {
  return W >= 32 ? 0xffffffffu : ~((1u << (32 - W)) - 1u);
}
template <int W> __device__ __forceinline__ constexpr uint32_t low_mask() {
  return W >= 32 ? 0xffffffffu : ((1u << W) - 1u);
}

// Code v of a packet, moved to bits [32-W, 32) with zeros below.
template <int S, int W>
__device__ __forceinline__ uint32_t field_top(const uint32_t *w, int v) {
  const int b = v * S;
  const int i = b >> 5;
  const int sh = b & 31;
  if (sh + W <= 32) {
    if (sh + W == 32) return w[i] & top_mask<W>();
    const uint32_t t = w[i] << (32 - sh - W);
    return sh == 0 ? t : (t & top_mask<W>());
  }
  return __funnelshift_l(w[i], w[i + 1], 64 - sh - W) & top_mask<W>();
}

// Code v of a packet, moved to bits [0, W).
template <int S, int W>
__device__ __forceinline__ uint32_t field_low(const uint32_t *w, int v) {
  const int b = v * S;
  const int i = b >> 5;
  const int sh = b & 31;
  if (sh + W <= 32) {
    const uint32_t t = w[i] >> sh;
    return sh + W == 32 ? t : (t & low_mask<W>());
  }
  return __funnelshift_r(w[i], w[i + 1], sh) & low_mask<W>();
}

// Scalar code load for ragged tails: dense streams read two words (the
// stream's guard word keeps the second read in bounds); padded streams read
// one container.
template <int S, int W>
__device__ __forceinline__ uint32_t load_code(const unsigned char *base,
                                              uint64_t i) {
  if constexpr (S == 8) {
    return static_cast<uint32_t>(__ldg(base + i)) & low_mask<W>();
  } else if constexpr (S == 16) {
    return static_cast<uint32_t>(
               __ldg(reinterpret_cast<const unsigned short *>(base) + i)) &
           low_mask<W>();
  } else if constexpr (S == 32) {
    return __ldg(reinterpret_cast<const unsigned int *>(base) + i) &
           low_mask<W>();
  } else {
    const uint32_t *words = reinterpret_cast<const uint32_t *>(base);
    const uint64_t bit = i * static_cast<uint64_t>(S);
    const uint64_t wi = bit >> 5;
    const unsigned sh = static_cast<unsigned>(bit & 31u);
    const uint32_t lo = __ldg(words + wi);
    const uint32_t hi = (sh + W > 32) ? __ldg(words + wi + 1) : 0u;
    return __funnelshift_r(lo, hi, sh) & low_mask<W>();
  }
}

// ---- per-thread accumulators -------------------------------------------------
// FP32: four independent FMA chains, carried into FP64 at every flush().
struct acc_f32 {
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  double total = 0.0;
  __device__ __forceinline__ void mac(int slot, float x, float y) {
    a[slot & 3] = fmaf(x, y, a[slot & 3]);
  }
  __device__ __forceinline__ void mac_d(int slot, double x, double y) {
    total = fma(x, y, total);
  }
  __device__ __forceinline__ void add_exact(double v) { total += v; }
  __device__ __forceinline__ void flush() {
    total += static_cast<double>(a[0]) + static_cast<double>(a[1]);
    total += static_cast<double>(a[2]) + static_cast<double>(a[3]);
    a[0] = a[1] = a[2] = a[3] = 0.f;
  }
  __device__ __forceinline__ double value() {
    flush();
    return total;
  }
};

// FP64: two independent FMA chains of exactly widened operands.
struct acc_f64 {
  double a[2] = {0.0, 0.0};
  __device__ __forceinline__ void mac(int slot, float x, float y) {
    a[slot & 1] = fma(static_cast<double>(x), static_cast<double>(y), a[slot & 1]);
  }
  __device__ __forceinline__ void mac_d(int slot, double x, double y) {
    a[slot & 1] = fma(x, y, a[slot & 1]);
  }
  __device__ __forceinline__ void add_exact(double v) { a[0] += v; }
  __device__ __forceinline__ void flush() {}
  __device__ __forceinline__ double value() { return a[0] + a[1]; }
};

// ---- block / grid reduction (deterministic) ------------------------------------
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block; the result is valid in thread 0.
__device__ __forceinline__ double block_sum(double v, double *scratch) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double s = 0.0;
  if (warp == 0) {
    s = lane < (kThreads / 32) ? scratch[lane] : 0.0;
    s = warp_sum(s);
  }
  __syncthreads();
  return s;
}

// Single-pass grid reduction: every block publishes its partial, the last
// block to arrive (atomic ticket after a fence) sums the partials in block
// order and resets the ticket for the next launch.  No block waits on
// another, so the pattern cannot hang.
__device__ __forceinline__ void grid_finish(double block_partial,
                                            double *partials,
                                            unsigned int *ticket,
                                            double *result, double *scratch) {
  __shared__ bool last_block;
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = block_partial;
    __threadfence();
    const unsigned int arrived = atomicAdd(ticket, 1u);
    last_block = (arrived == gridDim.x - 1);
  }
  __syncthreads();
  if (!last_block) return;
  __threadfence();
  double s = 0.0;
  for (unsigned int b = threadIdx.x; b < gridDim.x; b += kThreads)
    s += __ldcg(partials + b);
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) {
    *result = s;
    *ticket = 0u;
  }
}

} // namespace aut::dev

#endif

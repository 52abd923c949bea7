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

// ---- double-double arithmetic ------------------------------------------------
// A sum carried as hi + lo with |lo| <= ulp(hi) / 2: the per-thread partials
// of the FP64 accumulators and every step of the block and grid reductions,
// so the reductions add no rounding of their own and the DOT is rounded
// once at the end.  Explicit _rn intrinsics keep the compiler from fusing
// the error terms into FMAs.
struct dd {
  double hi, lo;
};

// s + e = a + b exactly (Knuth's two-sum).
__device__ __forceinline__ void two_sum(double a, double b, double &s, double &e) {
  s = __dadd_rn(a, b);
  const double bb = __dsub_rn(s, a);
  e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
}

// An inf or NaN high part stays inf or NaN whatever is added to it, so its
// low part (then inf - inf or NaN) carries nothing and is dropped: inf and
// NaN pass through the reductions as a plain sum would give them.
__device__ __forceinline__ dd dd_add(dd a, dd b) {
  double s, e;
  two_sum(a.hi, b.hi, s, e);
  if (!isfinite(s)) return {s, 0.0};
  e = __dadd_rn(e, __dadd_rn(a.lo, b.lo));
  dd r;
  two_sum(s, e, r.hi, r.lo);
  if (!isfinite(r.hi)) r.lo = 0.0;  // s + e overflowed
  return r;
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
  __device__ __forceinline__ dd pair() { return {value(), 0.0}; }
};

// FP32, compensated (raw FP32 storage, HBM-bound with FP32 issue to
// spare): four FP32 chains, each product split into its rounded value and
// exact error by one FMA, added by an FP32 two-sum whose error joins a
// second FP32 chain; every flush carries hi + lo of each chain into an FP64
// double-double total.  All per-product arithmetic stays FP32; the error of
// a 32-product chain is then second order (~2^-48 relative), so the DOT is
// close to the exact sum rounded once.
struct acc_f32c {
  float hi[4] = {0.f, 0.f, 0.f, 0.f};
  float lo[4] = {0.f, 0.f, 0.f, 0.f};
  dd total = {0.0, 0.0};
  __device__ __forceinline__ void mac(int slot, float x, float y) {
    const int k = slot & 3;
    const float p = __fmul_rn(x, y);
    const float pe = __fmaf_rn(x, y, -p);
    const float s = __fadd_rn(hi[k], p);
    const float bb = __fsub_rn(s, hi[k]);
    const float e = __fadd_rn(__fsub_rn(hi[k], __fsub_rn(s, bb)), __fsub_rn(p, bb));
    hi[k] = s;
    lo[k] = __fadd_rn(lo[k], __fadd_rn(e, pe));
  }
  __device__ __forceinline__ void mac_d(int, double x, double y) {
    const double p = __dmul_rn(x, y);
    total = dd_add(total, {p, __fma_rn(x, y, -p)});
  }
  __device__ __forceinline__ void add_exact(double v) { total = dd_add(total, {v, 0.0}); }
  __device__ __forceinline__ void flush() {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const double h = static_cast<double>(hi[k]);
      total = dd_add(total, {h, isfinite(h) ? static_cast<double>(lo[k]) : 0.0});
      hi[k] = lo[k] = 0.f;
    }
  }
  __device__ __forceinline__ dd pair() {
    flush();
    return total;
  }
  __device__ __forceinline__ double value() {
    const dd r = pair();
    return r.hi + r.lo;
  }
};

// FP64: two independent FMA chains of exactly widened operands, joined
// without rounding for the double-double reductions.
struct acc_f64 {
  double a[2] = {0.0, 0.0};
  // Values 2k and 2k + 1 share a chain (chain k mod 2): on data whose signs
  // alternate from value to value (the LNS cancellation pair) each chain's
  // partial sum then cancels as it goes instead of growing with one sign,
  // which keeps its rounding errors small (lns8_r3, N = 2^28: normalised
  // error 6.6e-19 -> 4.8e-20).
  __device__ __forceinline__ void mac(int slot, float x, float y) {
    a[(slot >> 1) & 1] =
        fma(static_cast<double>(x), static_cast<double>(y), a[(slot >> 1) & 1]);
  }
  __device__ __forceinline__ void mac_d(int slot, double x, double y) {
    a[(slot >> 1) & 1] = fma(x, y, a[(slot >> 1) & 1]);
  }
  __device__ __forceinline__ void add_exact(double v) { a[0] += v; }
  __device__ __forceinline__ void flush() {}
  __device__ __forceinline__ double value() { return a[0] + a[1]; }
  __device__ __forceinline__ dd pair() { return dd_add({a[0], 0.0}, {a[1], 0.0}); }
};

// FP64, compensated per product (raw FP32 / FP64 storage, whose DOTs are
// HBM-bound with FP64 issue to spare): each product is split into its
// rounded value and exact error (exact already for FP32 operands; one FMA
// for FP64 ones), added by two-sum, and every rounding error is carried in
// lo.  The thread's sum is hi + lo to about 2^-100 relative, so the DOT is
// close to the exact sum rounded once.
struct acc_f64c {
  double hi[2] = {0.0, 0.0};
  double lo[2] = {0.0, 0.0};
  __device__ __forceinline__ void add(int k, double p, double pe) {
    double e;
    two_sum(hi[k], p, hi[k], e);
    lo[k] = __dadd_rn(lo[k], __dadd_rn(e, pe));
  }
  __device__ __forceinline__ void mac(int slot, float x, float y) {
    add(slot & 1, __dmul_rn(static_cast<double>(x), static_cast<double>(y)), 0.0);
  }
  __device__ __forceinline__ void mac_d(int slot, double x, double y) {
    const double p = __dmul_rn(x, y);
    add(slot & 1, p, __fma_rn(x, y, -p));
  }
  __device__ __forceinline__ void add_exact(double v) { add(0, v, 0.0); }
  __device__ __forceinline__ void flush() {}
  __device__ __forceinline__ dd pair() {
    return dd_add({hi[0], isfinite(hi[0]) ? lo[0] : 0.0},
                  {hi[1], isfinite(hi[1]) ? lo[1] : 0.0});
  }
  __device__ __forceinline__ double value() {
    const dd r = pair();
    return r.hi + r.lo;
  }
};

// ---- block / grid reduction (deterministic, double-double) ---------------------
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ dd warp_sum_dd(dd v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const dd w = {__shfl_down_sync(0xffffffffu, v.hi, o),
                  __shfl_down_sync(0xffffffffu, v.lo, o)};
    v = dd_add(v, w);
  }
  return v;  // valid in lane 0
}

// Largest block of any DOT kernel, and the words of shared scratch the
// block reduction needs for a block of NT threads.
constexpr int kMaxThreads = 1024;
template <int NT> constexpr int scratch_doubles = 2 * (NT / 32);
constexpr int kScratchDoubles = scratch_doubles<kThreads>;

// Sum over a block of NT threads; the result is valid in thread 0.
template <int NT = kThreads>
__device__ __forceinline__ dd block_sum_dd(dd v, double *scratch) {
  static_assert(NT % 32 == 0 && NT <= kMaxThreads, "whole warps, at most kMaxThreads");
  v = warp_sum_dd(v);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) {
    scratch[2 * warp] = v.hi;
    scratch[2 * warp + 1] = v.lo;
  }
  __syncthreads();
  dd s = {0.0, 0.0};
  if (warp == 0) {
    if (lane < NT / 32) s = {scratch[2 * lane], scratch[2 * lane + 1]};
    s = warp_sum_dd(s);
  }
  __syncthreads();
  return s;
}

// Programmatic dependent launch (the DOT kernels are launched with
// programmatic stream serialisation, so a DOT may be scheduled while the
// kernel before it on the stream is still finishing).  `pdl_wait` returns
// once every grid this one depends on has completed and its memory is
// visible: each DOT kernel calls it before its first global memory access,
// so it reads its inputs, tables, partials and ticket exactly as with
// ordinary stream order.  `pdl_release` then lets the next kernel on the
// stream be scheduled: it takes effect once every block of this grid has
// called it (so every block of this grid is resident by then) and the next
// kernel still waits for this grid's completion before its own first
// access.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Single-pass grid reduction: every block publishes its partial (hi, lo at
// partials[2b], [2b + 1]) and takes a ticket with a release-acquire atomic
// add, which orders the partial before the ticket; the last block to arrive
// (its acquire, then the block barrier, orders every other block's partial
// before its reads) sums the partials in block order and resets the ticket
// for the next launch.  No block waits on another, so the pattern cannot
// hang.  The result is hi + lo rounded once.  `claims` (optional) is a
// counter every block has finished with by the time it takes its ticket; the
// last block resets it too.
template <int NT = kThreads>
__device__ __forceinline__ void grid_finish_dd(dd block_partial, double *partials,
                                               unsigned int *ticket, double *result,
                                               double *scratch,
                                               unsigned int *claims = nullptr) {
  __shared__ bool last_block;
  if (threadIdx.x == 0) {
    partials[2 * blockIdx.x] = block_partial.hi;
    partials[2 * blockIdx.x + 1] = block_partial.lo;
    unsigned int arrived;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(arrived)
                 : "l"(ticket)
                 : "memory");
    last_block = (arrived == gridDim.x - 1);
  }
  __syncthreads();
  if (!last_block) return;
  dd s = {0.0, 0.0};
  for (unsigned int b = threadIdx.x; b < gridDim.x; b += NT)
    s = dd_add(s, {__ldcg(partials + 2 * b), __ldcg(partials + 2 * b + 1)});
  s = block_sum_dd<NT>(s, scratch);
  if (threadIdx.x == 0) {
    *result = __dadd_rn(s.hi, s.lo);
    *ticket = 0u;
    if (claims != nullptr) *claims = 0u;
  }
}

} // namespace aut::dev

#endif

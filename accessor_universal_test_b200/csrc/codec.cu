// codec.cu -- device encode (RNE + dense pack), bit-exact decode and the
// seeded synthetic generators.
//
// Encode replaces encode_padded_kernel + pack_dense_kernel
// (bitwidth_benchmark_kernels.cuh:625-668, lns_benchmark_kernels.cuh:309-357)
// in one pass: a thread encodes one aligned chunk of 32/gcd(B,32) values and
// writes its B/gcd whole words, so no two threads touch one word.  LNS codes
// come from a binary search over thresholds computed with the host's log2,
// which makes them equal to the host encoder's for every input.
#include "dot_device.cuh"
#include "internal.hpp"

#include "aut/detail/codec_core.hpp"
#include "aut/dot_dataset.hpp"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace aut::dev {

struct codec_params {
  int family;
  int total_bits;
  int exponent_bits;
  int finite;
  int stride;      // bits per stored slot
  // LNS encode / decode tables
  const double *thresholds;
  double zero_threshold;
  const float *lns_f32;
  const double *lns_f64;
};

__device__ __forceinline__ uint32_t encode_one(const codec_params &p, double v) {
  using namespace aut::detail;
  switch (p.family) {
  case AUT_FAMILY_BINARY:
    return p.exponent_bits == 0
               ? fixed_encode(p.total_bits, v)
               : ieee_encode(p.total_bits, p.exponent_bits, p.finite != 0, v);
  case AUT_FAMILY_FP64_PREFIX: return prefix_encode(p.total_bits - 12, v);
  case AUT_FAMILY_RAW_FP32: return __float_as_uint(__double2float_rn(v));
  default: {  // LNS
    const int B = p.total_bits;
    const uint32_t zero_raw = lns_special(B);
    const int32_t lo = -static_cast<int32_t>(lns_special(B)) + 1;
    const int32_t hi = static_cast<int32_t>(lns_special(B)) - 1;
    if (v != v) return lns_sign_mask(B) | zero_raw;
    const bool neg = v < 0.0;
    if (isinf(v))
      return (neg ? lns_sign_mask(B) : 0u) | (static_cast<uint32_t>(hi) & lns_log_mask(B));
    if (v == 0.0) return zero_raw;
    const double mag = fabs(v);
    if (mag < p.zero_threshold) return zero_raw;
    uint32_t a = 0, b = static_cast<uint32_t>(hi - lo);
    while (a < b) {  // count thresholds <= mag
      const uint32_t mid = (a + b) >> 1;
      if (__ldg(p.thresholds + mid) <= mag)
        a = mid + 1;
      else
        b = mid;
    }
    const int32_t code = lo + static_cast<int32_t>(a);
    return (neg ? lns_sign_mask(B) : 0u) | (static_cast<uint32_t>(code) & lns_log_mask(B));
  }
  }
}

__global__ void encode_dense_kernel(codec_params p, const double *values,
                                    uint64_t n, uint32_t *words,
                                    uint64_t word_count) {
  const int B = p.stride;
  int g = B, r = 32;
  while (r != 0) {
    const int t = g % r;
    g = r;
    r = t;
  }
  const int per_chunk = 32 / g;     // values per aligned chunk
  const int chunk_words = B / g;    // words per aligned chunk (<= 32)
  const uint64_t chunks = (n + per_chunk - 1) / per_chunk;
  const uint32_t mask = aut::detail::low_mask32(p.total_bits);
  for (uint64_t c = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
       c < chunks; c += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    uint32_t w[32];
    for (int k = 0; k < chunk_words; ++k) w[k] = 0u;
    for (int v = 0; v < per_chunk; ++v) {
      const uint64_t i = c * per_chunk + v;
      const uint32_t code = i < n ? (encode_one(p, __ldg(values + i)) & mask) : 0u;
      const int bit = v * B;
      const int k = bit >> 5;
      const int sh = bit & 31;
      const uint64_t placed = static_cast<uint64_t>(code) << sh;
      w[k] |= static_cast<uint32_t>(placed);
      if (sh + B > 32) w[k + 1] |= static_cast<uint32_t>(placed >> 32);
    }
    for (int k = 0; k < chunk_words; ++k) {
      const uint64_t idx = c * chunk_words + k;
      if (idx < word_count) words[idx] = w[k];
    }
  }
}

__global__ void encode_padded_kernel(codec_params p, const double *values,
                                     uint64_t n, void *out) {
  const uint32_t mask = aut::detail::low_mask32(p.total_bits);
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t code = encode_one(p, __ldg(values + i)) & mask;
    if (p.stride == 8) static_cast<uint8_t *>(out)[i] = static_cast<uint8_t>(code);
    else if (p.stride == 16) static_cast<uint16_t *>(out)[i] = static_cast<uint16_t>(code);
    else static_cast<uint32_t *>(out)[i] = code;
  }
}

__global__ void zero_word_kernel(uint32_t *w) { *w = 0u; }

__device__ __forceinline__ uint32_t load_any(const void *base, int stride,
                                             uint64_t i) {
  if (stride == 8) return static_cast<const uint8_t *>(base)[i];
  if (stride == 16) return static_cast<const uint16_t *>(base)[i];
  if (stride == 32) return static_cast<const uint32_t *>(base)[i];
  const uint32_t *w = static_cast<const uint32_t *>(base);
  const uint64_t bit = i * static_cast<uint64_t>(stride);
  const uint64_t k = bit >> 5;
  const unsigned sh = static_cast<unsigned>(bit & 31u);
  const uint32_t lo = w[k];
  const uint32_t hi = sh + stride > 32 ? w[k + 1] : 0u;
  return __funnelshift_r(lo, hi, sh);
}

__device__ __forceinline__ double decode_one_f64(const codec_params &p,
                                                 uint32_t raw) {
  using namespace aut::detail;
  switch (p.family) {
  case AUT_FAMILY_BINARY:
    return p.exponent_bits == 0
               ? fixed_decode(p.total_bits, raw)
               : ieee_decode(p.total_bits, p.exponent_bits, p.finite != 0, raw);
  case AUT_FAMILY_FP64_PREFIX: return prefix_decode(p.total_bits - 12, raw);
  case AUT_FAMILY_RAW_FP32: return static_cast<double>(__uint_as_float(raw));
  default: return p.lns_f64[raw & low_mask32(p.total_bits)];
  }
}

__device__ __forceinline__ float decode_one_f32(const codec_params &p,
                                                uint32_t raw) {
  if (p.family == AUT_FAMILY_LNS)
    return p.lns_f32[raw & aut::detail::low_mask32(p.total_bits)];
  if (p.family == AUT_FAMILY_RAW_FP32) return __uint_as_float(raw);
  // Same narrowing as the reference's FP32 decode (decode_reference<fp32>):
  // exact for E <= 8, M <= 23.
  return __double2float_rn(decode_one_f64(p, raw));
}

__global__ void decode_kernel(codec_params p, const void *codes, uint64_t n,
                              void *out, int target) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    if (p.family == AUT_FAMILY_RAW_FP64) {
      const double v = static_cast<const double *>(codes)[i];
      if (target == AUT_TARGET_FP64) static_cast<double *>(out)[i] = v;
      else static_cast<float *>(out)[i] = __double2float_rn(v);
      continue;
    }
    const uint32_t raw = load_any(codes, p.stride, i) &
                         aut::detail::low_mask32(p.total_bits);
    if (target == AUT_TARGET_FP64)
      static_cast<double *>(out)[i] = decode_one_f64(p, raw);
    else
      static_cast<float *>(out)[i] = decode_one_f32(p, raw);
  }
}

// ---- synthetic generators (restated on the host by the oracle) --------------
__device__ __forceinline__ uint64_t splitmix64(uint64_t v) {
  v += 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

__device__ __forceinline__ uint64_t lane_seed(uint64_t seed, int vector_id) {
  return seed ^ (0xd1b54a32d192ed03ull * static_cast<uint64_t>(vector_id + 1));
}

__device__ __forceinline__ double signed_unit_f64(uint64_t bits) {
  const int64_t centered = static_cast<int64_t>(bits >> 12) - (int64_t{1} << 51);
  return __dmul_rn(__ll2double_rn(centered), 0x1p-51);
}

__device__ __forceinline__ double synthetic(int kind, uint64_t seed,
                                            int vector_id, uint64_t i) {
  const uint64_t ls = lane_seed(seed, vector_id);
  switch (kind) {
  case AUT_GEN_SIGNED_UNIT_F64: return signed_unit_f64(splitmix64(i ^ ls));
  case AUT_GEN_SIGNED_UNIT_F32: {
    const uint32_t fraction = static_cast<uint32_t>(splitmix64(i ^ ls) >> 41);
    const int32_t centered = static_cast<int32_t>(fraction) - (1 << 22);
    return static_cast<double>(__fmul_rn(__int2float_rn(centered), 0x1p-22f));
  }
  case AUT_GEN_NORMAL: {
    uint64_t acc = 0;
#pragma unroll
    for (uint64_t k = 0; k < 12; ++k) acc += splitmix64((i * 12u + k) ^ ls) >> 11;
    return __dsub_rn(__dmul_rn(__ull2double_rn(acc), 0x1p-53), 6.0);
  }
  case AUT_GEN_POSITIVE_UNIT_F64:
    return __dmul_rn(__ull2double_rn((splitmix64(i ^ ls) >> 11) + 1u), 0x1p-53);
  default: {  // AUT_GEN_LNS_CANCEL
    const double x = signed_unit_f64(splitmix64(i ^ lane_seed(seed, 0)));
    if (vector_id == 0) return x;
    const double u = signed_unit_f64(splitmix64(i ^ lane_seed(seed, 2)));
    const double p = __dmul_rn(x, __dadd_rn(1.0, __dmul_rn(1e-6, u)));
    return (i & 1u) ? -p : p;
  }
  }
}

__global__ void generate_kernel(int kind, uint64_t seed, int vector_id,
                                uint64_t first, uint64_t n, double *out) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    out[i] = synthetic(kind, seed, vector_id, first + i);
}

// Values [first, first + n) of vector `vector_id` of a dot_v1 case of `count`
// values (dot_dataset.hpp: the reference's generators, bit for bit).
__global__ void generate_dot_v1_kernel(aut::dataset::parameters spec, int vector_id,
                                       uint64_t count, uint64_t first, uint64_t n, float *out) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    out[i] = aut::dataset::value(spec, vector_id, first + i, count);
}

// ---- the generic DOT: any registered format, one value per thread ---------------
// The runtime switch over the registry (the reference compiles one binary per
// width, src/bitwidth_strategy_bench.cu:955-1211): codes are read by absolute
// value index (one or two word loads, consecutive threads on consecutive
// values, so a warp's loads coalesce) and decoded by the bit-exact decoders
// above; products go into the same accumulators and single-pass grid
// reduction as the fused kernels.
struct generic_dot_params {
  codec_params codec;
  const unsigned char *x;
  const unsigned char *y;
  uint64_t n;
  uint64_t x_stride, y_stride;              // bytes between the pairs of a batch
  uint64_t x_first, y_first;                // value index of pair 0
  uint64_t x_index_stride, y_index_stride;  // values between the pairs of a batch
  int table_smem_bytes;  // LNS: full decode table staged in shared memory
  double *partials;
  unsigned int *tickets;
  double *results;
};

template <class Acc, bool kF32>
__global__ void __launch_bounds__(kThreads) dot_generic_kernel(const generic_dot_params g) {
  extern __shared__ __align__(16) unsigned char table[];
  __shared__ double scratch[kScratchDoubles];
  codec_params c = g.codec;
  if (g.table_smem_bytes > 0) {
    const uint4 *src = kF32 ? reinterpret_cast<const uint4 *>(c.lns_f32)
                            : reinterpret_cast<const uint4 *>(c.lns_f64);
    uint4 *dst = reinterpret_cast<uint4 *>(table);
    for (int k = threadIdx.x; k < g.table_smem_bytes / 16; k += kThreads) dst[k] = src[k];
    __syncthreads();
    if constexpr (kF32)
      c.lns_f32 = reinterpret_cast<const float *>(table);
    else
      c.lns_f64 = reinterpret_cast<const double *>(table);
  }
  const unsigned int batch = blockIdx.y;
  const unsigned char *xb = g.x + batch * g.x_stride;
  const unsigned char *yb = g.y + batch * g.y_stride;
  const uint64_t xo = g.x_first + batch * g.x_index_stride;
  const uint64_t yo = g.y_first + batch * g.y_index_stride;
  const uint32_t mask = aut::detail::low_mask32(c.total_bits);

  Acc acc;
  auto mac = [&](int slot, uint32_t rx, uint32_t ry) {
    if constexpr (kF32)
      acc.mac(slot, decode_one_f32(c, rx & mask), decode_one_f32(c, ry & mask));
    else
      acc.mac_d(slot, decode_one_f64(c, rx & mask), decode_one_f64(c, ry & mask));
  };
  const uint64_t step = static_cast<uint64_t>(gridDim.x) * kThreads;
  uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  int done = 0;
  // four independent values in flight per thread
  for (; i + 3 * step < g.n; i += 4 * step) {
    uint32_t rx[4], ry[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      rx[k] = load_any(xb, c.stride, xo + i + k * step);
      ry[k] = load_any(yb, c.stride, yo + i + k * step);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) mac(k, rx[k], ry[k]);
    if ((done += 4) == 128) {  // 32 products per FP32 chain between FP64 carries
      acc.flush();
      done = 0;
    }
  }
  for (; i < g.n; i += step) mac(0, load_any(xb, c.stride, xo + i), load_any(yb, c.stride, yo + i));
  const dd s = block_sum_dd(acc.pair(), scratch);
  grid_finish_dd(s, g.partials + 2 * static_cast<uint64_t>(batch) * gridDim.x, g.tickets + batch,
                 g.results + batch, scratch);
}

} // namespace aut::dev

namespace aut::lib {

namespace {
unsigned grid_for(uint64_t items) {
  const uint64_t b = (items + 255) / 256;
  return static_cast<unsigned>(b == 0 ? 1 : (b > 8192 ? 8192 : b));
}

aut_status make_params(aut_workspace *ws, const format_desc &f, int32_t format,
                       int32_t layout, aut::dev::codec_params &p) {
  p.family = f.family;
  p.total_bits = f.total_bits;
  p.exponent_bits = f.exponent_bits;
  p.finite = f.finite;
  p.stride = stride_bits(f, layout);
  p.thresholds = nullptr;
  p.zero_threshold = 0.0;
  p.lns_f32 = nullptr;
  p.lns_f64 = nullptr;
  if (f.family == AUT_FAMILY_LNS) {
    const code_tables *t = nullptr;
    const aut_status st = code_tables_for(ws, format, &t);
    if (st != AUT_OK) return st;
    p.thresholds = t->thresholds;
    p.zero_threshold = t->zero_threshold;
    p.lns_f32 = t->full_f32;
    p.lns_f64 = t->full_f64;
  }
  return AUT_OK;
}
} // namespace

aut_status launch_encode(aut_workspace *ws, const format_desc &f, int32_t format,
                         int32_t layout, const double *values, uint64_t n,
                         void *codes, cudaStream_t stream) {
  if (f.family == AUT_FAMILY_RAW_FP64)
    return fail(AUT_ERR_UNSUPPORTED, "fp64 storage needs no encode");
  aut::dev::codec_params p;
  aut_status st = make_params(ws, f, format, layout, p);
  if (st != AUT_OK) return st;
  const bool packed_words = !(p.stride == 8 || p.stride == 16 || p.stride == 32);
  if (layout == AUT_LAYOUT_PADDED || !packed_words) {
    if (n > 0) {
      aut::dev::encode_padded_kernel<<<grid_for(n), 256, 0, stream>>>(p, values, n, codes);
      AUT_CUDA_TRY(cudaGetLastError());
    }
    if (layout == AUT_LAYOUT_DENSE && f.family != AUT_FAMILY_RAW_FP32) {
      // dense 8/16/32-bit streams: zero the rest of the last word and the guard
      const uint64_t used = n * p.stride / 8;
      const uint64_t words = (n * p.stride + 31) / 32 + 1;
      AUT_CUDA_TRY(cudaMemsetAsync(static_cast<uint8_t *>(codes) + used, 0,
                                   words * 4 - used, stream));
    }
    return AUT_OK;
  }
  const uint64_t word_count = (n * p.stride + 31) / 32 + 1;
  if (n > 0) {
    aut::dev::encode_dense_kernel<<<grid_for(n / 4 + 1), 256, 0, stream>>>(
        p, values, n, static_cast<uint32_t *>(codes), word_count);
    AUT_CUDA_TRY(cudaGetLastError());
  }
  aut::dev::zero_word_kernel<<<1, 1, 0, stream>>>(static_cast<uint32_t *>(codes) + word_count - 1);
  AUT_CUDA_TRY(cudaGetLastError());
  return AUT_OK;
}

aut_status launch_decode(aut_workspace *ws, const format_desc &f, int32_t format,
                         int32_t layout, int32_t target, const void *codes,
                         uint64_t n, void *out, cudaStream_t stream) {
  aut::dev::codec_params p;
  aut_status st = make_params(ws, f, format, layout, p);
  if (st != AUT_OK) return st;
  if (n == 0) return AUT_OK;
  aut::dev::decode_kernel<<<grid_for(n), 256, 0, stream>>>(p, codes, n, out, target);
  AUT_CUDA_TRY(cudaGetLastError());
  return AUT_OK;
}

aut_status launch_generate(int32_t kind, uint64_t seed, int32_t vector_id,
                           uint64_t first, uint64_t n, double *out,
                           cudaStream_t stream) {
  if (n == 0) return AUT_OK;
  aut::dev::generate_kernel<<<grid_for(n), 256, 0, stream>>>(kind, seed, vector_id,
                                                             first, n, out);
  AUT_CUDA_TRY(cudaGetLastError());
  return AUT_OK;
}

aut_status launch_generate_dot_v1(int32_t family, uint64_t seed, int32_t parameter,
                                  int32_t vector_id, uint64_t count, uint64_t first,
                                  uint64_t n, float *out, cudaStream_t stream) {
  if (n == 0) return AUT_OK;
  aut::dataset::parameters spec;
  spec.kind = static_cast<aut::dataset::family>(family);
  spec.seed = seed;
  spec.parameter = parameter;
  aut::dev::generate_dot_v1_kernel<<<grid_for(n), 256, 0, stream>>>(spec, vector_id, count,
                                                                    first, n, out);
  AUT_CUDA_TRY(cudaGetLastError());
  return AUT_OK;
}

bool generic_dot_ok(const format_desc &f, int32_t accum) {
  switch (f.family) {
  case AUT_FAMILY_BINARY: {
    if (accum == AUT_ACCUM_FP64) return true;
    // FP32 only where every value is an FP32 value (decode_fp32_bits,
    // decoder_strategy_core.hpp:297-303: E <= 8, M <= 23)
    const int m = f.total_bits - f.exponent_bits - 1;
    return f.exponent_bits <= 8 && m <= 23;
  }
  case AUT_FAMILY_FP64_PREFIX: return accum == AUT_ACCUM_FP64;
  case AUT_FAMILY_LNS: return f.total_bits <= 16;  // host-built decode tables
  default: return false;  // raw FP32 / FP64 have fused kernels
  }
}

aut_status generic_dot_launch(aut_workspace *ws, const format_desc &f, int32_t format,
                              int32_t layout, int32_t accum, const void *x, const void *y,
                              uint64_t n, uint32_t batch, const batch_layout &bl,
                              double *results, cudaStream_t stream, double *partials,
                              unsigned int *tickets, int max_blocks_total) {
  if (!generic_dot_ok(f, accum))
    return fail(AUT_ERR_UNSUPPORTED, std::string("no DOT kernel for ") + f.name +
                                         " with this accumulator");
  aut::dev::generic_dot_params g{};
  aut_status st = make_params(ws, f, format, layout, g.codec);
  if (st != AUT_OK) return st;
  const bool f32 = accum == AUT_ACCUM_FP32;
  if (f.family == AUT_FAMILY_LNS) {
    const int bytes = (1 << f.total_bits) * (f32 ? 4 : 8);
    g.table_smem_bytes = bytes <= 32 * 1024 ? bytes : 0;  // larger tables stay in L2
  }
  using fn_t = void (*)(aut::dev::generic_dot_params);
  const fn_t fn = f32 ? aut::dev::dot_generic_kernel<aut::dev::acc_f32, true>
                      : aut::dev::dot_generic_kernel<aut::dev::acc_f64, false>;
  static std::atomic<int> occupancy[2];  // blocks per SM without a staged table
  int per_sm = occupancy[f32].load(std::memory_order_relaxed);
  if (g.table_smem_bytes > 0 || per_sm == 0) {
    AUT_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      32 * 1024));
    AUT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, fn, aut::dev::kThreads, g.table_smem_bytes));
    if (g.table_smem_bytes == 0) occupancy[f32].store(per_sm, std::memory_order_relaxed);
  }
  if (per_sm < 1) per_sm = 1;
  const uint64_t cap = static_cast<uint64_t>(ws->sm_count) * per_sm;
  uint64_t wanted = (n + aut::dev::kThreads * 16 - 1) / (aut::dev::kThreads * 16);
  if (wanted == 0) wanted = 1;
  for (uint32_t b0 = 0; b0 < batch; b0 += kMaxBatchPerLaunch) {
    const uint32_t nb = batch - b0 < static_cast<uint32_t>(kMaxBatchPerLaunch)
                            ? batch - b0
                            : static_cast<uint32_t>(kMaxBatchPerLaunch);
    uint64_t per_pair = (cap + nb - 1) / nb;
    if (per_pair > wanted) per_pair = wanted;
    if (per_pair > static_cast<uint64_t>(max_blocks_total)) per_pair = max_blocks_total;
    if (per_pair < 1) per_pair = 1;
    g.x = static_cast<const unsigned char *>(x) + static_cast<uint64_t>(b0) * bl.x_stride;
    g.y = static_cast<const unsigned char *>(y) + static_cast<uint64_t>(b0) * bl.y_stride;
    g.n = n;
    g.x_stride = bl.x_stride;
    g.y_stride = bl.y_stride;
    g.x_first = static_cast<uint64_t>(b0) * bl.x_index_stride;
    g.y_first = static_cast<uint64_t>(b0) * bl.y_index_stride;
    g.x_index_stride = bl.x_index_stride;
    g.y_index_stride = bl.y_index_stride;
    g.partials = partials;
    g.tickets = tickets;
    g.results = results + b0;
    dim3 grid(static_cast<unsigned>(per_pair), nb);
    fn<<<grid, aut::dev::kThreads, g.table_smem_bytes, stream>>>(g);
    AUT_CUDA_TRY(cudaGetLastError());
  }
  return AUT_OK;
}

} // namespace aut::lib

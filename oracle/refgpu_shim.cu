// refgpu_shim.cu -- the reference's own GPU DOT kernels behind a C ABI.
//
// TEST INFRASTRUCTURE ONLY: built into oracle/_ref/librefgpu.so by
// oracle/Makefile from the reference's headers where they lie (nvcc,
// sm_100a), and loaded only by tests/ to run the reference's kernels on the
// same B200 and the same device buffers as libautdot -- the normalised
// error and GB/s of "the reference's own GPU kernel for the same format and
// accumulator".  The product never loads it.
//
// Kernels (unchanged, instantiated here):
//   dot_thread_kernel + finalize_dot_kernel  include/bitwidth_benchmark_kernels.cuh:403-457
//   raw_dot_kernel                           include/bitwidth_benchmark_kernels.cuh:681-703
//   LNS dot_thread_kernel + finalize         include/lns_benchmark_kernels.cuh:80-131
// launched the way the reference's benchmarks launch them: 256 threads,
// min(512, ceil(packets / 256)) blocks (src/bitwidth_strategy_bench.cu:
// 620-649, src/lns_strategy_bench.cu:844-869), dynamic shared memory =
// shared table + 256 accumulators.  Decode tables of the LNS table decoders
// are built on the host from the reference's own host decoder (full table)
// and exp2 of each fraction step (fraction table).
#include "bitwidth_benchmark_kernels.cuh"
#include "lns_benchmark_kernels.cuh"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

namespace {

namespace bw = aut::bitwidth;
namespace ls = aut::lns_strategy;
namespace st = aut::storage;

struct run_out {
  double result;
  double ms;  // per DOT (dot kernel + finalize), CUDA events
};

int grid_for(std::size_t count, int lanes) {
  const std::size_t packets = (count + lanes - 1) / lanes;
  const std::size_t blocks = (packets + 255) / 256;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > 512 ? 512 : blocks));
}

template <typename T> struct device_buf {
  T *p = nullptr;
  explicit device_buf(std::size_t n) { cudaMalloc(&p, (n ? n : 1) * sizeof(T)); }
  ~device_buf() { cudaFree(p); }
};

template <typename Launch>
int time_it(Launch launch, int reps, double &ms) {
  launch();
  launch();
  if (cudaDeviceSynchronize() != cudaSuccess) return 1;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a);
  for (int r = 0; r < reps; ++r) launch();
  cudaEventRecord(b);
  cudaEventSynchronize(b);
  float t = 0.f;
  cudaEventElapsedTime(&t, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  ms = static_cast<double>(t) / reps;
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

// bit formats: dot_thread_kernel<Format, Compute, Layout, Lanes, Decoder>
template <typename Format, bw::compute_kind Compute, bw::storage_layout Layout, int Lanes,
          bw::decoder_kind Decoder>
int run_bits(const void *x, const void *y, std::uint64_t n, int reps, run_out &out) {
  using T = bw::compute_t<Compute>;
  const int blocks = grid_for(n, Lanes);
  device_buf<T> partials(512), result(1);
  bw::storage_view<Format, Layout> left{static_cast<const std::uint32_t *>(x),
                                        static_cast<const bw::padded_storage_t<Format> *>(x)};
  bw::storage_view<Format, Layout> right{static_cast<const std::uint32_t *>(y),
                                         static_cast<const bw::padded_storage_t<Format> *>(y)};
  const std::size_t smem = 256 * sizeof(T);
  auto launch = [&] {
    bw::dot_thread_kernel<Format, Compute, Layout, Lanes, Decoder>
        <<<blocks, 256, smem>>>(left, right, n, bw::decoder_tables{}, partials.p);
    bw::finalize_dot_kernel<<<1, 256>>>(partials.p, static_cast<std::size_t>(blocks), result.p);
  };
  if (time_it(launch, reps, out.ms)) return 1;
  T r{};
  if (cudaMemcpy(&r, result.p, sizeof r, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
  out.result = static_cast<double>(r);
  return 0;
}

// raw FP32 / FP64 storage: raw_dot_kernel<T, Lanes>
template <typename T, int Lanes>
int run_raw(const void *x, const void *y, std::uint64_t n, int reps, run_out &out) {
  const int blocks = grid_for(n, Lanes);
  device_buf<T> partials(512), result(1);
  auto launch = [&] {
    bw::raw_dot_kernel<T, Lanes><<<blocks, 256>>>(static_cast<const T *>(x),
                                                   static_cast<const T *>(y), n, partials.p);
    bw::finalize_dot_kernel<<<1, 256>>>(partials.p, static_cast<std::size_t>(blocks), result.p);
  };
  if (time_it(launch, reps, out.ms)) return 1;
  T r{};
  if (cudaMemcpy(&r, result.p, sizeof r, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
  out.result = static_cast<double>(r);
  return 0;
}

// LNS: dot_thread_kernel<Format, Compute, dense, Lanes, Decoder, Multiply>
template <typename Format, bw::compute_kind Compute, ls::decoder_kind Decoder,
          ls::multiply_kind Multiply>
int run_lns(const void *x, const void *y, std::uint64_t n, int reps, run_out &out) {
  using T = bw::compute_t<Compute>;
  constexpr int Lanes = 4;
  const int blocks = grid_for(n, Lanes);
  device_buf<T> partials(512), result(1);
  // tables from the reference's host decoder
  std::vector<T> full(std::size_t{1} << Format::total_bits);
  for (std::size_t c = 0; c < full.size(); ++c)
    full[c] = aut::lns::decode<Format, T>(static_cast<std::uint32_t>(c));
  std::vector<T> fraction(std::size_t{1} << Format::log_fraction_bits);
  for (std::size_t f = 0; f < fraction.size(); ++f)
    fraction[f] = static_cast<T>(
        std::exp2(static_cast<double>(f) / static_cast<double>(fraction.size())));
  device_buf<T> d_full(full.size()), d_fraction(fraction.size());
  cudaMemcpy(d_full.p, full.data(), full.size() * sizeof(T), cudaMemcpyHostToDevice);
  cudaMemcpy(d_fraction.p, fraction.data(), fraction.size() * sizeof(T),
             cudaMemcpyHostToDevice);
  ls::table_bundle<Compute> tables{};
  tables.full = d_full.p;
  tables.fraction = d_fraction.p;
  ls::storage_view<Format, bw::storage_layout::dense> left{
      static_cast<const std::uint32_t *>(x), nullptr};
  ls::storage_view<Format, bw::storage_layout::dense> right{
      static_cast<const std::uint32_t *>(y), nullptr};
  const std::size_t smem = ls::shared_table_bytes_v<Format, Compute, Decoder> + 256 * sizeof(T);
  auto kernel = ls::dot_thread_kernel<Format, Compute, bw::storage_layout::dense, Lanes,
                                      Decoder, Multiply>;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  auto launch = [&] {
    kernel<<<blocks, 256, smem>>>(left, right, n, tables, partials.p);
    ls::finalize_dot_kernel<<<1, 256>>>(partials.p, static_cast<std::size_t>(blocks), result.p);
  };
  if (time_it(launch, reps, out.ms)) return 1;
  T r{};
  if (cudaMemcpy(&r, result.p, sizeof r, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
  out.result = static_cast<double>(r);
  return 0;
}

using runner = int (*)(const void *, const void *, std::uint64_t, int, run_out &);
struct variant {
  const char *name;  // format/accumulator/layout/lanes/decoder[/multiply]
  runner fn;
};

constexpr auto F32 = bw::compute_kind::fp32;
constexpr auto F64 = bw::compute_kind::fp64;
constexpr auto DENSE = bw::storage_layout::dense;
constexpr auto PADDED = bw::storage_layout::padded;
constexpr auto DIRECT = bw::decoder_kind::direct_branchy;
constexpr auto NATIVE = bw::decoder_kind::native_packed;

#define AUT_BITS(fmt, name)                                                                 \
  {name "/fp32/dense/x4/direct_branchy", run_bits<st::fmt, F32, DENSE, 4, DIRECT>},          \
      {name "/fp64/dense/x4/direct_branchy", run_bits<st::fmt, F64, DENSE, 4, DIRECT>},      \
      {name "/fp32/padded/x4/direct_branchy", run_bits<st::fmt, F32, PADDED, 4, DIRECT>},    \
      {name "/fp64/padded/x4/direct_branchy", run_bits<st::fmt, F64, PADDED, 4, DIRECT>}
#define AUT_LNS(fmt, name)                                                                  \
  {name "/fp32/dense/x4/ex2_approx/ordinary",                                               \
   run_lns<aut::lns::fmt, F32, ls::decoder_kind::ex2_approx, ls::multiply_kind::ordinary>}, \
      {name "/fp32/dense/x4/ex2_approx/fused",                                              \
       run_lns<aut::lns::fmt, F32, ls::decoder_kind::ex2_approx, ls::multiply_kind::fused>}, \
      {name "/fp64/dense/x4/ex2_approx/fused",                                              \
       run_lns<aut::lns::fmt, F64, ls::decoder_kind::ex2_approx, ls::multiply_kind::fused>}, \
      {name "/fp32/dense/x4/fraction_lut_shared/fused",                                     \
       run_lns<aut::lns::fmt, F32, ls::decoder_kind::fraction_lut_shared,                   \
               ls::multiply_kind::fused>},                                                  \
      {name "/fp64/dense/x4/fraction_lut_shared/fused",                                     \
       run_lns<aut::lns::fmt, F64, ls::decoder_kind::fraction_lut_shared,                   \
               ls::multiply_kind::fused>}

const variant variants[] = {
    {"fp32/fp32/raw/x4/direct", run_raw<float, 4>},
    {"fp64/fp64/raw/x4/direct", run_raw<double, 4>},
    AUT_BITS(e2m3, "e2m3"),
    {"e2m3/fp32/dense/x4/native_packed", run_bits<st::e2m3, F32, DENSE, 4, NATIVE>},
    {"e2m3/fp64/dense/x4/native_packed", run_bits<st::e2m3, F64, DENSE, 4, NATIVE>},
    AUT_BITS(e8m0, "e8m0"),
    AUT_BITS(e8m1, "e8m1"),
    AUT_BITS(e8m3, "e8m3"),
    AUT_BITS(e8m5, "e8m5"),
    AUT_BITS(bf16_e8m7, "bf16_e8m7"),
    AUT_BITS(e8m15, "e8m15"),
    AUT_LNS(lns8_r3, "lns8_r3"),
    // the full table of 8-bit codes fits shared memory (that of 16-bit codes,
    // 2^16 entries, does not)
    {"lns8_r3/fp32/dense/x4/full_lut_shared/ordinary",
     run_lns<aut::lns::lns8_r3, F32, ls::decoder_kind::full_lut_shared,
             ls::multiply_kind::ordinary>},
    {"lns8_r3/fp64/dense/x4/full_lut_shared/ordinary",
     run_lns<aut::lns::lns8_r3, F64, ls::decoder_kind::full_lut_shared,
             ls::multiply_kind::ordinary>},
    AUT_LNS(lns16_r11, "lns16_r11"),
};
constexpr int variant_count = sizeof(variants) / sizeof(variants[0]);

} // namespace

extern "C" {

int refgpu_variant_count() { return variant_count; }

const char *refgpu_variant_name(int i) {
  return (i >= 0 && i < variant_count) ? variants[i].name : "";
}

// Runs variant i on device buffers x, y (n values, the reference's layouts:
// dense LSB-first words with the guard word, or one container per code):
// `reps` timed DOTs after two warm-up DOTs.  Returns 0 on success.
int refgpu_run(int i, const void *x, const void *y, std::uint64_t n, int reps,
               double *result, double *ms_per_dot) {
  if (i < 0 || i >= variant_count || x == nullptr || y == nullptr || reps < 1) return 2;
  run_out out{};
  const int rc = variants[i].fn(x, y, n, reps, out);
  if (rc != 0) return rc;
  *result = out.result;
  *ms_per_dot = out.ms;
  return 0;
}

} // extern "C"

// internal.hpp -- declarations shared by the library's translation units.
#ifndef AUT_INTERNAL_HPP_
#define AUT_INTERNAL_HPP_

#include "autdot.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

namespace aut {
// Bound of the bulk-copy kernels' barrier waits: ~2 s of SM clock at 2 GHz.
constexpr long long kWaitCyclesDefault = 4000000000LL;
} // namespace aut

namespace aut::lib {

// ---- registry ---------------------------------------------------------------
struct format_desc {
  const char *name;
  int family;
  int total_bits;
  int exponent_bits; // LNS: log fraction bits R
  int finite;
};

const format_desc *find_format(int32_t id); // nullptr when out of range
int stride_bits(const format_desc &f, int layout); // bits per stored value
int container_bits(const format_desc &f);          // padded container width

// ---- errors -----------------------------------------------------------------
aut_status fail(aut_status code, const std::string &message);
aut_status cuda_fail(cudaError_t err, const char *what);
void clear_error();

#define AUT_CUDA_TRY(expr)                                                     \
  do {                                                                         \
    cudaError_t aut_err_ = (expr);                                             \
    if (aut_err_ != cudaSuccess) return ::aut::lib::cuda_fail(aut_err_, #expr); \
  } while (0)

// ---- decode tables kept per workspace ----------------------------------------
// LNS formats (B <= 16) and bit formats with codes of at most 8 bits decode
// through tables built on the host from the host decoder (for LNS the
// reference's exp2f / exp2), so device values are bit-identical to it.
struct code_tables {
  int ready = 0;
  float *full_f32 = nullptr;   // 2^B entries
  double *full_f64 = nullptr;  // 2^B entries
  // bit formats of 9 to 14 bits whose FP64 values all have a zero low word:
  // the high word per code (the reference's full table for the FP64 target)
  uint32_t *full_hi = nullptr;  // 2^B entries
  // E8 codes with 1 to 5 mantissa bits: the partial tables of the prefix and
  // subnormal decoders, [512 prefix FP32 words | 512 prefix FP64 high words
  // | 2^M subnormal FP32 words | 2^M subnormal FP64 high words]
  uint32_t *part = nullptr;
  uint32_t part_sub_entries = 0;
  // LNS only:
  float *frac_f32 = nullptr;   // 2^R entries: exp2f(f / 2^R)
  double *frac_f64 = nullptr;  // 2^R entries: exp2(f / 2^R)
  // B <= 12: entry i = T(exp2((i - 2^(B-1)) / 2^R)), the magnitude of a
  // product whose two log codes, each biased by 2^(B-2), sum to i
  float *prod_f32 = nullptr;   // 2^B entries
  double *prod_f64 = nullptr;  // 2^B entries
  double *thresholds = nullptr; // encode thresholds, 2^(B-1) - 2 entries
  double zero_threshold = 0.0; // smallest magnitude that does not encode to 0
  // +-2^q * frac[f] equals the full decode for every code (FP32 / FP64), so
  // the fraction-table kernels may serve this format on this host
  int split_f32 = 0;
  int split_f64 = 0;
};

// The generic DOT (one value per thread, any registered format): whether it
// decodes `f` exactly for accumulator `accum`, and its launcher (codec.cu).
bool generic_dot_ok(const format_desc &f, int32_t accum);

constexpr int kMaxBatchPerLaunch = 1024;

// Where the pairs of a batched launch live: pair b reads x at byte
// b * x_stride and value index x_first + b * x_index_stride (and likewise y).
// Byte strides serve pairs that start on 16-byte boundaries (the vector
// paths); value-index strides serve rows of a dense matrix that start inside
// a byte or word, which the per-value path reads by absolute index.
struct batch_layout {
  uint64_t x_stride = 0, y_stride = 0;
  uint64_t x_index_stride = 0, y_index_stride = 0;
};
constexpr int kTableFormatsCached = 64;  // every table-decoded registered format

} // namespace aut::lib

struct aut_workspace {
  int device = 0;
  int sm_count = 0;
  int max_blocks = 0;       // per launch, all batches together
  double *partials = nullptr; // [kMaxBatchPerLaunch * max_blocks]
  unsigned int *tickets = nullptr; // [2 * kMaxBatchPerLaunch + 1], kept at zero:
                                   // the grid tickets, the sticky status word,
                                   // then the dynamic-tail tile counters
  unsigned int *claims = nullptr;  // = tickets + kMaxBatchPerLaunch + 1
  std::mutex mutex;
  // failure-detection test hook (aut_workspace_inject_stall)
  long long wait_cycles = aut::kWaitCyclesDefault;
  uint64_t stall_tile = ~0ull;
  int table_ids[aut::lib::kTableFormatsCached];
  aut_workspace() {
    for (int &id : table_ids) id = -1;
  }
  aut::lib::code_tables tables[aut::lib::kTableFormatsCached];
};

namespace aut::lib {
// Returns the decode tables of a format (LNS, or a bit format of at most 8
// bits), building them on first use.
aut_status code_tables_for(aut_workspace *ws, int32_t format_id,
                          const code_tables **out);
} // namespace aut::lib

#endif

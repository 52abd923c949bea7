// noalloc.cu -- aut_dot_noalloc: the fused DOT for callers that cannot
// allocate device memory.
//
// aut_dot keeps its grid-reduction scratch (one FP64 partial per block, one
// arrival counter per DOT) in a workspace made by cudaMalloc.  Some callers
// cannot make that call: code that runs inside a host framework which owns
// all of the GPU's memory through its own pool and forbids side allocations,
// code on a latency-critical path where cudaMalloc's implicit device-wide
// synchronisation is not acceptable, or a foreign-language caller with no
// place to keep a workspace alive.  This entry point serves them: its scratch
// is a file-scope device array that is loaded with the library's device code
// and stays resident, on every GPU that loads it, until the process exits.
//
// Limits and rules:
//   * at most kMaxPairs DOTs per call and kSlots partial slots in total
//     (32 KiB of FP64 partials + counters); larger batches are refused with
//     AUT_ERR_TOO_LARGE;
//   * formats that decode through tables (lns8_r3, lns16_r11) need a
//     workspace and are refused with AUT_ERR_UNSUPPORTED;
//   * every call, on every stream, shares the one array: calls that overlap
//     on the same GPU race and their results are undefined; serialise them
//     (one stream, or events);
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, which also loads the module if it is not loaded
//     yet); make that first call before any stream capture.  Only a
//     successful lookup is kept: a call whose lookup failed returns
//     AUT_ERR_CUDA and the next call on that device tries again;
//   * there is no status query: a DOT whose bounded bulk-copy wait gave up
//     (AUT_STATUS_WAIT_TIMEOUT under aut_dot) shows up only as NaN in its
//     results[b];
//   * a call refused for its arguments or format touches nothing on the
//     device;
//   * nothing here calls cudaMalloc, cudaFree or an allocating library.
#include "dot_device.cuh"
#include "internal.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace {

constexpr int kSlots = 4096;     // FP64 words of partials, two per block of a call
constexpr int kMaxPairs = 64;    // DOTs per call
constexpr int kMaxDevices = 64;

struct scratch_layout {
  double partials[kSlots];
  unsigned int tickets[kMaxPairs];  // arrival counters, must start at zero
  unsigned int status;              // sticky AUT_STATUS_* bits of the call
};

// The scratch array.  Host code must not pass this name to a kernel (on the
// host it only stands for the symbol); it passes the device address found
// by cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char
    noalloc_scratch[sizeof(scratch_layout)];

struct device_setup {
  std::mutex mutex;
  scratch_layout *scratch = nullptr;  // device address of noalloc_scratch
  int sm_count = 0;
  int major = 0;
};
device_setup setups[kMaxDevices];

// Looks the array up on `device` (current) until a lookup succeeds; the
// result is published only when every query succeeded.
cudaError_t set_up(device_setup &s, int device) {
  std::lock_guard<std::mutex> lock(s.mutex);
  if (s.scratch != nullptr) return cudaSuccess;
  void *ptr = nullptr;
  int sm_count = 0, major = 0;
  cudaError_t err = cudaGetSymbolAddress(&ptr, noalloc_scratch);
  if (err == cudaSuccess)
    err = cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device);
  if (err == cudaSuccess)
    err = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (err != cudaSuccess) return err;
  s.sm_count = sm_count;
  s.major = major;
  s.scratch = static_cast<scratch_layout *>(ptr);
  return cudaSuccess;
}

} // namespace

namespace aut::lib {
aut_status dot_launch_scratch(int sm_count, int32_t format, int32_t layout,
                              int32_t accum, const void *x, const void *y,
                              uint64_t n, uint32_t batch, const batch_layout &bl,
                              double *results, void *stream, double *partials,
                              unsigned int *tickets, unsigned int *status,
                              int slots, void *clear, size_t clear_bytes);
}

extern "C" aut_status aut_dot_noalloc(int32_t format, int32_t layout,
                                      int32_t accum, const void *x,
                                      const void *y, uint64_t n, uint32_t batch,
                                      uint64_t batch_stride_bytes,
                                      double *results, void *stream) {
  using namespace aut::lib;
  clear_error();
  if (find_format(format) == nullptr)
    return fail(AUT_ERR_INVALID_ARGUMENT, "unknown format id");
  if (layout != AUT_LAYOUT_DENSE && layout != AUT_LAYOUT_PADDED)
    return fail(AUT_ERR_INVALID_ARGUMENT, "layout must be DENSE or PADDED");
  if (accum != AUT_ACCUM_FP32 && accum != AUT_ACCUM_FP64)
    return fail(AUT_ERR_INVALID_ARGUMENT, "accum must be FP32 or FP64");
  if (results == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "results is NULL");
  if (batch == 0) return AUT_OK;
  if (batch > static_cast<uint32_t>(kMaxPairs))
    return fail(AUT_ERR_TOO_LARGE,
                "aut_dot_noalloc runs at most 64 DOTs per call (its scratch holds "
                "2048 block partials and 64 counters); split the batch or use "
                "aut_dot_batched");
  if (n > 0 && (x == nullptr || y == nullptr))
    return fail(AUT_ERR_INVALID_ARGUMENT, "x or y is NULL");
  if (batch > 1 && batch_stride_bytes < aut_storage_bytes(format, layout, n))
    return fail(AUT_ERR_INVALID_ARGUMENT, "batch stride smaller than one vector");

  int device = 0;
  AUT_CUDA_TRY(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices)
    return fail(AUT_ERR_INVALID_ARGUMENT, "device index beyond the set-up table");
  device_setup &s = setups[device];
  const cudaError_t err = set_up(s, device);
  if (err != cudaSuccess) return cuda_fail(err, "aut_dot_noalloc set-up");
  if (s.major != 10)
    return fail(AUT_ERR_NO_DEVICE, "libautdot is built for sm_100a");

  // The counters and the status word are cleared on the caller's stream
  // right before the launch (once the format has been accepted): a call that
  // never finished (launch error, killed context) could have left them
  // non-zero.
  batch_layout bl;
  bl.x_stride = bl.y_stride = batch_stride_bytes;
  return dot_launch_scratch(s.sm_count, format, layout, accum, x, y, n, batch,
                            bl, results, stream,
                            s.scratch->partials, s.scratch->tickets,
                            &s.scratch->status, kSlots, s.scratch->tickets,
                            sizeof(s.scratch->tickets) + sizeof(s.scratch->status));
}

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
//     yet); make that first call before any stream capture;
//   * nothing here calls cudaMalloc, cudaFree or an allocating library.
#include "dot_device.cuh"
#include "internal.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace {

constexpr int kSlots = 4096;     // FP64 partials, one per block of a call
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
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  scratch_layout *scratch = nullptr;  // device address of noalloc_scratch
  int sm_count = 0;
  int major = 0;
};
device_setup setups[kMaxDevices];

// Runs once per device, with that device current.
void set_up(device_setup &s, int device) {
  void *ptr = nullptr;
  s.err = cudaGetSymbolAddress(&ptr, noalloc_scratch);
  if (s.err != cudaSuccess) return;
  s.scratch = static_cast<scratch_layout *>(ptr);
  s.err = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, device);
  if (s.err != cudaSuccess) return;
  s.err = cudaDeviceGetAttribute(&s.major, cudaDevAttrComputeCapabilityMajor, device);
}

} // namespace

namespace aut::lib {
aut_status dot_launch_scratch(int sm_count, int32_t format, int32_t layout,
                              int32_t accum, const void *x, const void *y,
                              uint64_t n, uint32_t batch, const batch_layout &bl,
                              double *results, void *stream, double *partials,
                              unsigned int *tickets, unsigned int *status,
                              int slots);
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
                "4096 partial slots and 64 counters); split the batch or use "
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
  std::call_once(s.once, set_up, std::ref(s), device);
  if (s.err != cudaSuccess) return cuda_fail(s.err, "aut_dot_noalloc set-up");
  if (s.major != 10)
    return fail(AUT_ERR_NO_DEVICE, "libautdot is built for sm_100a");

  // The counters must start at zero; a call that never finished (launch
  // error, killed context) could have left them otherwise.
  AUT_CUDA_TRY(cudaMemsetAsync(s.scratch->tickets, 0,
                               sizeof(s.scratch->tickets) + sizeof(s.scratch->status),
                               static_cast<cudaStream_t>(stream)));
  batch_layout bl;
  bl.x_stride = bl.y_stride = batch_stride_bytes;
  return dot_launch_scratch(s.sm_count, format, layout, accum, x, y, n, batch,
                            bl, results, stream,
                            s.scratch->partials, s.scratch->tickets,
                            &s.scratch->status, kSlots);
}

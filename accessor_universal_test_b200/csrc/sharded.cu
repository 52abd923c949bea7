// sharded.cu -- multi-GPU DOTs: each rank reduces its contiguous shard with
// the fused DOT and one NCCL all-reduce of FP64 partials, on the caller's
// stream, combines them.
//
// The reference runs on one GPU and has no collective; its long-vector
// DOTs become, across the GPUs of one node, a sum of per-shard partials.
// Shards are contiguous value ranges; for dense streams a shard that starts
// on a whole 16-byte packet (128 / gcd(bits, 128) values) is a byte offset
// into the global stream, so every rank reads its part of one stream in
// place.  NCCL is loaded at the first communicator call (dlopen of
// libnccl.so.2, the one already in the process if a framework loaded it),
// so the library itself loads and runs single-GPU DOTs without NCCL.
#include "internal.hpp"

#include <nccl.h>

#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>

namespace {

struct nccl_api {
  void *handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                             ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  std::string why;  // empty when loaded
};

void load(nccl_api &a) {
  for (const char *name : {"libnccl.so.2", "libnccl.so"}) {
    a.handle = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    if (a.handle != nullptr) break;
  }
  if (a.handle == nullptr) {
    const char *e = dlerror();
    a.why = std::string("NCCL is not available: ") + (e ? e : "libnccl.so.2 not found");
    return;
  }
  a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(a.handle, "ncclGetUniqueId"));
  a.comm_init_rank =
      reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(a.handle, "ncclCommInitRank"));
  a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(a.handle, "ncclCommDestroy"));
  a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(a.handle, "ncclAllReduce"));
  a.error_string =
      reinterpret_cast<decltype(a.error_string)>(dlsym(a.handle, "ncclGetErrorString"));
  if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_reduce ||
      !a.error_string)
    a.why = "libnccl.so.2 lacks an expected entry point";
}

nccl_api &api() {
  static nccl_api a;
  static std::once_flag once;
  std::call_once(once, load, std::ref(a));
  return a;
}

aut_status nccl_fail(ncclResult_t r, const char *what) {
  const char *text = api().error_string ? api().error_string(r) : "unknown";
  return aut::lib::fail(AUT_ERR_COMM, std::string(what) + ": " + text);
}

} // namespace

struct aut_comm {
  ncclComm_t comm = nullptr;
  bool owned = false;
  int device = -1;
};

extern "C" {

aut_status aut_comm_unique_id(void *id) {
  using namespace aut::lib;
  clear_error();
  if (id == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "id is NULL");
  nccl_api &a = api();
  if (!a.why.empty()) return fail(AUT_ERR_COMM, a.why);
  ncclUniqueId u;
  const ncclResult_t r = a.get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof u);
  return AUT_OK;
}

aut_status aut_comm_create(const void *id, int32_t nranks, int32_t rank, int32_t device,
                           aut_comm **out) {
  using namespace aut::lib;
  clear_error();
  if (id == nullptr || out == nullptr)
    return fail(AUT_ERR_INVALID_ARGUMENT, "id or out is NULL");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(AUT_ERR_INVALID_ARGUMENT, "rank must lie in [0, nranks)");
  nccl_api &a = api();
  if (!a.why.empty()) return fail(AUT_ERR_COMM, a.why);
  int previous = 0;
  AUT_CUDA_TRY(cudaGetDevice(&previous));
  AUT_CUDA_TRY(cudaSetDevice(device));
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof u);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = a.comm_init_rank(&comm, nranks, u, rank);
  cudaSetDevice(previous);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  aut_comm *c = new aut_comm;
  c->comm = comm;
  c->owned = true;
  c->device = device;
  *out = c;
  return AUT_OK;
}

aut_status aut_comm_wrap(void *nccl_comm, int32_t device, aut_comm **out) {
  using namespace aut::lib;
  clear_error();
  if (nccl_comm == nullptr || out == nullptr)
    return fail(AUT_ERR_INVALID_ARGUMENT, "communicator or out is NULL");
  nccl_api &a = api();
  if (!a.why.empty()) return fail(AUT_ERR_COMM, a.why);
  aut_comm *c = new aut_comm;
  c->comm = static_cast<ncclComm_t>(nccl_comm);
  c->owned = false;
  c->device = device;
  *out = c;
  return AUT_OK;
}

aut_status aut_comm_destroy(aut_comm *comm) {
  using namespace aut::lib;
  clear_error();
  if (comm == nullptr) return AUT_OK;
  aut_status st = AUT_OK;
  if (comm->owned) {
    const ncclResult_t r = api().comm_destroy(comm->comm);
    if (r != ncclSuccess) st = nccl_fail(r, "ncclCommDestroy");
  }
  delete comm;
  return st;
}

aut_status aut_comm_allreduce(aut_comm *comm, double *values, uint64_t count, void *stream) {
  using namespace aut::lib;
  clear_error();
  if (comm == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "communicator is NULL");
  if (count == 0) return AUT_OK;
  if (values == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "values is NULL");
  int previous = -1;
  if (comm->device >= 0) {
    AUT_CUDA_TRY(cudaGetDevice(&previous));
    if (previous != comm->device) AUT_CUDA_TRY(cudaSetDevice(comm->device));
  }
  const ncclResult_t r = api().all_reduce(values, values, static_cast<size_t>(count),
                                          ncclFloat64, ncclSum, comm->comm,
                                          static_cast<cudaStream_t>(stream));
  if (previous >= 0 && previous != comm->device) cudaSetDevice(previous);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return AUT_OK;
}

aut_status aut_dot_sharded(aut_comm *comm, aut_workspace *ws, int32_t format, int32_t layout,
                           int32_t accum, const void *x, const void *y, uint64_t n_local,
                           double *result, void *stream) {
  using namespace aut::lib;
  clear_error();
  if (comm == nullptr) return fail(AUT_ERR_INVALID_ARGUMENT, "communicator is NULL");
  if (ws != nullptr && comm->device >= 0 && ws->device != comm->device)
    return fail(AUT_ERR_INVALID_ARGUMENT, "workspace and communicator are on different devices");
  const aut_status st = aut_dot(ws, format, layout, accum, x, y, n_local, result, stream);
  if (st != AUT_OK) return st;
  return aut_comm_allreduce(comm, result, 1, stream);
}

} // extern "C"

// NCCL for tensor parallelism, loaded at run time.
//
// The library does not link NCCL: the first tensor-parallel call opens
// libnccl.so.2 with dlopen (in a process that already loaded NCCL, such as
// one running torch.distributed, that is the same library) and resolves the
// handful of functions it needs.  Only NCCL's public types come from nccl.h.
// The collectives run on the context's stream, so they are captured into the
// speculative step's CUDA graph like the kernels around them.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "tp.cuh"

namespace alm {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  std::string why;
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(sym("ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(sym("ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(sym("ncclCommDestroy"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(sym("ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(sym("ncclAllGather"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(sym("ncclGetErrorString"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_reduce && a.all_gather && a.error_string;
    if (!a.ok) a.why = "libnccl.so.2 lacks a required function";
  });
  return a;
}

int nccl_fail(ncclResult_t r, const char* what, std::string* err) {
  *err = std::string(what) + ": " + (api().error_string ? api().error_string(r) : "NCCL error");
  return 1;
}

}  // namespace

int tp_unique_id(unsigned char* out, std::string* err) {
  NcclApi& a = api();
  if (!a.ok) {
    *err = a.why;
    return 1;
  }
  ncclUniqueId id;
  const ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId", err);
  static_assert(sizeof(id.internal) == kTpIdBytes, "NCCL unique id size");
  for (int i = 0; i < kTpIdBytes; ++i) out[i] = static_cast<unsigned char>(id.internal[i]);
  return 0;
}

int tp_comm_init(int rank, int world, const unsigned char* id_bytes, void** comm, std::string* err) {
  NcclApi& a = api();
  if (!a.ok) {
    *err = a.why;
    return 1;
  }
  ncclUniqueId id;
  for (int i = 0; i < kTpIdBytes; ++i) id.internal[i] = static_cast<char>(id_bytes[i]);
  ncclComm_t c = nullptr;
  const ncclResult_t r = a.comm_init_rank(&c, world, id, rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank", err);
  *comm = c;
  return 0;
}

void tp_comm_destroy(void* comm) {
  if (comm && api().ok) api().comm_destroy(static_cast<ncclComm_t>(comm));
}

int tp_allreduce_sum_f32(void* comm, float* buf, size_t n, cudaStream_t st, std::string* err) {
  const ncclResult_t r = api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st);
  return r == ncclSuccess ? 0 : nccl_fail(r, "ncclAllReduce", err);
}

int tp_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank, cudaStream_t st,
                 std::string* err) {
  const ncclResult_t r =
      api().all_gather(send, recv, bytes_per_rank, ncclUint8, static_cast<ncclComm_t>(comm), st);
  return r == ncclSuccess ? 0 : nccl_fail(r, "ncclAllGather", err);
}

}  // namespace alm

// Tensor-parallel collectives: a sum all-reduce and an all-gather over NCCL,
// issued on the caller's stream so that they are recorded into the same CUDA
// graph as the kernels of a decode step.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or a path the caller
// gives), so the library has no link-time NCCL dependency and shares the NCCL
// that torch.distributed already loaded in the process.  Only NCCL's public
// C API is used: ncclGetUniqueId, ncclCommInitRank, ncclAllReduce,
// ncclAllGather, ncclCommDestroy, ncclGetErrorString, with the documented enum values
// ncclSum = 0, ncclFloat32 = 7, ncclBfloat16 = 9 and 128-byte unique ids.
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace cb {
namespace {

constexpr int kIdBytes = 128;
struct UniqueId {
  char internal[kIdBytes];
};

using GetUniqueIdFn = int (*)(UniqueId*);
using CommInitRankFn = int (*)(void**, int, UniqueId, int);
using AllReduceFn = int (*)(const void*, void*, size_t, int, int, void*, cudaStream_t);
using AllGatherFn = int (*)(const void*, void*, size_t, int, void*, cudaStream_t);
using CommDestroyFn = int (*)(void*);
using ErrorStringFn = const char* (*)(int);

struct Nccl {
  void* handle = nullptr;
  GetUniqueIdFn get_unique_id = nullptr;
  CommInitRankFn comm_init_rank = nullptr;
  AllReduceFn all_reduce = nullptr;
  AllGatherFn all_gather = nullptr;
  CommDestroyFn comm_destroy = nullptr;
  ErrorStringFn error_string = nullptr;
};

Nccl g_nccl;
std::mutex g_nccl_mutex;

int load_nccl(const char* path) {
  std::lock_guard<std::mutex> lock(g_nccl_mutex);
  if (g_nccl.handle != nullptr) return CB_OK;
  void* h = dlopen(path != nullptr && path[0] != '\0' ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) {
    set_error("cb_comm: cannot load NCCL (%s)", dlerror());
    return CB_ERR_INVALID;
  }
  Nccl n;
  n.handle = h;
  n.get_unique_id = reinterpret_cast<GetUniqueIdFn>(dlsym(h, "ncclGetUniqueId"));
  n.comm_init_rank = reinterpret_cast<CommInitRankFn>(dlsym(h, "ncclCommInitRank"));
  n.all_reduce = reinterpret_cast<AllReduceFn>(dlsym(h, "ncclAllReduce"));
  n.all_gather = reinterpret_cast<AllGatherFn>(dlsym(h, "ncclAllGather"));
  n.comm_destroy = reinterpret_cast<CommDestroyFn>(dlsym(h, "ncclCommDestroy"));
  n.error_string = reinterpret_cast<ErrorStringFn>(dlsym(h, "ncclGetErrorString"));
  if (!n.get_unique_id || !n.comm_init_rank || !n.all_reduce || !n.all_gather || !n.comm_destroy ||
      !n.error_string) {
    set_error("cb_comm: the loaded NCCL lacks a required symbol");
    dlclose(h);
    return CB_ERR_INVALID;
  }
  g_nccl = n;
  return CB_OK;
}

int nccl_status(int r, const char* what) {
  if (r == 0) return CB_OK;
  set_error("%s: NCCL error %d (%s)", what, r, g_nccl.error_string != nullptr ? g_nccl.error_string(r) : "?");
  return CB_ERR_CUDA;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_comm_load(const char* path) { return load_nccl(path); }

int cb_comm_unique_id(void* out, int bytes) {
  CB_REQUIRE(out != nullptr && bytes >= kIdBytes, "cb_comm_unique_id: needs a %d-byte buffer", kIdBytes);
  const int loaded = load_nccl(nullptr);
  if (loaded != CB_OK) return loaded;
  UniqueId id;
  const int r = nccl_status(g_nccl.get_unique_id(&id), "ncclGetUniqueId");
  if (r == CB_OK) std::memcpy(out, id.internal, kIdBytes);
  return r;
}

int cb_comm_init(const void* id, int bytes, int nranks, int rank, void** comm) {
  CB_REQUIRE(id != nullptr && bytes >= kIdBytes && comm != nullptr, "cb_comm_init: id and comm are required");
  CB_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "cb_comm_init: rank %d of %d", rank, nranks);
  const int loaded = load_nccl(nullptr);
  if (loaded != CB_OK) return loaded;
  UniqueId uid;
  std::memcpy(uid.internal, id, kIdBytes);
  *comm = nullptr;
  return nccl_status(g_nccl.comm_init_rank(comm, nranks, uid, rank), "ncclCommInitRank");
}

int cb_comm_destroy(void* comm) {
  if (comm == nullptr || g_nccl.handle == nullptr) return CB_OK;
  return nccl_status(g_nccl.comm_destroy(comm), "ncclCommDestroy");
}

int cb_all_reduce(void* comm, const void* src, void* dst, long long count, int dtype, cb_stream_t stream) {
  CB_REQUIRE(comm != nullptr && g_nccl.handle != nullptr, "cb_all_reduce: no communicator");
  CB_REQUIRE(count >= 0 && (count == 0 || (src != nullptr && dst != nullptr)), "cb_all_reduce: bad buffers");
  CB_REQUIRE(dtype == CB_F32 || dtype == CB_BF16, "cb_all_reduce: float32 or bfloat16 only");
  if (count == 0) return CB_OK;
  const int nccl_dtype = dtype == CB_F32 ? 7 : 9;  // ncclFloat32, ncclBfloat16
  return nccl_status(g_nccl.all_reduce(src, dst, static_cast<size_t>(count), nccl_dtype, /*ncclSum*/ 0, comm,
                                       static_cast<cudaStream_t>(stream)),
                     "ncclAllReduce");
}

int cb_all_gather(void* comm, const void* src, void* dst, long long count, int dtype, cb_stream_t stream) {
  CB_REQUIRE(comm != nullptr && g_nccl.handle != nullptr, "cb_all_gather: no communicator");
  CB_REQUIRE(count >= 0 && (count == 0 || (src != nullptr && dst != nullptr)), "cb_all_gather: bad buffers");
  CB_REQUIRE(dtype == CB_F32 || dtype == CB_BF16, "cb_all_gather: float32 or bfloat16 only");
  if (count == 0) return CB_OK;
  const int nccl_dtype = dtype == CB_F32 ? 7 : 9;  // ncclFloat32, ncclBfloat16
  return nccl_status(g_nccl.all_gather(src, dst, static_cast<size_t>(count), nccl_dtype, comm,
                                       static_cast<cudaStream_t>(stream)),
                     "ncclAllGather");
}

}  // extern "C"

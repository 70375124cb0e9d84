// One-shot all-reduce over NVLink peer memory (tensor parallel).
//
// The tensor-parallel decode sums the row-sharded O and down projections
// over the group after every layer: small messages (batch x hidden float32,
// 256 KB for Llama-3-8B at batch 16) whose cost is latency, not bandwidth.
// NCCL's ring / tree moves them in several dependent hops; here every rank
// writes its partial straight into every rank's exchange region over NVLink
// (plain stores through CUDA-IPC-mapped pointers), raises one flag per
// (block, source rank) in each region, waits -- bounded -- for the flags of
// all ranks in its own region, and sums the ranks' partials in rank order, so
// every rank computes the same float32 sums.  The residual add that follows
// the all-reduce in the graph (hidden + sum) can ride along.
//
// Exchange region of every rank (identical layout, one cudaMalloc each,
// shared by cudaIpcGetMemHandle / cudaIpcOpenMemHandle):
//   data   [2][ranks][max_count] float32   (two buffers by call parity)
//   flags  [kPeerBlocks][ranks] uint64     (the call number a source reached)
//   local  epoch (uint64), done counter (uint32): this rank's own state
//
// Calls are numbered 1, 2, ... (the epoch, read from device memory by every
// block, so a CUDA graph can replay the launch; the last block of a call
// advances it).  Call e writes data buffer e & 1.  Rank A writes buffer
// (e + 2) & 1 == e & 1 again only in call e + 2, after its call e + 1
// finished, which needed every rank's flags of call e + 1; a rank's call
// e + 1 starts after its whole call e finished reading (stream order).  So
// no rank overwrites a buffer another rank still reads, with two buffers.
//
// Waits are bounded (wait_ns, 10 s by default): a rank that does not arrive
// makes the others store CB_FLAG_WAIT_PEER in the caller's error flag and
// return; the host reads the flag after the step.  No TMA and no multicast:
// plain loads and stores only.
#include <cstring>
#include <vector>

#include "common.cuh"
#include "sync.cuh"

namespace cb {
namespace {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerBlocks = 32;
constexpr int kPeerThreads = 512;
constexpr int kIpcBytes = 64;  // sizeof(cudaIpcMemHandle_t)
// Default bound of a wait for the other ranks: long enough for the host-side
// skew between ranks (one rank still planning or capturing while another
// already waits), short of a hang.
constexpr unsigned long long kPeerWaitNs = 10ull * 1000000000ull;

struct PeerGroup {
  int ranks = 0, rank = 0;
  long long max_count = 0;
  long long data_bytes = 0, flag_bytes = 0, region_bytes = 0;
  char* local = nullptr;                 // this rank's region (cudaMalloc)
  char* regions[kPeerMaxRanks] = {};     // every rank's region as seen here (peers IPC-mapped)
  bool connected = false;
  unsigned long long wait_ns = kPeerWaitNs;
};

struct PeerArgs {
  char* regions[kPeerMaxRanks];
  int ranks, rank;
  long long max_count, data_bytes;
  const float* src;
  const void* residual;  // optional: out = residual + sum
  int residual_dtype;
  void* out;
  int out_dtype;
  long long count;
  int* error_flag;
  unsigned long long wait_ns;
};

__device__ __forceinline__ float* peer_data(char* region, long long max_count, int parity, int src_rank,
                                            int ranks) {
  return reinterpret_cast<float*>(region) + (static_cast<long long>(parity) * ranks + src_rank) * max_count;
}

__device__ __forceinline__ unsigned long long* peer_flags(char* region, long long data_bytes) {
  return reinterpret_cast<unsigned long long*>(region + data_bytes);
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kPeerThreads) peer_all_reduce_kernel(const PeerArgs a) {
  __shared__ unsigned long long s_epoch;
  __shared__ int s_ok;
  char* mine = a.regions[a.rank];
  unsigned long long* my_flags = peer_flags(mine, a.data_bytes);
  const int flag_words = kPeerBlocks * a.ranks;
  unsigned long long* epoch = my_flags + flag_words;
  unsigned int* done = reinterpret_cast<unsigned int*>(epoch + 1);
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile unsigned long long*>(epoch) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned long long e = s_epoch;
  const int parity = static_cast<int>(e & 1);
  // this block's elements: [lo, hi), a multiple of 4 long except the last
  const long long per = ((a.count + kPeerBlocks - 1) / kPeerBlocks + 3) / 4 * 4;
  const long long lo = per * blockIdx.x < a.count ? per * blockIdx.x : a.count;
  const long long hi = lo + per < a.count ? lo + per : a.count;
  // 16-byte pieces when src allows (lo is a multiple of 4 and every data buffer starts 16-byte aligned)
  const long long n4 = (reinterpret_cast<uintptr_t>(a.src) & 15) == 0 ? (hi - lo) / 4 : 0;

  // 1. push this rank's partial into every rank's buffer (destinations in rank order rotated by rank)
  for (int k = 0; k < a.ranks; ++k) {
    const int dst = (a.rank + k) % a.ranks;
    float* to = peer_data(a.regions[dst], a.max_count, parity, a.rank, a.ranks);
    for (long long t = threadIdx.x; t < n4; t += kPeerThreads)
      *reinterpret_cast<float4*>(to + lo + 4 * t) = *reinterpret_cast<const float4*>(a.src + lo + 4 * t);
    for (long long j = lo + 4 * n4 + threadIdx.x; j < hi; j += kPeerThreads) to[j] = a.src[j];
  }
  __syncthreads();
  // 2. one flag per destination: this block of this rank reached call e
  if (threadIdx.x < a.ranks) {
    __threadfence_system();
    st_release_sys(peer_flags(a.regions[threadIdx.x], a.data_bytes) + blockIdx.x * a.ranks + a.rank, e);
  }
  // 3. wait (bounded) until every rank's block blockIdx.x has written call e here
  if (threadIdx.x < a.ranks) {
    const unsigned long long* f = my_flags + blockIdx.x * a.ranks + threadIdx.x;
    uint64_t start = 0;
    bool ok = false;
    for (uint32_t it = 0; it < kWaitPolls; ++it) {
      if (ld_acquire_sys(f) >= e) {
        ok = true;
        break;
      }
      if ((it & 31u) == 31u) {
        const uint64_t now = global_ns();
        if (start == 0) start = now;
        else if (now - start > a.wait_ns) break;
      }
    }
    if (!ok) {
      s_ok = 0;
      if (a.error_flag != nullptr) atomicCAS(a.error_flag, 0, CB_FLAG_WAIT_PEER);
    }
  }
  __syncthreads();
  // 4. the sum in rank order (+ residual), the same on every rank
  if (s_ok) {
    for (long long i = lo + threadIdx.x; i < hi; i += kPeerThreads) {
      float acc = __ldcg(peer_data(mine, a.max_count, parity, 0, a.ranks) + i);
      for (int r = 1; r < a.ranks; ++r) acc = __fadd_rn(acc, __ldcg(peer_data(mine, a.max_count, parity, r, a.ranks) + i));
      if (a.residual != nullptr) acc = __fadd_rn(load_as_f32(a.residual, i, a.residual_dtype), acc);
      store_from_f32(a.out, i, a.out_dtype, acc);
    }
  }
  // 5. the last block of this rank's call advances the epoch for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == kPeerBlocks - 1) {
      *done = 0u;
      *reinterpret_cast<volatile unsigned long long*>(epoch) = e;
      __threadfence();
    }
  }
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CB_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return CB_ERR_CUDA;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_peer_create(int ranks, int rank, long long max_count, void** group, void* handle_out, int handle_bytes) {
  CB_REQUIRE(group != nullptr && handle_out != nullptr && handle_bytes >= kIpcBytes,
             "cb_peer_create: group and a %d-byte handle buffer are required", kIpcBytes);
  CB_REQUIRE(ranks >= 1 && ranks <= kPeerMaxRanks && rank >= 0 && rank < ranks, "cb_peer_create: rank %d of %d",
             rank, ranks);
  CB_REQUIRE(max_count > 0 && max_count % 4 == 0 && max_count <= (1LL << 28),
             "cb_peer_create: max_count must be a positive multiple of 4 (got %lld)", max_count);
  *group = nullptr;
  auto* g = new PeerGroup();
  g->ranks = ranks;
  g->rank = rank;
  g->max_count = max_count;
  g->data_bytes = 2LL * ranks * max_count * 4;
  g->flag_bytes = (static_cast<long long>(kPeerBlocks) * ranks + 2) * 8;
  g->region_bytes = (g->data_bytes + g->flag_bytes + 4095) / 4096 * 4096;
  int r = cuda_status(cudaMalloc(&g->local, static_cast<size_t>(g->region_bytes)), "cb_peer_create: cudaMalloc");
  if (r == CB_OK) r = cuda_status(cudaMemset(g->local, 0, static_cast<size_t>(g->region_bytes)), "cb_peer_create");
  cudaIpcMemHandle_t h;
  if (r == CB_OK) r = cuda_status(cudaIpcGetMemHandle(&h, g->local), "cb_peer_create: cudaIpcGetMemHandle");
  if (r != CB_OK) {
    if (g->local != nullptr) cudaFree(g->local);
    delete g;
    return r;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == kIpcBytes, "IPC handle size");
  std::memcpy(handle_out, &h, kIpcBytes);
  g->regions[rank] = g->local;
  *group = g;
  return CB_OK;
}

int cb_peer_connect(void* group, const void* handles, int handle_bytes) {
  CB_REQUIRE(group != nullptr && handles != nullptr && handle_bytes == kIpcBytes,
             "cb_peer_connect: a group and its ranks' %d-byte handles are required", kIpcBytes);
  auto* g = static_cast<PeerGroup*>(group);
  CB_REQUIRE(!g->connected, "cb_peer_connect: already connected");
  const char* all = static_cast<const char*>(handles);
  for (int p = 0; p < g->ranks; ++p) {
    if (p == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, all + static_cast<size_t>(p) * kIpcBytes, kIpcBytes);
    void* mapped = nullptr;
    const int r = cuda_status(cudaIpcOpenMemHandle(&mapped, h, cudaIpcMemLazyEnablePeerAccess),
                              "cb_peer_connect: cudaIpcOpenMemHandle");
    if (r != CB_OK) {
      for (int q = 0; q < p; ++q)
        if (q != g->rank && g->regions[q] != nullptr) {
          cudaIpcCloseMemHandle(g->regions[q]);
          g->regions[q] = nullptr;
        }
      return r;
    }
    g->regions[p] = static_cast<char*>(mapped);
  }
  g->connected = true;
  return CB_OK;
}

int cb_peer_set_wait(void* group, long long wait_ns) {
  CB_REQUIRE(group != nullptr && wait_ns > 0, "cb_peer_set_wait: a group and a positive limit are required");
  static_cast<PeerGroup*>(group)->wait_ns = static_cast<unsigned long long>(wait_ns);
  return CB_OK;
}

int cb_peer_max_count(void* group, long long* count) {
  CB_REQUIRE(group != nullptr && count != nullptr, "cb_peer_max_count: null pointer");
  *count = static_cast<PeerGroup*>(group)->max_count;
  return CB_OK;
}

int cb_peer_all_reduce(void* group, const float* src, void* out, int out_dtype, const void* residual,
                       int residual_dtype, long long count, int* error_flag, cb_stream_t stream) {
  CB_REQUIRE(group != nullptr, "cb_peer_all_reduce: no group");
  auto* g = static_cast<PeerGroup*>(group);
  CB_REQUIRE(g->connected || g->ranks == 1, "cb_peer_all_reduce: the group is not connected");
  CB_REQUIRE(count >= 0 && count <= g->max_count, "cb_peer_all_reduce: %lld elements exceed the group's %lld",
             count, g->max_count);
  CB_REQUIRE(out_dtype == CB_F32 || out_dtype == CB_BF16, "cb_peer_all_reduce: float32 or bfloat16 output");
  CB_REQUIRE(residual == nullptr || residual_dtype == CB_F32 || residual_dtype == CB_BF16,
             "cb_peer_all_reduce: float32 or bfloat16 residual");
  if (count == 0) return CB_OK;
  CB_REQUIRE(src != nullptr && out != nullptr, "cb_peer_all_reduce: null buffer");
  PeerArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int p = 0; p < g->ranks; ++p) a.regions[p] = g->regions[p];
  a.ranks = g->ranks;
  a.rank = g->rank;
  a.max_count = g->max_count;
  a.data_bytes = g->data_bytes;
  a.src = src;
  a.residual = residual;
  a.residual_dtype = residual_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.count = count;
  a.error_flag = error_flag;
  a.wait_ns = g->wait_ns;
  peer_all_reduce_kernel<<<kPeerBlocks, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("cb_peer_all_reduce");
}

int cb_peer_destroy(void* group) {
  if (group == nullptr) return CB_OK;
  auto* g = static_cast<PeerGroup*>(group);
  int r = CB_OK;
  for (int p = 0; p < g->ranks; ++p) {
    if (p == g->rank || g->regions[p] == nullptr) continue;
    const int c = cuda_status(cudaIpcCloseMemHandle(g->regions[p]), "cb_peer_destroy: cudaIpcCloseMemHandle");
    if (r == CB_OK) r = c;
  }
  if (g->local != nullptr) {
    const int c = cuda_status(cudaFree(g->local), "cb_peer_destroy: cudaFree");
    if (r == CB_OK) r = c;
  }
  delete g;
  return r;
}

}  // extern "C"

// Shared pieces of the tcgen05 kernels (cb_gemm_tc, cb_sdpa_tc): TMA tile
// loads, shared-memory matrix descriptors for 128-byte-swizzled K-major bf16
// tiles, MMA issue/commit, TMEM loads, bounded mbarrier waits and tensor-map
// encoding.
//
// Tile convention: a K-major operand tile is stored as "chunks" of 64 bf16
// (one 128-byte swizzle atom) along K; one chunk of `rows` rows is rows x 128
// bytes, 8-row groups 1024 bytes apart, written by TMA with SWIZZLE_128B
// (box {64, rows}) or by threads with the same XOR pattern (swizzle_offset).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sync.cuh"

namespace cb {
namespace tc {

constexpr int kChunk = 64;          // bf16 elements per swizzle atom row (128 bytes)
constexpr int kChunkRowBytes = 128;
constexpr int kUmmaK = 16;          // K of one kind::f16 MMA

// bf16 x bf16 -> float32, M x N, A and B K-major (tcgen05 instruction descriptor).
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4)                                  // D format: float32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Shared-memory matrix descriptor of a K-major chunk with SWIZZLE_128B: rows
// of 128 bytes, 8-row groups 1024 bytes apart.  The chunk base must be
// 1024-byte aligned; a K offset inside the atom is added to the start address.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t addr = smem_addr(tile);
  return ((addr >> 4) & 0x3FFFull)  // start address
         | (1ull << 16)             // leading byte offset (unused for this layout)
         | (64ull << 32)            // stride byte offset: 1024 B
         | (1ull << 46)             // descriptor version (sm_100)
         | (2ull << 61);            // SWIZZLE_128B
}

// Byte offset of the 16-byte group `g` (0..7) of row `r` inside a swizzled chunk.
__device__ __forceinline__ int swizzle_offset(int r, int g) { return r * kChunkRowBytes + ((g ^ (r & 7)) << 4); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

// Arrives on `bar` once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Makes this thread's generic-proxy shared-memory stores visible to the async
// proxy (the tensor cores reading an operand these threads wrote).
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, int cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, int cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

// 16 consecutive float32 columns of this thread's TMEM lane (warp-wide).
__device__ __forceinline__ void tmem_load16(uint32_t taddr, float* out) {
  uint32_t v[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  // the wait names the registers, so no use of them moves above it
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = __uint_as_float(v[i]);
}

// 32 consecutive float32 columns of this thread's TMEM lane (warp-wide),
// without waiting: several loads can be in flight before one tmem_wait_ld().
__device__ __forceinline__ void tmem_load32_nowait(uint32_t taddr, float* out) {
  uint32_t v[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(v[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// One float32 column of this thread's TMEM lane (warp-wide): store (then
// tmem_wait_st before signalling a reader) and load (waits for the value).
__device__ __forceinline__ void tmem_store1(uint32_t taddr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(__float_as_uint(v)) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float tmem_load1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(taddr) : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(v)::"memory");
  return __uint_as_float(v);
}
// After tmem_wait_ld(): ties the loaded registers to a point after the wait,
// so the compiler cannot move their first use above it.
template <int N>
__device__ __forceinline__ void reg_fence(float* x) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+f"(x[i]));
}

// mbarrier wait that also gives up once *abort != 0 (bounded like mbar_wait;
// no suspend hint, so a waiter resumes as soon as the phase completes).
// The clock (%globaltimer) is read only every 64 polls, starting at the first
// such read: a read costs about half a microsecond, and a wait whose phase has
// already completed (a ring stage that landed) must cost one poll.
__device__ inline bool wait_or_abort(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  uint64_t start = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait_short(bar, parity)) return true;
    if ((i & 63u) == 63u) {
      if (*abort != 0) return false;
      const uint64_t now = global_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitNs) return false;
    }
  }
  return false;
}

// Bounded wait without an abort flag (drains, teardown).
__device__ inline bool wait_short(uint64_t* bar, uint32_t parity) {
  uint64_t start = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait_short(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      const uint64_t now = global_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitNs) return false;
    }
  }
  return false;
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map: rows x cols (cols contiguous), row stride ld elements,
// boxes of 64 columns x box_rows rows, 128-byte swizzle, zero fill outside.
inline bool make_map(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunk), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace tc
}  // namespace cb

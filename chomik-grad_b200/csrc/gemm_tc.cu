// Tensor-core GEMM for sm_100a: cb_gemm_tc, C (m x n, float32) = A (m x k) x B^T,
// B the (n x k) bf16 weight of a Linear layer.
//
// One block of 128 threads per 128 x BN output tile (BN = 256 or 128):
//  * thread 0 streams K in 64-element steps -- one 128-byte swizzle atom of
//    bf16 -- with TMA (cp.async.bulk.tensor, SWIZZLE_128B) into a ring of
//    shared-memory stages: A's plane(s) and B per stage, completion counted
//    on an mbarrier per stage;
//  * thread 32 issues tcgen05.mma (kind::f16, bf16 x bf16 -> float32, M=128,
//    N=BN, K=16 per instruction) from those stages into a float32
//    accumulator in TMEM, and tcgen05.commit frees each stage when its MMAs
//    have read it;
//  * after the last commit all four warps read the accumulator back with
//    tcgen05.ld (warp w owns TMEM lanes 32w..32w+31 = tile rows) and store it.
// A float32 A enters as two bf16 planes (hi = bf16(a), lo = bf16(a - hi)),
// split by a pre-pass; each K step then issues the MMAs of both planes into
// the same accumulator.
//
// Every wait is bounded (sync.cuh): on a timeout the kernel records an error,
// lets its issued copies land, lets issued MMAs finish, frees its TMEM and
// returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sync.cuh"

namespace cb {
namespace {

constexpr int kBM = 128;              // tile rows = TMEM lanes
constexpr int kBK = 64;               // K per stage: one 128-byte swizzle atom of bf16
constexpr int kUmmaK = 16;            // K of one kind::f16 MMA
constexpr int kGemmThreads = 128;
constexpr int kStageBudget = 192 * 1024;

template <int BN, int NA>
struct GemmShape {
  static constexpr int kA = kBM * kBK * 2;  // one A plane of a stage
  static constexpr int kB = BN * kBK * 2;
  static constexpr int kStage = NA * kA + kB;
  static constexpr int kStages = kStageBudget / kStage;
  static constexpr int kSmem = kStages * kStage + 1024;  // + 1024-byte alignment of the swizzled tiles
  static_assert(kStages >= 2, "at least double buffering");
};

// bf16 x bf16 -> float32, M = 128, N = BN, A and B K-major (tcgen05 instruction descriptor).
template <int BN>
__host__ __device__ constexpr uint32_t umma_idesc() {
  return (1u << 4)                                  // D format: float32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(BN >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(kBM >> 4) << 24); // M / 16
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with
// SWIZZLE_128B: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t addr = smem_addr(tile);
  return ((addr >> 4) & 0x3FFFull)  // start address
         | (1ull << 16)             // leading byte offset (unused for this layout)
         | (64ull << 32)            // stride byte offset: 1024 B
         | (1ull << 46)             // descriptor version (sm_100)
         | (2ull << 61);            // SWIZZLE_128B
}

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

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive float32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_load16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// mbarrier wait that also gives up once *abort != 0.
__device__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  const uint64_t start = global_ns();
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && (*abort != 0 || global_ns() - start > kWaitNs)) return false;
  }
  return false;
}

template <int BN, int NA>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                   const __grid_constant__ CUtensorMap map_b, float* __restrict__ c, long long ldc, int m, int k,
                   int* error_flag) {
  using G = GemmShape<BN, NA>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[G::kStages];
  __shared__ __align__(8) uint64_t empty[G::kStages];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
  const int kblocks = k / kBK;

  if (warp == 0) {  // TMEM for the accumulator: BN float32 columns x 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(&acc_full, 1);
    mbar_fence_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int kb = 0;
    for (; kb < kblocks; ++kb) {
      const int s = kb % G::kStages, round = kb / G::kStages;
      if (round > 0 && !wait_or_abort(empty + s, static_cast<uint32_t>((round - 1) & 1), &abort_flag)) {
        if (error_flag != nullptr) atomicCAS(error_flag, 0, CB_FLAG_WAIT_SLOT);
        abort_flag = 1;
        break;
      }
      unsigned char* st = smem + s * G::kStage;
      mbar_arrive_expect_tx(full + s, static_cast<uint32_t>(G::kStage));
      tma_load_2d(st, &map_a, kb * kBK, m0, full + s);
      if (NA == 2) tma_load_2d(st + G::kA, &map_a2, kb * kBK, m0, full + s);
      tma_load_2d(st + NA * G::kA, &map_b, kb * kBK, n0, full + s);
    }
    // drain: the copies of the last round of every stage land before we go on
    for (int t = kb - 1; t >= 0 && t >= kb - G::kStages; --t) {
      if (!mbar_wait(full + t % G::kStages, static_cast<uint32_t>((t / G::kStages) & 1))) {
        if (error_flag != nullptr) atomicCAS(error_flag, 0, CB_FLAG_WAIT_DRAIN);
        break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = umma_idesc<BN>();
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % G::kStages, round = kb / G::kStages;
      if (!wait_or_abort(full + s, static_cast<uint32_t>(round & 1), &abort_flag)) {
        if (error_flag != nullptr) atomicCAS(error_flag, 0, CB_FLAG_WAIT_DATA);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const unsigned char* st = smem + s * G::kStage;
#pragma unroll
      for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
        const uint64_t db = sw128_desc(st + NA * G::kA + kk * kUmmaK * 2);
#pragma unroll
        for (int pl = 0; pl < NA; ++pl)
          umma_bf16(tmem, sw128_desc(st + pl * G::kA + kk * kUmmaK * 2), db, idesc,
                    (kb | kk | pl) != 0 ? 1u : 0u);
      }
      umma_commit(empty + s);  // the stage is free once these MMAs have read it
    }
    umma_commit(&acc_full);  // every issued MMA has completed (also after an abort)
  }
  __syncwarp();

  // ---- epilogue: TMEM -> registers -> global ----
  bool ok = wait_or_abort(&acc_full, 0u, &abort_flag) || mbar_wait(&acc_full, 0u);
  ok = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int*>(&abort_flag) == 0);
  tc_fence_after();
  if (ok) {
    const int row = m0 + warp * 32 + lane;
    float* crow = c + static_cast<long long>(row) * ldc + n0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t v[16];
      tmem_load16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(c0), v);
      if (row < m) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<float4*>(crow + c0)[q] =
              make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]), __uint_as_float(v[4 * q + 2]),
                          __uint_as_float(v[4 * q + 3]));
      }
    }
  } else if (threadIdx.x == 0 && error_flag != nullptr) {
    atomicCAS(error_flag, 0, CB_FLAG_WAIT_DATA);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

// float32 (or strided bf16) A -> bf16 planes hi = bf16(a), lo = bf16(a - hi).
__global__ void split_planes_kernel(const void* a, int a_dtype, long long lda, long long m, long long k,
                                    __nv_bfloat16* hi, __nv_bfloat16* lo) {
  const long long total = m * k;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / k, col = i % k;
    const float x = load_as_f32(a, r * lda + col, a_dtype);
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    hi[i] = h;
    if (lo != nullptr) lo[i] = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(h)));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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
// boxes of 64 columns x box_rows rows, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// bf16 A usable by TMA as it is (no plane copy).
bool a_direct(const cb_gemm_args& g) {
  return g.a_dtype == CB_BF16 && aligned16(g.a) && g.lda % 8 == 0 && g.lda >= g.k;
}

template <int BN, int NA>
cudaError_t launch_gemm(const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap& mb, const cb_gemm_args& g,
                        cudaStream_t s) {
  using G = GemmShape<BN, NA>;
  auto kernel = gemm_tc_kernel<BN, NA>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>(g.n / BN), static_cast<unsigned>((g.m + kBM - 1) / kBM));
  kernel<<<grid, kGemmThreads, G::kSmem, s>>>(ma, ma2, mb, g.c, g.ldc, static_cast<int>(g.m), static_cast<int>(g.k),
                                                g.error_flag);
  return cudaGetLastError();
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

long long cb_gemm_tc_scratch(const cb_gemm_args* g) {
  if (g == nullptr || g->m <= 0 || g->k <= 0) return 0;
  if (g->a_dtype == CB_F32) return 2 * g->m * g->k * 2;
  return a_direct(*g) ? 0 : g->m * g->k * 2;
}

int cb_gemm_tc(const cb_gemm_args* g, cb_stream_t stream) {
  CB_REQUIRE(g != nullptr && g->a != nullptr && g->b != nullptr && g->c != nullptr, "gemm: a, b and c are required");
  CB_REQUIRE(g->m > 0 && g->n > 0 && g->k > 0, "gemm: empty problem");
  CB_REQUIRE(g->k % kBK == 0, "gemm: k=%lld must be a multiple of %d", g->k, kBK);
  CB_REQUIRE(g->n % 128 == 0, "gemm: n=%lld must be a multiple of 128", g->n);
  CB_REQUIRE(g->m < 65535LL * kBM && g->k < (1LL << 31), "gemm: problem too large");
  CB_REQUIRE(g->a_dtype == CB_BF16 || g->a_dtype == CB_F32, "gemm: a must be bf16 or float32");
  CB_REQUIRE(aligned16(g->b) && g->ldb % 8 == 0 && g->ldb >= g->k, "gemm: b must be 16-byte aligned rows");
  CB_REQUIRE(aligned16(g->c) && g->ldc % 4 == 0 && g->ldc >= g->n, "gemm: c must be 16-byte aligned rows");
  const bool split = g->a_dtype == CB_F32;
  const bool direct = a_direct(*g);
  CB_REQUIRE(direct || (g->a_split != nullptr && aligned16(g->a_split)), "gemm: a needs %lld bytes of a_split",
             cb_gemm_tc_scratch(g));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* a_hi = g->a;
  const void* a_lo = nullptr;
  long long lda = g->lda;
  if (!direct) {
    __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(g->a_split);
    __nv_bfloat16* lo = split ? hi + g->m * g->k : nullptr;
    const long long total = g->m * g->k;
    const int blocks = static_cast<int>((total + 255) / 256 < 65535 ? (total + 255) / 256 : 65535);
    split_planes_kernel<<<blocks, 256, 0, s>>>(g->a, g->a_dtype, g->lda, g->m, g->k, hi, lo);
    a_hi = hi;
    a_lo = lo;
    lda = g->k;
  }
  const int bn = g->n % 256 == 0 ? 256 : 128;
  CUtensorMap ma, ma2, mb;
  CB_REQUIRE(make_map(&ma, a_hi, g->m, g->k, lda, kBM) && make_map(&mb, g->b, g->n, g->k, g->ldb, bn) &&
                 (a_lo == nullptr || make_map(&ma2, a_lo, g->m, g->k, lda, kBM)),
             "gemm: tensor map encoding failed");
  if (a_lo == nullptr) ma2 = ma;
  cudaError_t e;
  if (bn == 256)
    e = split ? launch_gemm<256, 2>(ma, ma2, mb, *g, s) : launch_gemm<256, 1>(ma, ma2, mb, *g, s);
  else
    e = split ? launch_gemm<128, 2>(ma, ma2, mb, *g, s) : launch_gemm<128, 1>(ma, ma2, mb, *g, s);
  if (e != cudaSuccess) {
    set_error("cb_gemm_tc: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_gemm_tc");
}

}  // extern "C"

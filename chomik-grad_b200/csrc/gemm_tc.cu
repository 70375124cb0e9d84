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
#include "tc_core.cuh"

namespace cb {
namespace {

using namespace tc;

constexpr int kBM = 128;              // tile rows = TMEM lanes
constexpr int kBK = kChunk;           // K per stage: one 128-byte swizzle atom of bf16
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

// Tile order: groups of kGroupM row tiles; inside a group the row tile varies
// fastest, so the blocks resident at one time share a few B (weight) tiles and
// a group's A rows, and each weight tile is read from HBM about once per group.
constexpr int kGroupM = 16;

__device__ __forceinline__ void tile_of(int t, int tiles_m, int tiles_n, int* tm, int* tn) {
  const int per_group = kGroupM * tiles_n;
  const int first = (t / per_group) * kGroupM;
  const int rows = min(tiles_m - first, kGroupM);
  const int r = t % per_group;
  *tm = first + r % rows;
  *tn = r / rows;
}

template <int BN, int NA>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                   const __grid_constant__ CUtensorMap map_b, float* __restrict__ c, long long ldc, int m, int n,
                   int k, int* error_flag) {
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
  int tm, tn;
  tile_of(blockIdx.x, (m + kBM - 1) / kBM, (n + BN - 1) / BN, &tm, &tn);
  const int m0 = tm * kBM, n0 = tn * BN;
  const int kblocks = (k + kBK - 1) / kBK;  // the tensor maps zero-fill K past k

  if (warp == 0) tmem_alloc(&tmem_base, BN);  // the accumulator: BN float32 columns x 128 lanes
  if (threadIdx.x == 32) {
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(&acc_full, 1);
    mbar_fence_init();
    abort_flag = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
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
      if (!wait_short(full + t % G::kStages, static_cast<uint32_t>((t / G::kStages) & 1))) {
        if (error_flag != nullptr) atomicCAS(error_flag, 0, CB_FLAG_WAIT_DRAIN);
        break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16(kBM, BN);
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % G::kStages, round = kb / G::kStages;
      if (!wait_or_abort(full + s, static_cast<uint32_t>(round & 1), &abort_flag)) {
        if (error_flag != nullptr) atomicCAS(error_flag, 0, CB_FLAG_WAIT_DATA);
        abort_flag = 1;
        break;
      }
      fence_after();
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
  bool ok = wait_or_abort(&acc_full, 0u, &abort_flag) || wait_short(&acc_full, 0u);
  ok = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int*>(&abort_flag) == 0);
  fence_after();
  if (ok) {
    const int row = m0 + warp * 32 + lane;
    float* crow = c + static_cast<long long>(row) * ldc + n0;
    const int cols = min(BN, n - n0);  // a multiple of 4
#pragma unroll 1
    for (int c0 = 0; c0 < cols; c0 += 16) {
      float v[16];
      tmem_load16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(c0), v);
      if (row < m) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (c0 + 4 * q < cols)
            reinterpret_cast<float4*>(crow + c0)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
  } else if (threadIdx.x == 0 && error_flag != nullptr) {
    atomicCAS(error_flag, 0, CB_FLAG_WAIT_DATA);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, BN);
}

// float32 (or strided bf16) A -> bf16 planes hi = bf16(a), lo = bf16(a - hi),
// rows of k elements.  One block per row; float4 loads when the row allows.
__global__ void split_planes_kernel(const void* a, int a_dtype, long long lda, long long k, __nv_bfloat16* hi,
                                    __nv_bfloat16* lo) {
  const long long r = blockIdx.x;
  __nv_bfloat16* hrow = hi + r * k;
  __nv_bfloat16* lrow = lo != nullptr ? lo + r * k : nullptr;
  const bool vec = a_dtype == CB_F32 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && lda % 4 == 0;
  if (vec) {
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(a) + r * lda);
    for (long long q = threadIdx.x; q < k / 4; q += blockDim.x) {
      const float4 x = src[q];
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(x.x, x.y), h23 = __floats2bfloat162_rn(x.z, x.w);
      reinterpret_cast<__nv_bfloat162*>(hrow)[2 * q] = h01;
      reinterpret_cast<__nv_bfloat162*>(hrow)[2 * q + 1] = h23;
      if (lrow != nullptr) {
        const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
        reinterpret_cast<__nv_bfloat162*>(lrow)[2 * q] =
            __floats2bfloat162_rn(__fsub_rn(x.x, f01.x), __fsub_rn(x.y, f01.y));
        reinterpret_cast<__nv_bfloat162*>(lrow)[2 * q + 1] =
            __floats2bfloat162_rn(__fsub_rn(x.z, f23.x), __fsub_rn(x.w, f23.y));
      }
    }
    return;
  }
  for (long long col = threadIdx.x; col < k; col += blockDim.x) {
    const float x = load_as_f32(a, r * lda + col, a_dtype);
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    hrow[col] = h;
    if (lrow != nullptr) lrow[col] = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(h)));
  }
}

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
  const long long tiles = ((g.n + BN - 1) / BN) * ((g.m + kBM - 1) / kBM);
  kernel<<<static_cast<unsigned>(tiles), kGemmThreads, G::kSmem, s>>>(
      ma, ma2, mb, g.c, g.ldc, static_cast<int>(g.m), static_cast<int>(g.n), static_cast<int>(g.k), g.error_flag);
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
  CB_REQUIRE(g->k % 8 == 0, "gemm: k=%lld must be a multiple of 8", g->k);
  CB_REQUIRE(g->n % 4 == 0, "gemm: n=%lld must be a multiple of 4", g->n);
  CB_REQUIRE(g->m < (1LL << 31) && g->n < (1LL << 31) && g->k < (1LL << 31) &&
                 ((g->m + kBM - 1) / kBM) * ((g->n + 127) / 128) < (1LL << 31),
             "gemm: problem too large");
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
    split_planes_kernel<<<static_cast<unsigned>(g->m), 256, 0, s>>>(g->a, g->a_dtype, g->lda, g->k, hi, lo);
    a_hi = hi;
    a_lo = lo;
    lda = g->k;
  }
  // 256-wide tiles unless 128 wastes less of the last column tile
  const int bn = (g->n + 255) / 256 * 256 - g->n <= (g->n + 127) / 128 * 128 - g->n ? 256 : 128;
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

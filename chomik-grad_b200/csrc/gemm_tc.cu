// Tensor-core GEMM for sm_100a: cb_gemm_tc / cb_gemm_tc_multi,
// C (m x n, float32) = A (m x k) x B^T, B the (n x k) bf16 weight of a Linear
// layer (chomikgrad/llama.py:275-277), with three epilogues:
//  * store, for up to three weights that share A (q/k/v of a prefill layer):
//    one launch, its tiles the concatenation of every weight's tiles;
//  * residual: C = R + A B^T (the residual add after the O and down
//    projections, llama.py:529-535), added in float32 before the store;
//  * SwiGLU: two weights (gate, up) computed on the same output tile into two
//    TMEM accumulators, stored as silu(g) * u = g / (1 + exp(-g)) * u
//    (llama.py:289-291, 371-380) -- the gate and up matrices are never
//    written.
//
// One block of 128 threads per 128 x BN output tile (BN = 256 or 128):
//  * thread 0 streams K in 64-element steps -- one 128-byte swizzle atom of
//    bf16 -- with TMA (cp.async.bulk.tensor, SWIZZLE_128B) into a ring of
//    shared-memory stages: A's plane(s) and B's (two for SwiGLU) per stage,
//    completion counted on an mbarrier per stage;
//  * thread 32 issues tcgen05.mma (kind::f16, bf16 x bf16 -> float32, M=128,
//    N=BN, K=16 per instruction) from those stages into float32
//    accumulators in TMEM, and tcgen05.commit frees each stage when its MMAs
//    have read it;
//  * after the last commit all four warps read the accumulators back with
//    tcgen05.ld (warp w owns TMEM lanes 32w..32w+31 = tile rows), apply the
//    epilogue and store.
// A float32 A enters as two bf16 planes (hi = bf16(a), lo = bf16(a - hi)),
// split by a pre-pass; each K step then issues the MMAs of both planes into
// the same accumulator.
//
// Every wait is bounded (sync.cuh): on a timeout the kernel records an error,
// lets its issued copies land, lets issued MMAs finish, frees its TMEM and
// returns.
#include "norm.cuh"
#include "tc_core.cuh"

namespace cb {
namespace {

using namespace tc;

constexpr int kBM = 128;              // tile rows = TMEM lanes
constexpr int kBK = kChunk;           // K per stage: one 128-byte swizzle atom of bf16
constexpr int kGemmThreads = 128;
constexpr int kStageBudget = 192 * 1024;

enum { kStore = 0, kResidual = 1, kSwiglu = 2 };

template <int BN, int NA, int MODE>
struct GemmShape {
  static constexpr int kW = MODE == kSwiglu ? 2 : 1;  // weight chunks per stage
  static constexpr int kA = kBM * kBK * 2;            // one A plane of a stage
  static constexpr int kB = BN * kBK * 2;
  static constexpr int kStage = NA * kA + kW * kB;
  static constexpr int kStages = kStageBudget / kStage;
  static constexpr int kSmem = kStages * kStage + 1024;  // + 1024-byte alignment of the swizzled tiles
  static constexpr int kTmemCols = kW * BN;
  static_assert(kStages >= 2, "at least double buffering");
};

struct GemmParams {
  float* c[3];
  long long ldc[3];
  int n[3];        // output columns of each weight
  int tiles_n[3];  // BN-wide column tiles of each weight (store: 1..3 weights; else 1)
  int n_seg;
  int m, k;
  const float* residual;
  long long ldr;
  int* error_flag;
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

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(expf(-g), 1.0f)), u);
}

template <int BN, int NA, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                   const __grid_constant__ CUtensorMap map_b0, const __grid_constant__ CUtensorMap map_b1,
                   const __grid_constant__ CUtensorMap map_b2, const __grid_constant__ GemmParams p) {
  using G = GemmShape<BN, NA, MODE>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[G::kStages];
  __shared__ __align__(8) uint64_t empty[G::kStages];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (p.m + kBM - 1) / kBM;
  int t = blockIdx.x, seg = 0;
  while (seg + 1 < p.n_seg && t >= tiles_m * p.tiles_n[seg]) t -= tiles_m * p.tiles_n[seg++];
  int tm, tn;
  tile_of(t, tiles_m, p.tiles_n[seg], &tm, &tn);
  const int m0 = tm * kBM, n0 = tn * BN;
  const int kblocks = (p.k + kBK - 1) / kBK;  // the tensor maps zero-fill K past k
  const CUtensorMap* mb = seg == 0 ? &map_b0 : seg == 1 ? &map_b1 : &map_b2;

  if (warp == 0) tmem_alloc(&tmem_base, G::kTmemCols);  // the accumulator(s): BN float32 columns x 128 lanes
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
        if (p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_SLOT);
        abort_flag = 1;
        break;
      }
      unsigned char* st = smem + s * G::kStage;
      mbar_arrive_expect_tx(full + s, static_cast<uint32_t>(G::kStage));
      tma_load_2d(st, &map_a, kb * kBK, m0, full + s);
      if (NA == 2) tma_load_2d(st + G::kA, &map_a2, kb * kBK, m0, full + s);
      tma_load_2d(st + NA * G::kA, MODE == kSwiglu ? &map_b0 : mb, kb * kBK, n0, full + s);
      if (MODE == kSwiglu) tma_load_2d(st + NA * G::kA + G::kB, &map_b1, kb * kBK, n0, full + s);
    }
    // drain: the copies of the last round of every stage land before we go on
    for (int q = kb - 1; q >= 0 && q >= kb - G::kStages; --q) {
      if (!wait_short(full + q % G::kStages, static_cast<uint32_t>((q / G::kStages) & 1))) {
        if (p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_DRAIN);
        break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16(kBM, BN);
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % G::kStages, round = kb / G::kStages;
      if (!wait_or_abort(full + s, static_cast<uint32_t>(round & 1), &abort_flag)) {
        if (p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_DATA);
        abort_flag = 1;
        break;
      }
      fence_after();
      const unsigned char* st = smem + s * G::kStage;
#pragma unroll
      for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
#pragma unroll
        for (int w = 0; w < G::kW; ++w) {
          const uint64_t db = sw128_desc(st + NA * G::kA + w * G::kB + kk * kUmmaK * 2);
#pragma unroll
          for (int pl = 0; pl < NA; ++pl)
            umma_bf16(tmem + static_cast<uint32_t>(w * BN), sw128_desc(st + pl * G::kA + kk * kUmmaK * 2), db, idesc,
                      (kb | kk | pl) != 0 ? 1u : 0u);
        }
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
    float* crow = p.c[seg] + static_cast<long long>(row) * p.ldc[seg] + n0;
    const float* rrow = MODE == kResidual ? p.residual + static_cast<long long>(row) * p.ldr + n0 : nullptr;
    const int cols = min(BN, p.n[seg] - n0);  // a multiple of 4
    const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int c0 = 0; c0 < cols; c0 += 16) {
      float v[16];
      tmem_load16(lanes + static_cast<uint32_t>(c0), v);
      if (MODE == kSwiglu) {
        float u[16];
        tmem_load16(lanes + static_cast<uint32_t>(BN + c0), u);
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = silu_mul(v[e], u[e]);
      }
      if (row < p.m) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (c0 + 4 * q >= cols) continue;
          float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          if (MODE == kResidual) {
            const float* r4 = rrow + c0 + 4 * q;
            o = make_float4(__fadd_rn(r4[0], o.x), __fadd_rn(r4[1], o.y), __fadd_rn(r4[2], o.z), __fadd_rn(r4[3], o.w));
          }
          reinterpret_cast<float4*>(crow + c0)[q] = o;
        }
      }
    }
  } else if (threadIdx.x == 0 && p.error_flag != nullptr) {
    atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_DATA);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, G::kTmemCols);
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

// RMS prologue: rows of rms_norm(a) * w (cb_rmsnorm's roundings, rounded to
// dt_out) split into bf16 planes (lo omitted when dt_out is bf16: hi is
// exact).  One block per row; the row is staged in shared memory.
__global__ void __launch_bounds__(256) rms_planes_kernel(const void* a, int a_dtype, long long lda, long long k,
                                                         const void* w, int w_dtype, NormSpec n, int dt_out,
                                                         __nv_bfloat16* hi, __nv_bfloat16* lo) {
  extern __shared__ float row[];
  __shared__ float red[8];
  const long long r = blockIdx.x;
  const int width = static_cast<int>(k);
  // four elements per thread and access where alignment allows (same arithmetic per element)
  const bool vec = a_dtype == CB_F32 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && lda % 4 == 0 && k % 4 == 0 &&
                   (w_dtype == CB_BF16 || w_dtype == CB_F32) && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  if (vec) {
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(a) + r * lda);
    for (int q = threadIdx.x; q < width / 4; q += blockDim.x) reinterpret_cast<float4*>(row)[q] = src[q];
  } else {
    for (int i = threadIdx.x; i < width; i += blockDim.x) row[i] = load_as_f32(a, r * lda + i, a_dtype);
  }
  __syncthreads();
  const float d = norm_finish_d(n, norm_block_sum(n, row, width, red));
  if (vec) {
    __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(hi + r * k);
    __nv_bfloat162* l2 = lo != nullptr ? reinterpret_cast<__nv_bfloat162*>(lo + r * k) : nullptr;
    for (int q = threadIdx.x; q < width / 4; q += blockDim.x) {
      float wv[4];
      if (w_dtype == CB_BF16) {
        const uint2 wb = reinterpret_cast<const uint2*>(w)[q];
        wv[0] = __uint_as_float(wb.x << 16);
        wv[1] = __uint_as_float(wb.x & 0xffff0000u);
        wv[2] = __uint_as_float(wb.y << 16);
        wv[3] = __uint_as_float(wb.y & 0xffff0000u);
      } else {
        const float4 wf = reinterpret_cast<const float4*>(w)[q];
        wv[0] = wf.x; wv[1] = wf.y; wv[2] = wf.z; wv[3] = wf.w;
      }
      const float4 x = reinterpret_cast<const float4*>(row)[q];
      const float v0 = norm_apply(n, x.x, d, wv[0], dt_out), v1 = norm_apply(n, x.y, d, wv[1], dt_out);
      const float v2 = norm_apply(n, x.z, d, wv[2], dt_out), v3 = norm_apply(n, x.w, d, wv[3], dt_out);
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(v0, v1), h23 = __floats2bfloat162_rn(v2, v3);
      h2[2 * q] = h01;
      h2[2 * q + 1] = h23;
      if (l2 != nullptr) {
        const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
        l2[2 * q] = __floats2bfloat162_rn(__fsub_rn(v0, f01.x), __fsub_rn(v1, f01.y));
        l2[2 * q + 1] = __floats2bfloat162_rn(__fsub_rn(v2, f23.x), __fsub_rn(v3, f23.y));
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float v = norm_apply(n, row[i], d, load_as_f32(w, i, w_dtype), dt_out);
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[r * k + i] = h;
    if (lo != nullptr) lo[r * k + i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
  }
}

// bf16 A usable by TMA as it is (no plane copy).
bool a_direct(const cb_gemm_multi_args& g) {
  return g.x_mode == CB_ROWS_X_PLAIN && g.a_dtype == CB_BF16 && aligned16(g.a) && g.lda % 8 == 0 && g.lda >= g.k;
}

// dtype of the A the MMAs see (the prologue's output)
int a_effective_dtype(const cb_gemm_multi_args& g) { return g.x_mode == CB_ROWS_X_RMS ? g.dt_out : g.a_dtype; }

template <int BN, int NA, int MODE>
cudaError_t launch_gemm(const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap* mb, const GemmParams& p,
                        long long tiles, cudaStream_t s) {
  using G = GemmShape<BN, NA, MODE>;
  auto kernel = gemm_tc_kernel<BN, NA, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  if (e != cudaSuccess) return e;
  kernel<<<static_cast<unsigned>(tiles), kGemmThreads, G::kSmem, s>>>(ma, ma2, mb[0], mb[1], mb[2], p);
  return cudaGetLastError();
}

template <int BN, int MODE>
cudaError_t launch_mode(bool split, const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap* mb,
                        const GemmParams& p, long long tiles, cudaStream_t s) {
  return split ? launch_gemm<BN, 2, MODE>(ma, ma2, mb, p, tiles, s) : launch_gemm<BN, 1, MODE>(ma, ma2, mb, p, tiles, s);
}

long long round_up_to(long long v, long long m) { return (v + m - 1) / m * m; }

int run_multi(const cb_gemm_multi_args* g, cb_stream_t stream) {
  CB_REQUIRE(g != nullptr && g->a != nullptr, "gemm: a is required");
  CB_REQUIRE(g->m > 0 && g->k > 0, "gemm: empty problem");
  CB_REQUIRE(g->k % 8 == 0, "gemm: k=%lld must be a multiple of 8", g->k);
  CB_REQUIRE(g->epilogue == CB_GEMM_STORE || g->epilogue == CB_GEMM_RESIDUAL || g->epilogue == CB_GEMM_SWIGLU,
             "gemm: unknown epilogue %d", g->epilogue);
  const int expect_w = g->epilogue == CB_GEMM_SWIGLU ? 2 : g->epilogue == CB_GEMM_RESIDUAL ? 1 : 0;
  CB_REQUIRE(g->n_w >= 1 && g->n_w <= 3 && (expect_w == 0 || g->n_w == expect_w),
             "gemm: %d weights for epilogue %d", g->n_w, g->epilogue);
  CB_REQUIRE(g->m < (1LL << 31) && g->k < (1LL << 31), "gemm: problem too large");
  CB_REQUIRE(g->a_dtype == CB_BF16 || g->a_dtype == CB_F32, "gemm: a must be bf16 or float32");
  const int n_out = g->epilogue == CB_GEMM_SWIGLU ? 1 : g->n_w;
  for (int i = 0; i < g->n_w; ++i) {
    CB_REQUIRE(g->b[i] != nullptr && aligned16(g->b[i]) && g->ldb[i] % 8 == 0 && g->ldb[i] >= g->k,
               "gemm: weight %d must be 16-byte aligned rows", i);
    CB_REQUIRE(g->n[i] > 0 && g->n[i] % 4 == 0 && g->n[i] < (1LL << 31), "gemm: n=%lld must be a multiple of 4",
               g->n[i]);
  }
  if (g->epilogue == CB_GEMM_SWIGLU) CB_REQUIRE(g->n[0] == g->n[1], "gemm: SwiGLU needs gate and up of equal rows");
  for (int i = 0; i < n_out; ++i)
    CB_REQUIRE(g->c[i] != nullptr && aligned16(g->c[i]) && g->ldc[i] % 4 == 0 && g->ldc[i] >= g->n[i],
               "gemm: c must be 16-byte aligned rows");
  if (g->epilogue == CB_GEMM_RESIDUAL)
    CB_REQUIRE(g->residual != nullptr && aligned16(g->residual) && g->ldr % 4 == 0 && g->ldr >= g->n[0],
               "gemm: residual must be 16-byte aligned rows");
  CB_REQUIRE(g->x_mode == CB_ROWS_X_PLAIN || g->x_mode == CB_ROWS_X_RMS, "gemm: unknown A prologue %d", g->x_mode);
  if (g->x_mode == CB_ROWS_X_RMS)
    CB_REQUIRE(g->norm_w != nullptr && g->k <= 49152 && g->divisor != 0.0f &&
                   (g->dt_out == CB_F32 || g->dt_out == CB_BF16),
               "gemm: RMS prologue needs norm_w, k <= 49152 and a float32 or bf16 output");
  const bool split = a_effective_dtype(*g) == CB_F32;
  const bool direct = a_direct(*g);
  CB_REQUIRE(direct || (g->a_split != nullptr && aligned16(g->a_split)), "gemm: a needs %lld bytes of a_split",
             cb_gemm_tc_multi_scratch(g));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* a_hi = g->a;
  const void* a_lo = nullptr;
  long long lda = g->lda;
  if (g->x_mode == CB_ROWS_X_RMS) {
    __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(g->a_split);
    __nv_bfloat16* lo = split ? hi + g->m * g->k : nullptr;
    const NormSpec n{g->divisor, g->eps, g->dt_sq, g->dt_sum, g->dt_mean, g->dt_t, g->dt_d, g->dt_y};
    const size_t smem = static_cast<size_t>(g->k) * sizeof(float);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(rms_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    rms_planes_kernel<<<static_cast<unsigned>(g->m), 256, smem, s>>>(g->a, g->a_dtype, g->lda, g->k, g->norm_w,
                                                                     g->norm_w_dtype, n, g->dt_out, hi, lo);
    a_hi = hi;
    a_lo = lo;
    lda = g->k;
  } else if (!direct) {
    __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(g->a_split);
    __nv_bfloat16* lo = split ? hi + g->m * g->k : nullptr;
    split_planes_kernel<<<static_cast<unsigned>(g->m), 256, 0, s>>>(g->a, g->a_dtype, g->lda, g->k, hi, lo);
    a_hi = hi;
    a_lo = lo;
    lda = g->k;
  }
  // 256-wide tiles unless 128 wastes less of the last column tiles
  long long waste256 = 0, waste128 = 0;
  for (int i = 0; i < (g->epilogue == CB_GEMM_SWIGLU ? 1 : g->n_w); ++i) {
    waste256 += round_up_to(g->n[i], 256) - g->n[i];
    waste128 += round_up_to(g->n[i], 128) - g->n[i];
  }
  const int bn = waste256 <= waste128 ? 256 : 128;
  GemmParams p{};
  const long long tiles_m = (g->m + kBM - 1) / kBM;
  long long tiles = 0;
  p.n_seg = g->epilogue == CB_GEMM_STORE ? g->n_w : 1;
  for (int i = 0; i < n_out; ++i) {
    p.c[i] = g->c[i];
    p.ldc[i] = g->ldc[i];
  }
  for (int i = 0; i < p.n_seg; ++i) {
    p.n[i] = static_cast<int>(g->n[i]);
    p.tiles_n[i] = static_cast<int>((g->n[i] + bn - 1) / bn);
    tiles += tiles_m * p.tiles_n[i];
  }
  CB_REQUIRE(tiles < (1LL << 31), "gemm: problem too large");
  p.m = static_cast<int>(g->m);
  p.k = static_cast<int>(g->k);
  p.residual = g->residual;
  p.ldr = g->ldr;
  p.error_flag = g->error_flag;
  CUtensorMap ma, ma2, mb[3];
  CB_REQUIRE(make_map(&ma, a_hi, g->m, g->k, lda, kBM) && (a_lo == nullptr || make_map(&ma2, a_lo, g->m, g->k, lda, kBM)),
             "gemm: tensor map encoding failed");
  if (a_lo == nullptr) ma2 = ma;
  for (int i = 0; i < 3; ++i) {
    const int j = i < g->n_w ? i : 0;
    CB_REQUIRE(make_map(mb + i, g->b[j], g->n[j], g->k, g->ldb[j], bn), "gemm: tensor map encoding failed");
  }
  cudaError_t e;
  if (bn == 256) {
    e = g->epilogue == CB_GEMM_SWIGLU     ? launch_mode<256, kSwiglu>(split, ma, ma2, mb, p, tiles, s)
        : g->epilogue == CB_GEMM_RESIDUAL ? launch_mode<256, kResidual>(split, ma, ma2, mb, p, tiles, s)
                                          : launch_mode<256, kStore>(split, ma, ma2, mb, p, tiles, s);
  } else {
    e = g->epilogue == CB_GEMM_SWIGLU     ? launch_mode<128, kSwiglu>(split, ma, ma2, mb, p, tiles, s)
        : g->epilogue == CB_GEMM_RESIDUAL ? launch_mode<128, kResidual>(split, ma, ma2, mb, p, tiles, s)
                                          : launch_mode<128, kStore>(split, ma, ma2, mb, p, tiles, s);
  }
  if (e != cudaSuccess) {
    set_error("cb_gemm_tc: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_gemm_tc");
}

cb_gemm_multi_args single(const cb_gemm_args* g) {
  cb_gemm_multi_args m{};
  m.a = g->a;
  m.a_dtype = g->a_dtype;
  m.lda = g->lda;
  m.m = g->m;
  m.k = g->k;
  m.n_w = 1;
  m.b[0] = g->b;
  m.ldb[0] = g->ldb;
  m.n[0] = g->n;
  m.c[0] = g->c;
  m.ldc[0] = g->ldc;
  m.epilogue = CB_GEMM_STORE;
  m.a_split = g->a_split;
  m.error_flag = g->error_flag;
  return m;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

long long cb_gemm_tc_multi_scratch(const cb_gemm_multi_args* g) {
  if (g == nullptr || g->m <= 0 || g->k <= 0) return 0;
  if (a_effective_dtype(*g) == CB_F32) return 2 * g->m * g->k * 2;
  return a_direct(*g) ? 0 : g->m * g->k * 2;
}

int cb_gemm_tc_multi(const cb_gemm_multi_args* g, cb_stream_t stream) { return run_multi(g, stream); }

long long cb_gemm_tc_scratch(const cb_gemm_args* g) {
  if (g == nullptr) return 0;
  const cb_gemm_multi_args m = single(g);
  return cb_gemm_tc_multi_scratch(&m);
}

int cb_gemm_tc(const cb_gemm_args* g, cb_stream_t stream) {
  CB_REQUIRE(g != nullptr && g->a != nullptr && g->b != nullptr && g->c != nullptr, "gemm: a, b and c are required");
  CB_REQUIRE(g->m > 0 && g->n > 0 && g->k > 0, "gemm: empty problem");
  CB_REQUIRE(g->k % 8 == 0, "gemm: k=%lld must be a multiple of 8", g->k);
  CB_REQUIRE(g->n % 4 == 0, "gemm: n=%lld must be a multiple of 4", g->n);
  const cb_gemm_multi_args m = single(g);
  return run_multi(&m, stream);
}

}  // extern "C"

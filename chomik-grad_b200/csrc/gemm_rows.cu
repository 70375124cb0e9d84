// Few-row tensor-core GEMM for batched decode: cb_gemm_rows.
//
// out_i (rows x n_i, float32) = x (rows x k) . W_i^T for up to three bf16
// weights W_i (n_i x k, HF (out, in) layout) sharing one x -- the q/k/v or
// gate/up Linears of a decode step over a batch of sequences
// (chomikgrad/llama.py:275-277).  With few rows (a batch of 1..256
// sequences) a weight-streaming GEMM is bound by the weight bytes, so the
// operands are swapped: the weight rows are the MMA's M = 128 side, the
// batch rows its N side (rows padded to a multiple of 16 by the tensor map's
// zero fill), and K is split across CTAs so that the weight stream is spread
// over every SM:
//  * thread 0 streams 64-wide K chunks of the weight tile and of x's bf16
//    hi/lo planes (split once by a pre-pass) with TMA into a ring of stages;
//  * thread 32 issues tcgen05.mma (kind::f16, M=128, N=rows padded, K=16)
//    W.x_hi + W.x_lo into a TMEM accumulator;
//  * all four warps read the accumulator (warp w owns weight rows 32w..);
//    with one split they store out directly, otherwise they store a partial
//    and the last CTA of the weight tile (a ticket counter) sums the splits
//    in split order -- deterministic -- stores out and re-arms the counter.
// Every wait is bounded (sync.cuh).
#include "tc_core.cuh"

namespace cb {
namespace {

using namespace tc;

constexpr int kRowsThreads = 128;
constexpr int kWTile = 128;  // weight rows per tile = TMEM lanes

template <int NB>
struct RowsShape {
  static constexpr int kW = kWTile * kChunk * 2;  // weight chunk bytes
  static constexpr int kX = NB * kChunk * 2;      // one x plane chunk
  static constexpr int kStage = kW + 2 * kX;
  static constexpr int kStages = (NB <= 64 ? 96 * 1024 : 192 * 1024) / kStage;
  static constexpr int kSmem = kStages * kStage + 1024;
  static constexpr int kTmemCols = NB < 32 ? 32 : NB;
  static_assert(kStages >= 2, "at least double buffering");
};

struct RowsParams {
  float* out[3];
  long long ldo[3];
  int tiles[3];        // 128-row weight tiles of each weight (prefix order)
  int n[3];
  int n_w;
  int rows;
  int kchunks;         // 64-wide K chunks
  int splits;
  float* partial;      // (tiles, splits, NB, 128) float32, splits > 1
  unsigned* counters;  // one per tile, 0 between launches
  int* error_flag;
};

template <int NB>
__global__ void __launch_bounds__(kRowsThreads)
    gemm_rows_kernel(const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1,
                     const __grid_constant__ CUtensorMap map_w2, const __grid_constant__ CUtensorMap map_xh,
                     const __grid_constant__ CUtensorMap map_xl, const __grid_constant__ RowsParams p) {
  using G = RowsShape<NB>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[G::kStages];
  __shared__ __align__(8) uint64_t empty[G::kStages];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ int last_split;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  int seg = 0, seg_tile = tile;
  while (seg + 1 < p.n_w && seg_tile >= p.tiles[seg]) seg_tile -= p.tiles[seg++];
  const int row0 = seg_tile * kWTile;
  const int per = (p.kchunks + p.splits - 1) / p.splits;
  const int c_begin = split * per, c_end = min(p.kchunks, c_begin + per);
  const int nchunks = max(c_end - c_begin, 0);

  if (warp == 0) tmem_alloc(&tmem_base, G::kTmemCols);
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
  volatile int* abort = &abort_flag;

  if (warp == 0 && lane == 0) {
    int i = 0;
    for (; i < nchunks; ++i) {
      const int s = i % G::kStages, round = i / G::kStages;
      if (round > 0 && !wait_or_abort(empty + s, static_cast<uint32_t>((round - 1) & 1), abort)) {
        if (p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_SLOT);
        *abort = 1;
        break;
      }
      unsigned char* st = smem + s * G::kStage;
      const int kx = (c_begin + i) * kChunk;
      mbar_arrive_expect_tx(full + s, static_cast<uint32_t>(G::kStage));
      if (seg == 0)
        tma_load_2d(st, &map_w0, kx, row0, full + s);
      else if (seg == 1)
        tma_load_2d(st, &map_w1, kx, row0, full + s);
      else
        tma_load_2d(st, &map_w2, kx, row0, full + s);
      tma_load_2d(st + G::kW, &map_xh, kx, 0, full + s);
      tma_load_2d(st + G::kW + G::kX, &map_xl, kx, 0, full + s);
    }
    for (int t = i - 1; t >= 0 && t >= i - G::kStages; --t) {
      if (!wait_short(full + t % G::kStages, static_cast<uint32_t>((t / G::kStages) & 1))) {
        if (p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_DRAIN);
        break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16(kWTile, NB < 16 ? 16 : NB);
    for (int i = 0; i < nchunks; ++i) {
      const int s = i % G::kStages, round = i / G::kStages;
      if (!wait_or_abort(full + s, static_cast<uint32_t>(round & 1), abort)) {
        if (p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_DATA);
        *abort = 1;
        break;
      }
      fence_after();
      const unsigned char* st = smem + s * G::kStage;
#pragma unroll
      for (int kk = 0; kk < kChunk / kUmmaK; ++kk) {
        const uint64_t dw = sw128_desc(st + kk * kUmmaK * 2);
        umma_bf16(tmem, dw, sw128_desc(st + G::kW + kk * kUmmaK * 2), idesc, (i | kk) != 0 ? 1u : 0u);
        umma_bf16(tmem, dw, sw128_desc(st + G::kW + G::kX + kk * kUmmaK * 2), idesc, 1u);
      }
      umma_commit(empty + s);
    }
    umma_commit(&acc_full);
  }
  __syncwarp();

  bool ok = wait_or_abort(&acc_full, 0u, abort) || wait_short(&acc_full, 0u);
  ok = __all_sync(0xffffffffu, ok && *abort == 0 && nchunks > 0);
  fence_after();
  const int r = warp * 32 + lane;  // weight row within the tile
  const int row = row0 + r;
  const int n = p.n[seg];
  float* out = p.out[seg];
  const long long ldo = p.ldo[seg];
  if (p.splits == 1) {
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < NB; c0 += 16) {
        float v[16];
        tmem_load16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(c0), v);
        if (row < n) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c0 + e < p.rows) out[static_cast<long long>(c0 + e) * ldo + row] = v[e];
        }
      }
    }
  } else {
    float* mine = p.partial + (static_cast<long long>(tile) * p.splits + split) * NB * kWTile;
#pragma unroll 1
    for (int c0 = 0; c0 < NB; c0 += 16) {
      float v[16];
      if (ok) {
        tmem_load16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(c0), v);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.0f;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) mine[(c0 + e) * kWTile + r] = v[e];
    }
    if (!ok && threadIdx.x == 0 && nchunks > 0 && p.error_flag != nullptr) atomicCAS(p.error_flag, 0, CB_FLAG_WAIT_DATA);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_split = atomicAdd(p.counters + tile, 1u) == static_cast<unsigned>(p.splits - 1);
    __syncthreads();
    if (last_split) {
      __threadfence();
      const float* base = p.partial + static_cast<long long>(tile) * p.splits * NB * kWTile;
      for (int b = 0; b < p.rows; ++b) {
        float acc = 0.0f;
        for (int s = 0; s < p.splits; ++s) acc += __ldcg(base + (static_cast<long long>(s) * NB + b) * kWTile + r);
        if (row < n) out[static_cast<long long>(b) * ldo + row] = acc;
      }
      if (threadIdx.x == 0) p.counters[tile] = 0u;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, G::kTmemCols);
}

// x rows (float32 or bf16, row stride ldx) -> bf16 planes hi, lo (rows x k).
__global__ void rows_planes_kernel(const void* x, int x_dtype, long long ldx, long long k, __nv_bfloat16* hi,
                                   __nv_bfloat16* lo) {
  const long long r = blockIdx.x;
  for (long long c = threadIdx.x; c < k; c += blockDim.x) {
    const float v = load_as_f32(x, r * ldx + c, x_dtype);
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[r * k + c] = h;
    lo[r * k + c] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
  }
}

int padded_rows(long long rows) { return rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256; }

struct RowsPlan {
  int nb, tiles, splits, kchunks;
  long long plane_elems, partial_floats;
};

RowsPlan plan_rows(const cb_gemm_rows_args& a, int sms) {
  RowsPlan r{};
  r.nb = padded_rows(a.rows);
  r.kchunks = static_cast<int>((a.k + kChunk - 1) / kChunk);
  for (int i = 0; i < a.n_w; ++i) r.tiles += static_cast<int>((a.w_rows[i] + kWTile - 1) / kWTile);
  // spread the weight stream over about two CTAs per SM, at least 4 K chunks per split
  int splits = a.splits > 0 ? a.splits : (2 * sms + r.tiles - 1) / r.tiles;
  const int most = r.kchunks / 4 > 0 ? r.kchunks / 4 : 1;
  splits = splits < 1 ? 1 : splits;
  splits = splits > most ? most : splits;
  splits = splits > 16 ? 16 : splits;
  r.splits = splits;
  r.plane_elems = a.rows * a.k;
  r.partial_floats = splits > 1 ? static_cast<long long>(r.tiles) * splits * r.nb * kWTile : 0;
  return r;
}

template <int NB>
int launch_rows(const cb_gemm_rows_args& a, const RowsPlan& pl, cudaStream_t s) {
  using G = RowsShape<NB>;
  __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(a.scratch);
  __nv_bfloat16* lo = hi + pl.plane_elems;
  rows_planes_kernel<<<static_cast<unsigned>(a.rows), 256, 0, s>>>(a.x, a.x_dtype, a.ldx, a.k, hi, lo);
  CB_REQUIRE(cudaGetLastError() == cudaSuccess, "cb_gemm_rows: plane pass launch failed");
  CUtensorMap mw[3], mxh, mxl;
  for (int i = 0; i < 3; ++i) {
    const int j = i < a.n_w ? i : 0;
    CB_REQUIRE(make_map(mw + i, a.w[j], a.w_rows[j], a.k, a.k, kWTile), "cb_gemm_rows: weight tensor map failed");
  }
  CB_REQUIRE(make_map(&mxh, hi, a.rows, a.k, a.k, NB) && make_map(&mxl, lo, a.rows, a.k, a.k, NB),
             "cb_gemm_rows: x tensor map failed");
  RowsParams p{};
  for (int i = 0; i < a.n_w; ++i) {
    p.out[i] = a.out[i];
    p.ldo[i] = a.ldo[i];
    p.n[i] = static_cast<int>(a.w_rows[i]);
    p.tiles[i] = static_cast<int>((a.w_rows[i] + kWTile - 1) / kWTile);
  }
  p.n_w = a.n_w;
  p.rows = static_cast<int>(a.rows);
  p.kchunks = pl.kchunks;
  p.splits = pl.splits;
  p.partial = reinterpret_cast<float*>(lo + pl.plane_elems + (pl.plane_elems & 1 ? 1 : 0));
  p.counters = a.counters;
  p.error_flag = a.error_flag;
  auto kernel = gemm_rows_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  if (e == cudaSuccess) {
    kernel<<<static_cast<unsigned>(pl.tiles * pl.splits), kRowsThreads, G::kSmem, s>>>(mw[0], mw[1], mw[2], mxh,
                                                                                        mxl, p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_error("cb_gemm_rows: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_gemm_rows");
}

int sm_count_cached() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  return sms;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

long long cb_gemm_rows_scratch(const cb_gemm_rows_args* a) {
  if (a == nullptr || a->rows <= 0 || a->k <= 0 || a->n_w < 1 || a->n_w > 3) return 0;
  const RowsPlan pl = plan_rows(*a, sm_count_cached());
  const long long planes = 2 * pl.plane_elems * 2 + 16;  // hi, lo (+ alignment of the partials)
  return (planes + 15) / 16 * 16 + pl.partial_floats * 4;
}

long long cb_gemm_rows_counters(const cb_gemm_rows_args* a) {
  if (a == nullptr || a->n_w < 1 || a->n_w > 3) return 0;
  long long tiles = 0;
  for (int i = 0; i < a->n_w; ++i) tiles += (a->w_rows[i] + kWTile - 1) / kWTile;
  return tiles;
}

int cb_gemm_rows(const cb_gemm_rows_args* a, cb_stream_t stream) {
  CB_REQUIRE(a != nullptr && a->x != nullptr && a->scratch != nullptr, "gemm_rows: x and scratch are required");
  CB_REQUIRE(a->n_w >= 1 && a->n_w <= 3, "gemm_rows: 1 to 3 weights");
  CB_REQUIRE(a->rows >= 1 && a->rows <= 256, "gemm_rows: rows=%lld (1..256)", a->rows);
  CB_REQUIRE(a->k > 0 && a->k % 8 == 0 && a->k < (1LL << 31), "gemm_rows: k=%lld must be a multiple of 8", a->k);
  CB_REQUIRE(a->x_dtype == CB_F32 || a->x_dtype == CB_BF16, "gemm_rows: x must be float32 or bf16");
  CB_REQUIRE(aligned16(a->scratch), "gemm_rows: scratch must be 16-byte aligned");
  for (int i = 0; i < a->n_w; ++i) {
    CB_REQUIRE(a->w[i] != nullptr && aligned16(a->w[i]) && a->out[i] != nullptr, "gemm_rows: weight %d", i);
    CB_REQUIRE(a->w_rows[i] > 0 && a->w_rows[i] < (1LL << 31) && a->ldo[i] >= a->w_rows[i],
               "gemm_rows: weight %d shape", i);
  }
  const RowsPlan pl = plan_rows(*a, sm_count_cached());
  CB_REQUIRE(pl.splits == 1 || a->counters != nullptr, "gemm_rows: split K needs counters");
  CB_REQUIRE(static_cast<long long>(pl.tiles) * pl.splits < (1LL << 31), "gemm_rows: too many tiles");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (pl.nb) {
    case 16: return launch_rows<16>(*a, pl, s);
    case 32: return launch_rows<32>(*a, pl, s);
    case 64: return launch_rows<64>(*a, pl, s);
    case 128: return launch_rows<128>(*a, pl, s);
    default: return launch_rows<256>(*a, pl, s);
  }
}

}  // extern "C"

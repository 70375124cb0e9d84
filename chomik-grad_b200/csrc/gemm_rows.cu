// Few-row tensor-core GEMM for batched decode: cb_gemm_rows.
//
// out_i (rows x n_i, float32) = x (rows x k) . W_i^T for up to three bf16
// weights W_i (n_i x k, HF (out, in) layout) sharing one x -- the q/k/v or
// gate/up Linears of a decode step over a batch of sequences
// (chomikgrad/llama.py:275-277).  With few rows (a batch of 1..256
// sequences) the GEMM is bound by the weight bytes, so the operands are
// swapped: the weight rows are the MMA's M = 128 side, the batch rows its N
// side (rows padded to a multiple of 16 by the tensor map's zero fill).
//
// The weight stream is cut into 64-wide K chunks of 128-row tiles and the
// flattened (tile, chunk) sequence is split into one contiguous, equal range
// per CTA (one persistent CTA per SM; two, each with half the ring, for
// weights of 32 MB and more), so every SM streams the same number of bytes
// without a break:
//  * warp 4 streams its range with TMA (the weight chunk and x's bf16 hi/lo
//    planes, split once by a pre-pass) into a ring of stages;
//  * warp 5 issues tcgen05.mma (kind::f16, M=128, N=rows padded, K=16)
//    W.x_hi + W.x_lo (W.x_hi alone when x is exactly bf16, its lo plane
//    zero) into one of two TMEM accumulators, switching at each
//    tile boundary of the range (a "segment"), so the epilogue of one tile
//    overlaps the MMAs of the next;
//  * warps 0-3 read each finished accumulator (warp w owns weight rows
//    32w..): a segment that covers the whole tile stores out directly;
//    otherwise it stores a partial, and the last of the tile's parts (a
//    ticket counter) sums them in part order -- deterministic -- stores out
//    and re-arms the counter.
// Every wait is bounded (sync.cuh); on a timeout the kernel records an
// error, lets its copies land and its MMAs finish, frees TMEM and returns.
#include "norm.cuh"
#include "tc_core.cuh"

namespace cb {
namespace {

using namespace tc;

constexpr int kRowsThreads = 192;  // warps 0-3 epilogue, warp 4 TMA, warp 5 MMA
constexpr int kWTile = 128;        // weight rows per tile = TMEM lanes

// CTAS: resident CTAs per SM.  Two CTAs of half the ring stream a large
// weight faster than one (each CTA's stage hand-offs bound its own stream:
// about 32 GB/s per CTA); small GEMMs keep one, whose tiles split into fewer
// parts.
template <int NB, int CTAS = 1>
struct RowsShape {
  static constexpr int kW = kWTile * kChunk * 2;  // weight chunk bytes
  static constexpr int kX = NB * kChunk * 2;      // one x plane chunk
  static constexpr int kStage = kW + 2 * kX;
  static constexpr int kStages = (CTAS == 2 ? 100 : 200) * 1024 / kStage;
  static constexpr int kSmem = kStages * kStage + 1024;
  static constexpr int kAcc = NB < 32 ? 32 : NB;  // columns of one accumulator
  static constexpr int kTmemCols = 2 * kAcc;
  static_assert(kStages >= 2, "at least double buffering");
};

struct RowsParams {
  float* out[3];
  long long ldo[3];
  int tiles[3];        // 128-row weight tiles of each weight (prefix order)
  int n[3];
  int n_w;
  int rows;
  int kchunks;         // 64-wide K chunks per tile
  long long total;     // tiles * kchunks
  int max_parts;       // partial slots per tile
  int lo_plane;        // 0: x is exactly bf16 (its lo plane is zero): no lo loads, no lo MMAs
  float* partial;      // (tiles, max_parts, NB, 128) float32
  unsigned* counters;  // one per tile, 0 between launches
  int* error_flag;
  const float* residual;  // n_w == 1: out = residual + x W^T
  long long ldr;
};

// The CTA whose range holds flattened chunk f: ranges are [c T / G, (c+1) T / G).
__device__ __forceinline__ int cta_of(long long f, long long total, int grid) {
  return static_cast<int>(((f + 1) * grid + total - 1) / total - 1);
}

__device__ __forceinline__ void set_flag(int* flag, int code) {
  if (flag != nullptr) atomicCAS(flag, 0, code);
}

template <int NB, int CTAS>
__global__ void __launch_bounds__(kRowsThreads, CTAS)
    gemm_rows_kernel(const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1,
                     const __grid_constant__ CUtensorMap map_w2, const __grid_constant__ CUtensorMap map_xh,
                     const __grid_constant__ CUtensorMap map_xl, const __grid_constant__ RowsParams p) {
  using G = RowsShape<NB, CTAS>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[G::kStages];
  __shared__ __align__(8) uint64_t empty[G::kStages];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ __align__(8) uint64_t parts_in;    // the epilogue's partials of a segment are written (128)
  __shared__ __align__(8) uint64_t ticket_out;  // thread 0 has taken the tile's ticket (1)
  __shared__ int last_part[2];                  // by split-segment parity
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long f0 = static_cast<long long>(blockIdx.x) * p.total / gridDim.x;
  const long long f1 = static_cast<long long>(blockIdx.x + 1) * p.total / gridDim.x;

  if (warp == 0) tmem_alloc(&tmem_base, G::kTmemCols);
  if (threadIdx.x == 32) {
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 128);
    }
    mbar_init(&mma_done, 1);
    mbar_init(&parts_in, 128);
    mbar_init(&ticket_out, 1);
    mbar_fence_init();
    abort_flag = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* abort = &abort_flag;

  if (warp == 4) {
    if (lane == 0) {
      // ---- TMA producer: the range's chunks in order ----
      // The weights do not depend on the previous kernel: the first ring's
      // worth of weight chunks is issued before waiting for it (programmatic
      // dependent launch), the x planes (written by the plane pass just
      // before) only after.
      auto weight_load = [&](long long f, int s) {
        int tile = static_cast<int>(f / p.kchunks);
        const int kx = static_cast<int>(f % p.kchunks) * kChunk;
        int seg = 0;
        while (seg + 1 < p.n_w && tile >= p.tiles[seg]) tile -= p.tiles[seg++];
        const CUtensorMap* mw = seg == 0 ? &map_w0 : seg == 1 ? &map_w1 : &map_w2;
        tma_load_2d(smem + s * G::kStage, mw, kx, tile * kWTile, full + s);
      };
      auto x_load = [&](long long f, int s) {
        const int kx = static_cast<int>(f % p.kchunks) * kChunk;
        unsigned char* st = smem + s * G::kStage;
        tma_load_2d(st + G::kW, &map_xh, kx, 0, full + s);
        if (p.lo_plane) tma_load_2d(st + G::kW + G::kX, &map_xl, kx, 0, full + s);
      };
      const long long pre = f1 - f0 < G::kStages ? f1 - f0 : G::kStages;
      const uint32_t stage_bytes = static_cast<uint32_t>(p.lo_plane ? G::kStage : G::kW + G::kX);
      for (long long j = 0; j < pre; ++j) {
        mbar_arrive_expect_tx(full + j, stage_bytes);
        weight_load(f0 + j, static_cast<int>(j));
      }
      pdl_wait();
      pdl_launch_dependents();
      for (long long j = 0; j < pre; ++j) x_load(f0 + j, static_cast<int>(j));
      long long i = pre;
      for (long long f = f0 + pre; f < f1; ++f, ++i) {
        const int s = static_cast<int>(i % G::kStages);
        const long long round = i / G::kStages;
        if (round > 0 && !wait_or_abort(empty + s, static_cast<uint32_t>((round - 1) & 1), abort)) {
          set_flag(p.error_flag, CB_FLAG_WAIT_SLOT);
          *abort = 1;
          break;
        }
        mbar_arrive_expect_tx(full + s, stage_bytes);
        weight_load(f, s);
        x_load(f, s);
      }
      // drain: every copy issued lands before the block can exit
      for (long long t = i - 1; t >= 0 && t >= i - G::kStages; --t) {
        if (!wait_short(full + t % G::kStages, static_cast<uint32_t>((t / G::kStages) & 1))) {
          set_flag(p.error_flag, CB_FLAG_WAIT_DRAIN);
          break;
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---- MMA issuer: one accumulator per segment, alternating ----
      constexpr uint32_t idesc = idesc_bf16(kWTile, NB < 16 ? 16 : NB);
      long long i = 0;
      int seg_no = 0;
      bool ok = true;
      for (long long a = f0; ok && a < f1; ++seg_no) {
        const long long b = min(f1, (a / p.kchunks + 1) * p.kchunks);  // segment [a, b): one tile
        const int buf = seg_no & 1;
        if (seg_no >= 2 && !wait_or_abort(acc_empty + buf, static_cast<uint32_t>(((seg_no >> 1) - 1) & 1), abort)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * G::kAcc);
        for (long long f = a; f < b; ++f, ++i) {
          const int s = static_cast<int>(i % G::kStages);
          if (!wait_or_abort(full + s, static_cast<uint32_t>((i / G::kStages) & 1), abort)) {
            ok = false;
            break;
          }
          fence_after();
          const unsigned char* st = smem + s * G::kStage;
#pragma unroll
          for (int kk = 0; kk < kChunk / kUmmaK; ++kk) {
            const uint64_t dw = sw128_desc(st + kk * kUmmaK * 2);
            umma_bf16(d, dw, sw128_desc(st + G::kW + kk * kUmmaK * 2), idesc, (f != a || kk != 0) ? 1u : 0u);
            if (p.lo_plane) umma_bf16(d, dw, sw128_desc(st + G::kW + G::kX + kk * kUmmaK * 2), idesc, 1u);
          }
          umma_commit(empty + s);
        }
        if (ok) umma_commit(acc_full + buf);
        a = b;
      }
      if (!ok) {
        set_flag(p.error_flag, CB_FLAG_WAIT_DATA);
        *abort = 1;
      }
      umma_commit(&mma_done);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---- epilogue: warps 0-3, thread = weight row of the tile ----
    pdl_wait();  // residual, partials, counters and out: after the previous kernel
    const int r = warp * 32 + lane;
    const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    int seg_no = 0, splits_done = 0;
    for (long long a = f0; a < f1; ++seg_no) {
      const long long tile_flat = a / p.kchunks;
      const long long b = min(f1, (tile_flat + 1) * p.kchunks);
      const int buf = seg_no & 1;
      if (!__all_sync(0xffffffffu, wait_or_abort(acc_full + buf, static_cast<uint32_t>((seg_no >> 1) & 1), abort))) {
        set_flag(p.error_flag, CB_FLAG_WAIT_DATA);
        *abort = 1;
        break;
      }
      fence_after();
      int tile = static_cast<int>(tile_flat), seg = 0;
      while (seg + 1 < p.n_w && tile >= p.tiles[seg]) tile -= p.tiles[seg++];
      const int row = tile * kWTile + r;
      const int n = p.n[seg];
      float* out = p.out[seg];
      const long long ldo = p.ldo[seg];
      const bool whole = a == tile_flat * p.kchunks && b == (tile_flat + 1) * p.kchunks;
      const long long c_first = cta_of(tile_flat * p.kchunks, p.total, gridDim.x);
      float* mine = p.partial + ((tile_flat * p.max_parts + (blockIdx.x - c_first)) * NB) * kWTile;
#pragma unroll 1
      for (int c0 = 0; c0 < NB; c0 += 16) {
        float v[16];
        tmem_load16(lanes + static_cast<uint32_t>(buf * G::kAcc + c0), v);
        if (whole) {
          if (row < n) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              if (c0 + e >= p.rows) continue;
              const float r = p.residual != nullptr ? p.residual[static_cast<long long>(c0 + e) * p.ldr + row] : 0.0f;
              out[static_cast<long long>(c0 + e) * ldo + row] = p.residual != nullptr ? __fadd_rn(r, v[e]) : v[e];
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) mine[(c0 + e) * kWTile + r] = v[e];
        }
      }
      fence_before();
      mbar_arrive(acc_empty + buf);  // the accumulator is free for segment seg_no + 2
      if (!whole) {
        // every thread's partial is visible GPU-wide before thread 0 takes
        // the tile's ticket; the last part sums all parts in part order
        const int parts = cta_of((tile_flat + 1) * p.kchunks - 1, p.total, gridDim.x) - static_cast<int>(c_first) + 1;
        const uint32_t phase = static_cast<uint32_t>(splits_done & 1);
        __threadfence();
        mbar_arrive(&parts_in);
        if (r == 0) {
          const bool in = wait_or_abort(&parts_in, phase, abort);
          if (!in) set_flag(p.error_flag, CB_FLAG_WAIT_DATA);
          last_part[splits_done & 1] =
              in && atomicAdd(p.counters + tile_flat, 1u) == static_cast<unsigned>(parts - 1);
          mbar_arrive(&ticket_out);
        }
        if (!__all_sync(0xffffffffu, wait_or_abort(&ticket_out, phase, abort))) {
          set_flag(p.error_flag, CB_FLAG_WAIT_DATA);
          *abort = 1;
          break;
        }
        if (last_part[splits_done & 1]) {
          // thread t sums 4 weight rows (float4 group t % 32) for batch rows
          // t / 32 + 4 j, every part in order; 8 batch rows per batch of
          // loads, all in flight together
          __threadfence();
          const float4* base = reinterpret_cast<const float4*>(p.partial + tile_flat * p.max_parts * NB * kWTile);
          const int g = r & 31, b0 = r >> 5;
          const int row4 = tile * kWTile + 4 * g;
          // The parts are summed in part order; the loads of kBatch parts
          // (and the residual values) are issued together, so a tile split
          // P ways waits for ceil(P / kBatch) L2 round trips, not P.
          constexpr int kBatch = CTAS == 2 ? 2 : 4;  // two CTAs per SM: 168 registers per thread
          auto part_loads = [&](int q, int bs, float4* v) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int bb = bs + 4 * j;
              v[j] = bb < p.rows ? __ldcg(base + ((static_cast<long long>(q) * NB + bb) * kWTile) / 4 + g)
                                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
          };
          auto part_add = [](float4* acc, const float4* v) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acc[j].x += v[j].x;
              acc[j].y += v[j].y;
              acc[j].z += v[j].z;
              acc[j].w += v[j].w;
            }
          };
          for (int bs = b0; bs < p.rows; bs += 32) {
            float res[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int bb = bs + 4 * j;
              const float* rr = p.residual != nullptr && bb < p.rows
                                    ? p.residual + static_cast<long long>(bb) * p.ldr : nullptr;
#pragma unroll
              for (int e = 0; e < 4; ++e) res[j][e] = rr != nullptr && row4 + e < n ? rr[row4 + e] : 0.0f;
            }
            float4 acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            int q = 0;
            for (; q + kBatch <= parts; q += kBatch) {
              float4 v[kBatch][8];
#pragma unroll
              for (int u = 0; u < kBatch; ++u) part_loads(q + u, bs, v[u]);
#pragma unroll
              for (int u = 0; u < kBatch; ++u) part_add(acc, v[u]);
            }
            for (; q < parts; ++q) {
              float4 v[8];
              part_loads(q, bs, v);
              part_add(acc, v);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int bb = bs + 4 * j;
              if (bb >= p.rows) continue;
              float* o = out + static_cast<long long>(bb) * ldo;
              const float a4[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (row4 + e < n) o[row4 + e] = p.residual != nullptr ? __fadd_rn(res[j][e], a4[e]) : a4[e];
            }
          }
          if (r == 0) p.counters[tile_flat] = 0u;
        }
        ++splits_done;
      }
      a = b;
    }
  }
  __syncwarp();
  fence_before();
  __syncthreads();
  if (warp == 0) {
    // TMEM is freed only after every MMA that writes it has completed
    if (!wait_short(&mma_done, 0u) && lane == 0) set_flag(p.error_flag, CB_FLAG_WAIT_DRAIN);
    fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}

__device__ __forceinline__ void split_store(float v, __nv_bfloat16* hi, __nv_bfloat16* lo, long long i) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  hi[i] = h;
  lo[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
}

// x rows (float32 or bf16, row stride ldx) -> bf16 planes hi, lo (rows x k),
// through the PLAIN or SWIGLU prologue; grid (rows, k chunks of 1024).
__global__ void rows_planes_kernel(const void* x, int x_dtype, long long ldx, long long k, const void* x2,
                                   int x2_dtype, long long ldx2, int swiglu, __nv_bfloat16* hi, __nv_bfloat16* lo) {
  pdl_wait();
  pdl_launch_dependents();
  const long long r = blockIdx.x;
  const long long c1 = min(k, (blockIdx.y + 1) * 1024LL);
  for (long long c = blockIdx.y * 1024LL + threadIdx.x; c < c1; c += blockDim.x) {
    float v = load_as_f32(x, r * ldx + c, x_dtype);
    if (swiglu) {  // the reference's float32 chain: x / (1 + exp(-x)) * x2
      const float u = load_as_f32(x2, r * ldx2 + c, x2_dtype);
      v = __fmul_rn(__fdiv_rn(v, __fadd_rn(expf(-v), 1.0f)), u);
    }
    split_store(v, hi, lo, r * k + c);
  }
}

// RMS prologue: one block per row (256 to 1024 threads); the row is staged in shared memory, its
// sum of squares reduced as cb_rmsnorm reduces it, then normalised, rounded
// to dt_out and split into the planes.
__global__ void __launch_bounds__(1024) rows_rms_planes_kernel(const void* x, int x_dtype, long long ldx, long long k,
                                                               const void* w, int w_dtype, NormSpec n, int dt_out,
                                                               __nv_bfloat16* hi, __nv_bfloat16* lo) {
  extern __shared__ float row[];
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const long long r = blockIdx.x;
  const int width = static_cast<int>(k);
  for (int i = threadIdx.x; i < width; i += blockDim.x) row[i] = load_as_f32(x, r * ldx + i, x_dtype);
  __syncthreads();
  const float d = norm_finish_d(n, norm_block_sum(n, row, width, red));
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    split_store(norm_apply(n, row[i], d, load_as_f32(w, i, w_dtype), dt_out), hi, lo, r * k + i);
}

constexpr long long kTwoCtaBytes = 32LL << 20;

int padded_rows(long long rows) { return rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256; }

struct RowsPlan {
  int nb, tiles, kchunks, grid, max_parts;
  int ctas;  // resident CTAs per SM
  long long total, plane_elems, partial_floats;
};

// The CTA range holding flattened chunk f (host copy of cta_of).
long long host_cta_of(long long f, long long total, long long grid) { return ((f + 1) * grid + total - 1) / total - 1; }

RowsPlan plan_rows(const cb_gemm_rows_args& a, int sms) {
  RowsPlan r{};
  r.nb = padded_rows(a.rows);
  r.kchunks = static_cast<int>((a.k + kChunk - 1) / kChunk);
  for (int i = 0; i < a.n_w; ++i) r.tiles += static_cast<int>((a.w_rows[i] + kWTile - 1) / kWTile);
  r.total = static_cast<long long>(r.tiles) * r.kchunks;
  // persistent CTAs, each streaming an equal range: two per SM for at least
  // kTwoCtaBytes of weights (measured: 12-18 % faster at 46-235 MB, slower
  // at 23 MB and below), else one (a.splits > 0: that many CTAs)
  long long bytes = 0;
  for (int i = 0; i < a.n_w; ++i) bytes += a.w_rows[i] * a.k * 2;
  r.ctas = r.nb <= 64 && bytes >= kTwoCtaBytes ? 2 : 1;
  long long grid = a.splits > 0 ? a.splits : static_cast<long long>(r.ctas) * sms;
  if (grid > r.total) grid = r.total;
  if (grid < 1) grid = 1;
  r.grid = static_cast<int>(grid);
  r.max_parts = 1;
  for (long long t = 0; t < r.tiles; ++t) {
    const long long parts = host_cta_of((t + 1) * r.kchunks - 1, r.total, grid) - host_cta_of(t * r.kchunks, r.total, grid) + 1;
    if (parts > r.max_parts) r.max_parts = static_cast<int>(parts);
  }
  r.plane_elems = a.rows * a.k;
  r.partial_floats = r.max_parts > 1 ? static_cast<long long>(r.tiles) * r.max_parts * r.nb * kWTile : 0;
  return r;
}

template <int NB, int CTAS>
int launch_rows(const cb_gemm_rows_args& a, const RowsPlan& pl, cudaStream_t s) {
  using G = RowsShape<NB, CTAS>;
  __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(a.scratch);
  __nv_bfloat16* lo = hi + pl.plane_elems;
  if (a.x_mode == CB_ROWS_X_RMS) {
    const NormSpec n{a.divisor, a.eps, a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y};
    const size_t smem = static_cast<size_t>(a.k) * sizeof(float);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(rows_rms_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    // one block per row, up to 1024 threads: a few elements per thread (the row's chain is the cost)
    const unsigned threads = static_cast<unsigned>(a.k >= 4096 ? 1024 : a.k >= 2048 ? 512 : 256);
    const cudaError_t e = launch(rows_rms_planes_kernel, dim3(static_cast<unsigned>(a.rows)), dim3(threads), smem, s,
                                 a.pdl != 0, a.x, a.x_dtype, a.ldx, a.k, a.norm_w, a.norm_w_dtype, n, a.dt_out, hi,
                                 lo);
    CB_REQUIRE(e == cudaSuccess, "cb_gemm_rows: plane pass launch failed (%s)", cudaGetErrorString(e));
  } else {
    const dim3 pgrid(static_cast<unsigned>(a.rows), static_cast<unsigned>((a.k + 1023) / 1024));
    const cudaError_t e = launch(rows_planes_kernel, pgrid, dim3(256), 0, s, a.pdl != 0, a.x, a.x_dtype, a.ldx, a.k,
                                 a.x2, a.x2_dtype, a.ldx2, static_cast<int>(a.x_mode == CB_ROWS_X_SWIGLU), hi, lo);
    CB_REQUIRE(e == cudaSuccess, "cb_gemm_rows: plane pass launch failed (%s)", cudaGetErrorString(e));
  }
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
  p.total = pl.total;
  p.max_parts = pl.max_parts;
  // x that is exactly bf16 -- given as bf16, or the RMS prologue rounding to
  // bf16 -- splits into a zero lo plane: its MMAs would add exact zeros.  The
  // single MMA-issuing thread is what bounds a few-row GEMM's stream (each
  // tcgen05.mma takes it tens of cycles to issue), so they are skipped.
  p.lo_plane = !((a.x_mode == CB_ROWS_X_RMS && a.dt_out == CB_BF16) ||
                 (a.x_mode == CB_ROWS_X_PLAIN && a.x_dtype == CB_BF16));
  // partials after the planes, 16-byte aligned
  const uintptr_t after = reinterpret_cast<uintptr_t>(lo + pl.plane_elems);
  p.partial = reinterpret_cast<float*>((after + 15) & ~static_cast<uintptr_t>(15));
  p.counters = a.counters;
  p.error_flag = a.error_flag;
  p.residual = a.residual;
  p.ldr = a.ldr;
  auto kernel = gemm_rows_kernel<NB, CTAS>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  if (e == cudaSuccess)
    e = launch(kernel, dim3(static_cast<unsigned>(pl.grid)), dim3(kRowsThreads), static_cast<size_t>(G::kSmem), s,
               a.pdl != 0, mw[0], mw[1], mw[2], mxh, mxl, p);
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
  return (planes + 15) / 16 * 16 + pl.partial_floats * 4 + 16;
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
  CB_REQUIRE(a->x_mode == CB_ROWS_X_PLAIN || a->x_mode == CB_ROWS_X_RMS || a->x_mode == CB_ROWS_X_SWIGLU,
             "gemm_rows: unknown x mode %d", a->x_mode);
  if (a->x_mode == CB_ROWS_X_RMS)
    CB_REQUIRE(a->norm_w != nullptr && a->k <= 49152 && a->divisor != 0.0f, "gemm_rows: RMS prologue needs norm_w");
  if (a->x_mode == CB_ROWS_X_SWIGLU)
    CB_REQUIRE(a->x2 != nullptr && (a->x2_dtype == CB_F32 || a->x2_dtype == CB_BF16),
               "gemm_rows: SwiGLU prologue needs x2");
  if (a->residual != nullptr)
    CB_REQUIRE(a->n_w == 1 && a->ldr >= a->w_rows[0], "gemm_rows: a residual epilogue takes one weight");
  for (int i = 0; i < a->n_w; ++i) {
    CB_REQUIRE(a->w[i] != nullptr && aligned16(a->w[i]) && a->out[i] != nullptr, "gemm_rows: weight %d", i);
    CB_REQUIRE(a->w_rows[i] > 0 && a->w_rows[i] < (1LL << 31) && a->ldo[i] >= a->w_rows[i],
               "gemm_rows: weight %d shape", i);
  }
  const RowsPlan pl = plan_rows(*a, sm_count_cached());
  CB_REQUIRE(pl.max_parts == 1 || a->counters != nullptr, "gemm_rows: split tiles need counters");
  CB_REQUIRE(pl.total < (1LL << 40) && pl.tiles < (1 << 30), "gemm_rows: too many tiles");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (pl.nb) {
    case 16: return pl.ctas == 2 ? launch_rows<16, 2>(*a, pl, s) : launch_rows<16, 1>(*a, pl, s);
    case 32: return pl.ctas == 2 ? launch_rows<32, 2>(*a, pl, s) : launch_rows<32, 1>(*a, pl, s);
    case 64: return pl.ctas == 2 ? launch_rows<64, 2>(*a, pl, s) : launch_rows<64, 1>(*a, pl, s);
    case 128: return launch_rows<128, 1>(*a, pl, s);
    default: return launch_rows<256, 1>(*a, pl, s);
  }
}

}  // extern "C"

// Tensor-core attention for prefill (and verify blocks): cb_sdpa_tc.
//
// The same result as cb_sdpa -- out = softmax(q k^T / divisor + mask) v with
// grouped-query heads (chomikgrad/llama.py:332-369) -- computed flash-style
// with tcgen05 MMAs:
//  * a pre-pass writes q, k and v as bf16 hi/lo planes (hi = bf16(x),
//    lo = bf16(x - hi)); v is stored transposed (head_size x keys) so every
//    MMA operand is K-major;
//  * one CTA per (128-query tile, head, batch): warp 0 streams K/V tiles with
//    TMA into two stages, warp 1 issues the MMAs -- S = q k^T as
//    qh.kh + qh.kl + ql.kh into a double-buffered TMEM S, and O_tile = p v as
//    ph.vh + ph.vl + pl.vh into TMEM -- and warps 2-9 run the softmax, two
//    threads per query row (each half of the row's keys and of its output
//    dims; two warps per scheduler, so one warp's latency hides behind the
//    other's work): they read S from TMEM into registers, apply the divisor
//    and the mask, run the online softmax in float32 (the halves swap tile
//    maxima through shared memory), write p as bf16 hi/lo planes into
//    shared memory (swizzled like a TMA tile) and fold each O_tile into a
//    float32 accumulator in registers;
//  * with CB_CAUSAL_SKIP, key tiles that lie entirely above the diagonal are
//    skipped; the caller asserts the mask there is <= -5000, where
//    exp(score - row max) underflows to 0 in float32 for any row whose
//    scores span less than ~4900, so the skipped terms are the zeros the
//    full softmax would add; with CB_CAUSAL_ZERO_BELOW as well, the mask is
//    exactly 0 at and below the diagonal and is read only on the diagonal
//    tiles (adding 0 changes nothing).
// Exponentials use the __expf intrinsic (a few ulp): p only enters the MMAs
// through its bf16 hi/lo planes.
// The three-product split keeps every product to about 2^-16 of |q||k| (and
// |p||v|); accumulation is float32.
//
// Every wait is bounded (sync.cuh); on a timeout the kernel records an error,
// lets its copies land and its MMAs finish, frees TMEM and returns.
#include "tc_core.cuh"

namespace cb {
namespace {

using namespace tc;

constexpr int kBQ = 128;                 // query rows per CTA = TMEM lanes
constexpr int kAttnTcThreads = 320;      // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr int kPlanesRows = 64;          // rows per pre-pass block

template <int HD>
struct AttnShape {
  static constexpr int kBK = 8192 / HD;           // keys per tile (128 for HD 64, 64 for HD 128)
  static constexpr int kChunksD = HD / kChunk;    // 64-element chunks of a q/k row
  static constexpr int kChunksK = kBK / kChunk;   // 64-key chunks of a p row / v^T row
  static constexpr int kQPlane = kBQ * HD * 2;
  static constexpr int kKPlane = kBK * HD * 2;
  static constexpr int kVPlane = HD * kBK * 2;
  static constexpr int kPPlane = kBQ * kBK * 2;
  static constexpr int kStage = 2 * kKPlane + 2 * kVPlane;
  static constexpr int kStageOff = 2 * kQPlane;
  static constexpr int kPOff = kStageOff + 2 * kStage;
  static constexpr int kSmem = kPOff + 2 * kPPlane + 1024;  // + alignment of the swizzled tiles
  static constexpr int kOCol = 2 * kBK;                     // TMEM: S buffers at 0 and kBK, O_tile after
  static constexpr int kXCol = kOCol + HD;                  // 4 columns: [tile parity][half] exchange slots
  static constexpr int kTmemCols = kXCol + 4 <= 256 ? 256 : 512;
  static_assert(kSmem <= 227 * 1024 - 256, "shared memory");
};

struct AttnTcParams {
  const void* mask;
  int mask_dtype;
  long long mask_offset;
  long long mask_strides[4];
  float* out;  // (batch, heads, tq, head_size), element strides out_s* (d contiguous)
  long long out_sb, out_sh, out_st;
  int heads, kv_heads, tq, tk, tq_pad, tk_pad;
  float divisor, inv_divisor;
  int div_pow2;       // divisor is a power of two: x * inv_divisor == x / divisor exactly
  int causal_offset;  // key tiles past query + causal_offset are skipped
  int zero_below;     // the mask is exactly 0 at keys <= query + causal_offset: not read there
  int* error_flag;
};

__device__ __forceinline__ void flag_error(int* error_flag, int code) {
  if (error_flag != nullptr) atomicCAS(error_flag, 0, code);
}

template <int HD>
__global__ void __launch_bounds__(kAttnTcThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap map_qh, const __grid_constant__ CUtensorMap map_ql,
                   const __grid_constant__ CUtensorMap map_kh, const __grid_constant__ CUtensorMap map_kl,
                   const __grid_constant__ CUtensorMap map_vh, const __grid_constant__ CUtensorMap map_vl,
                   const AttnTcParams p) {
  using S = AttnShape<HD>;
  constexpr int kBK = S::kBK;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t kv_full[2];
  __shared__ __align__(8) uint64_t kv_empty[2];
  __shared__ __align__(8) uint64_t s_full[2];
  __shared__ __align__(8) uint64_t p_full;
  __shared__ __align__(8) uint64_t o_full;
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ __align__(8) uint64_t pair_bar[4];  // the two softmax warps of a TMEM lane quarter
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest (most keys) tiles first
  const int q0 = qt * kBQ;
  const int kvh = h / (p.heads / p.kv_heads);
  const int q_row0 = (b * p.heads + h) * p.tq_pad + q0;
  const int k_row0 = (b * p.kv_heads + kvh) * p.tk_pad;
  const int v_row0 = (b * p.kv_heads + kvh) * HD;
  const long long last = min(static_cast<long long>(p.tk) - 1, static_cast<long long>(q0) + kBQ - 1 + p.causal_offset);
  const int n_tiles = last < 0 ? 1 : static_cast<int>(last / kBK) + 1;

  if (warp == 0) tmem_alloc(&tmem_base, S::kTmemCols);
  if (threadIdx.x == 32) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
      mbar_init(s_full + s, 1);
    }
    mbar_init(&p_full, 2 * kBQ);
    for (int q = 0; q < 4; ++q) mbar_init(pair_bar + q, 64);
    mbar_init(&o_full, 1);
    mbar_init(&mma_done, 1);
    mbar_fence_init();
    abort_flag = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      mbar_arrive_expect_tx(&q_full, static_cast<uint32_t>(2 * S::kQPlane));
#pragma unroll
      for (int c = 0; c < S::kChunksD; ++c) {
        tma_load_2d(smem + c * kBQ * kChunkRowBytes, &map_qh, c * kChunk, q_row0, &q_full);
        tma_load_2d(smem + S::kQPlane + c * kBQ * kChunkRowBytes, &map_ql, c * kChunk, q_row0, &q_full);
      }
      int j = 0;
      for (; j < n_tiles; ++j) {
        const int s = j & 1;
        if (j >= 2 && !wait_or_abort(kv_empty + s, static_cast<uint32_t>(((j >> 1) - 1) & 1), abort)) {
          flag_error(p.error_flag, CB_FLAG_WAIT_SLOT);
          *abort = 1;
          break;
        }
        unsigned char* st = smem + S::kStageOff + s * S::kStage;
        mbar_arrive_expect_tx(kv_full + s, static_cast<uint32_t>(S::kStage));
#pragma unroll
        for (int c = 0; c < S::kChunksD; ++c) {
          tma_load_2d(st + c * kBK * kChunkRowBytes, &map_kh, c * kChunk, k_row0 + j * kBK, kv_full + s);
          tma_load_2d(st + S::kKPlane + c * kBK * kChunkRowBytes, &map_kl, c * kChunk, k_row0 + j * kBK, kv_full + s);
        }
#pragma unroll
        for (int c = 0; c < S::kChunksK; ++c) {
          tma_load_2d(st + 2 * S::kKPlane + c * HD * kChunkRowBytes, &map_vh, j * kBK + c * kChunk, v_row0,
                      kv_full + s);
          tma_load_2d(st + 2 * S::kKPlane + S::kVPlane + c * HD * kChunkRowBytes, &map_vl, j * kBK + c * kChunk,
                      v_row0, kv_full + s);
        }
      }
      // drain: every copy issued lands before the block can exit
      bool drained = wait_short(&q_full, 0u);
      for (int t = j - 1; drained && t >= 0 && t >= j - 2; --t)
        drained = wait_short(kv_full + (t & 1), static_cast<uint32_t>((t >> 1) & 1));
      if (!drained) flag_error(p.error_flag, CB_FLAG_WAIT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t id_s = idesc_bf16(kBQ, kBK);
      constexpr uint32_t id_o = idesc_bf16(kBQ, HD);
      const unsigned char* qh = smem;
      const unsigned char* ql = smem + S::kQPlane;
      auto issue_s = [&](int jj) -> bool {
        const int s = jj & 1;
        if (!wait_or_abort(kv_full + s, static_cast<uint32_t>((jj >> 1) & 1), abort)) return false;
        fence_after();
        const unsigned char* kh = smem + S::kStageOff + s * S::kStage;
        const unsigned char* kl = kh + S::kKPlane;
        const uint32_t d = tmem + static_cast<uint32_t>(s * kBK);
#pragma unroll
        for (int c = 0; c < S::kChunksD; ++c)
#pragma unroll
          for (int kk = 0; kk < kChunk / kUmmaK; ++kk) {
            const int qo = c * kBQ * kChunkRowBytes + kk * kUmmaK * 2;
            const int ko = c * kBK * kChunkRowBytes + kk * kUmmaK * 2;
            const uint64_t dqh = sw128_desc(qh + qo), dql = sw128_desc(ql + qo);
            const uint64_t dkh = sw128_desc(kh + ko), dkl = sw128_desc(kl + ko);
            umma_bf16(d, dqh, dkh, id_s, (c | kk) != 0 ? 1u : 0u);
            umma_bf16(d, dqh, dkl, id_s, 1u);
            umma_bf16(d, dql, dkh, id_s, 1u);
          }
        umma_commit(s_full + s);
        return true;
      };
      bool ok = wait_or_abort(&q_full, 0u, abort) && (fence_after(), issue_s(0));
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!wait_or_abort(&p_full, static_cast<uint32_t>(j & 1), abort)) {
          ok = false;
          break;
        }
        fence_after();
        const unsigned char* ph = smem + S::kPOff;
        const unsigned char* pl = ph + S::kPPlane;
        const unsigned char* vh = smem + S::kStageOff + (j & 1) * S::kStage + 2 * S::kKPlane;
        const unsigned char* vl = vh + S::kVPlane;
        const uint32_t d = tmem + static_cast<uint32_t>(S::kOCol);
#pragma unroll
        for (int c = 0; c < S::kChunksK; ++c)
#pragma unroll
          for (int kk = 0; kk < kChunk / kUmmaK; ++kk) {
            const int po = c * kBQ * kChunkRowBytes + kk * kUmmaK * 2;
            const int vo = c * HD * kChunkRowBytes + kk * kUmmaK * 2;
            const uint64_t dph = sw128_desc(ph + po), dpl = sw128_desc(pl + po);
            const uint64_t dvh = sw128_desc(vh + vo), dvl = sw128_desc(vl + vo);
            umma_bf16(d, dph, dvh, id_o, (c | kk) != 0 ? 1u : 0u);
            umma_bf16(d, dph, dvl, id_o, 1u);
            umma_bf16(d, dpl, dvh, id_o, 1u);
          }
        umma_commit(&o_full);
        umma_commit(kv_empty + (j & 1));
      }
      if (!ok) {
        flag_error(p.error_flag, CB_FLAG_WAIT_DATA);
        *abort = 1;
      }
      umma_commit(&mma_done);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---- softmax: two threads per query row ----
    // Warp w (2..9) reads TMEM lane quarter w % 4; the two warps of a
    // quarter split each row: half h owns S columns [h kBK/2, (h+1) kBK/2)
    // of every tile and O dims [h HD/2, (h+1) HD/2).  The halves swap their
    // tile maxima (and at the end their sums) through shared memory, paced
    // by the quarter's mbarrier (64 arrivals per phase, bounded waits).
    constexpr int kCols = kBK / 2;  // S columns of this thread
    constexpr int kDims = HD / 2;   // O dims of this thread
    static_assert(kCols % 32 == 0 && kDims % 32 == 0, "32-column TMEM loads");
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int qi = q0 + r;
    const int col0 = half * kCols;
    const int dim0 = half * kDims;
    const uint32_t lanes = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    uint64_t* pair = pair_bar + quarter;
    const long long mrow = p.mask_offset + b * p.mask_strides[0] + h * p.mask_strides[1] +
                           static_cast<long long>(min(qi, p.tq - 1)) * p.mask_strides[2];
    float o[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) o[d] = 0.0f;
    float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
    bool ok = true;
    auto fold = [&](int jj) -> bool {  // o = o * alpha_prev + O_tile(jj)
      if (!__all_sync(0xffffffffu, wait_or_abort(&o_full, static_cast<uint32_t>(jj & 1), abort))) return false;
      fence_after();
#pragma unroll
      for (int c0 = 0; c0 < kDims; c0 += 16) {  // 16 columns at a time: x[] is live meanwhile
        float v[16];
        tmem_load16(lanes + static_cast<uint32_t>(S::kOCol + dim0 + c0), v);
#pragma unroll
        for (int d = 0; d < 16; ++d) o[c0 + d] = fmaf(o[c0 + d], alpha_prev, v[d]);
      }
      return true;
    };
    for (int j = 0; j < n_tiles; ++j) {
      // warp-uniform outcome: the TMEM loads below are warp-wide (.sync.aligned)
      if (!__all_sync(0xffffffffu, wait_or_abort(s_full + (j & 1), static_cast<uint32_t>((j >> 1) & 1), abort))) {
        ok = false;
        break;
      }
      fence_after();
      float x[kCols];
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += 32)
        tmem_load32_nowait(lanes + static_cast<uint32_t>((j & 1) * kBK + col0 + c0), x + c0);
      tmem_wait_ld();
      reg_fence<kCols>(x);
      const int key0 = j * kBK + col0;
      const bool use_mask = p.mask != nullptr && !(p.zero_below && static_cast<long long>(j) * kBK + kBK - 1 <=
                                                                        static_cast<long long>(q0) + p.causal_offset);
      if (!use_mask && p.div_pow2 && key0 + kCols <= p.tk) {  // the common tile: a scale only
#pragma unroll
        for (int e = 0; e < kCols; ++e) x[e] *= p.inv_divisor;
      } else {
#pragma unroll
        for (int e = 0; e < kCols; ++e) {
          const int key = key0 + e;
          float v = p.div_pow2 ? x[e] * p.inv_divisor : __fdiv_rn(x[e], p.divisor);
          if (use_mask && key < p.tk) v = __fadd_rn(v, load_as_f32(p.mask, mrow + key * p.mask_strides[3], p.mask_dtype));
          x[e] = key < p.tk ? v : -INFINITY;
        }
      }
      float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < kCols; ++e) t4[e & 3] = fmaxf(t4[e & 3], x[e]);
      const float tmax_mine = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
      // swap tile maxima with the other half of the row through this lane's
      // TMEM exchange columns (slot by tile parity)
      tmem_store1(lanes + static_cast<uint32_t>(S::kXCol + (j & 1) * 2 + half), tmax_mine);
      tmem_wait_st();
      fence_before();
      mbar_arrive(pair);
      if (!__all_sync(0xffffffffu, wait_or_abort(pair, static_cast<uint32_t>(j & 1), abort))) {
        ok = false;
        break;
      }
      fence_after();
      const float tmax =
          fmaxf(tmax_mine, tmem_load1(lanes + static_cast<uint32_t>(S::kXCol + (j & 1) * 2 + (half ^ 1))));
      const float m_new = fmaxf(m, tmax);
      const float alpha = __expf(m - m_new);
      if (j > 0 && !fold(j - 1)) {  // O_tile of the previous key tile (p of that tile, max m)
        ok = false;
        break;
      }
      // p = exp(x - m_new) as bf16 hi/lo into the swizzled P planes (free: the
      // previous tile's p.v has completed)
      float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += 8) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float x0 = __expf(x[c0 + 2 * i] - m_new), x1 = __expf(x[c0 + 2 * i + 1] - m_new);
          s4[i] += x0 + x1;
          const __nv_bfloat162 hi = __floats2bfloat162_rn(x0, x1);
          const float2 hf = __bfloat1622float2(hi);
          const __nv_bfloat162 lo = __floats2bfloat162_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
          hw[i] = *reinterpret_cast<const uint32_t*>(&hi);
          lw[i] = *reinterpret_cast<const uint32_t*>(&lo);
        }
        const int kin = col0 + c0;
        unsigned char* dst = smem + S::kPOff + (kin / kChunk) * kBQ * kChunkRowBytes + swizzle_offset(r, (kin % kChunk) / 8);
        *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(dst + S::kPPlane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      l = l * alpha + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
      m = m_new;
      alpha_prev = alpha;
      fence_async_shared();
      fence_before();
      mbar_arrive(&p_full);
    }
    if (ok && fold(n_tiles - 1)) {
      // the row's sum is the two halves' sums (both scaled to the same max)
      tmem_store1(lanes + static_cast<uint32_t>(S::kXCol + (n_tiles & 1) * 2 + half), l);
      tmem_wait_st();
      fence_before();
      mbar_arrive(pair);
      ok = __all_sync(0xffffffffu, wait_or_abort(pair, static_cast<uint32_t>(n_tiles & 1), abort));
      if (ok) {
        fence_after();
        const float lt = l + tmem_load1(lanes + static_cast<uint32_t>(S::kXCol + (n_tiles & 1) * 2 + (half ^ 1)));
        if (qi < p.tq) {
          float* dst = p.out + b * p.out_sb + h * p.out_sh + static_cast<long long>(qi) * p.out_st + dim0;
#pragma unroll
          for (int d = 0; d < kDims; d += 4)
            *reinterpret_cast<float4*>(dst + d) = make_float4(__fdiv_rn(o[d], lt), __fdiv_rn(o[d + 1], lt),
                                                             __fdiv_rn(o[d + 2], lt), __fdiv_rn(o[d + 3], lt));
        }
      }
    } else {
      ok = false;
    }
    if (!ok) {
      flag_error(p.error_flag, CB_FLAG_WAIT_DATA);
      *abort = 1;
    }
  }
  __syncwarp();
  fence_before();
  __syncthreads();
  if (warp == 0) {
    // TMEM is freed only after the MMAs that write it have completed
    if (!wait_short(&mma_done, 0u) && lane == 0) flag_error(p.error_flag, CB_FLAG_WAIT_DRAIN);
    fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// q, k, v (any strides, float32/bf16/f16) -> bf16 hi/lo planes: q and k as
// (batch * heads, t_pad, HD) rows, v transposed as (batch * kv_heads * HD,
// tk_pad); rows past the sequence are zero.  blockIdx.z selects q, k or v.
template <int HD>
__global__ void __launch_bounds__(256) attn_planes_kernel(const cb_sdpa_args a, int tq_pad, int tk_pad,
                                                          __nv_bfloat16* qh, __nv_bfloat16* ql, __nv_bfloat16* kh,
                                                          __nv_bfloat16* kl, __nv_bfloat16* vh, __nv_bfloat16* vl) {
  __shared__ float tile[kPlanesRows][HD + 1];
  const int which = blockIdx.z;
  const int nheads = which == 0 ? static_cast<int>(a.heads) : static_cast<int>(a.kv_heads);
  const int maxh = static_cast<int>(a.heads > a.kv_heads ? a.heads : a.kv_heads);
  const int b = blockIdx.y / maxh, hh = blockIdx.y % maxh;
  const int t_pad = which == 0 ? tq_pad : tk_pad;
  const long long tlen = which == 0 ? a.tq : a.tk;
  const int t0 = blockIdx.x * kPlanesRows;
  if (hh >= nheads || t0 >= t_pad) return;
  const void* src = which == 0 ? a.q : which == 1 ? a.k : a.v;
  const int dt = which == 0 ? a.q_dtype : which == 1 ? a.k_dtype : a.v_dtype;
  const long long off = which == 0 ? a.q_offset : which == 1 ? a.k_offset : a.v_offset;
  const long long* st = which == 0 ? a.q_strides : which == 1 ? a.k_strides : a.v_strides;
  const long long base = off + b * st[0] + hh * st[1];
  __nv_bfloat16* hi = which == 0 ? qh : kh;
  __nv_bfloat16* lo = which == 0 ? ql : kl;
  const long long plane_row0 = (static_cast<long long>(b) * nheads + hh) * t_pad + t0;
  for (int i = threadIdx.x; i < kPlanesRows * HD; i += blockDim.x) {
    const int tr = i / HD, d = i % HD;
    const long long t = t0 + tr;
    const float x = t < tlen ? load_as_f32(src, base + t * st[2] + d * st[3], dt) : 0.0f;
    if (which < 2) {
      const __nv_bfloat16 xh = __float2bfloat16_rn(x);
      hi[(plane_row0 + tr) * HD + d] = xh;
      lo[(plane_row0 + tr) * HD + d] = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(xh)));
    } else {
      tile[tr][d] = x;
    }
  }
  if (which < 2) return;
  __syncthreads();
  const long long vrow0 = (static_cast<long long>(b) * nheads + hh) * HD;
  for (int i = threadIdx.x; i < kPlanesRows * HD; i += blockDim.x) {
    const int d = i / kPlanesRows, tr = i % kPlanesRows;
    const float x = tile[tr][d];
    const __nv_bfloat16 xh = __float2bfloat16_rn(x);
    vh[(vrow0 + d) * tk_pad + t0 + tr] = xh;
    vl[(vrow0 + d) * tk_pad + t0 + tr] = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(xh)));
  }
}

long long round_up(long long x, long long m) { return (x + m - 1) / m * m; }

struct Planes {
  long long q, k;  // elements of one q plane / one k (= v) plane
};

Planes planes_of(const cb_sdpa_args& a) {
  const long long tq_pad = round_up(a.tq, kBQ), tk_pad = round_up(a.tk, kBQ);
  return {a.batch * a.heads * tq_pad * a.head_size, a.batch * a.kv_heads * tk_pad * a.head_size};
}

template <int HD>
int launch_sdpa_tc(const cb_sdpa_args& a, int causal, void* scratch, int* error_flag, cudaStream_t s) {
  using Sh = AttnShape<HD>;
  const int tq_pad = static_cast<int>(round_up(a.tq, kBQ)), tk_pad = static_cast<int>(round_up(a.tk, kBQ));
  const Planes n = planes_of(a);
  __nv_bfloat16* qh = static_cast<__nv_bfloat16*>(scratch);
  __nv_bfloat16* ql = qh + n.q;
  __nv_bfloat16* kh = ql + n.q;
  __nv_bfloat16* kl = kh + n.k;
  __nv_bfloat16* vh = kl + n.k;
  __nv_bfloat16* vl = vh + n.k;
  const long long maxh = a.heads > a.kv_heads ? a.heads : a.kv_heads;
  const dim3 pgrid(static_cast<unsigned>((tq_pad > tk_pad ? tq_pad : tk_pad) / kPlanesRows),
                   static_cast<unsigned>(a.batch * maxh), 3);
  attn_planes_kernel<HD><<<pgrid, 256, 0, s>>>(a, tq_pad, tk_pad, qh, ql, kh, kl, vh, vl);
  CB_REQUIRE(cudaGetLastError() == cudaSuccess, "cb_sdpa_tc: plane pass launch failed");

  CUtensorMap m_qh, m_ql, m_kh, m_kl, m_vh, m_vl;
  const long long qrows = a.batch * a.heads * tq_pad, krows = a.batch * a.kv_heads * tk_pad;
  const long long vrows = a.batch * a.kv_heads * HD;
  CB_REQUIRE(make_map(&m_qh, qh, qrows, HD, HD, kBQ) && make_map(&m_ql, ql, qrows, HD, HD, kBQ) &&
                 make_map(&m_kh, kh, krows, HD, HD, Sh::kBK) && make_map(&m_kl, kl, krows, HD, HD, Sh::kBK) &&
                 make_map(&m_vh, vh, vrows, tk_pad, tk_pad, HD) && make_map(&m_vl, vl, vrows, tk_pad, tk_pad, HD),
             "cb_sdpa_tc: tensor map encoding failed");

  AttnTcParams p{};
  p.mask = a.mask;
  p.mask_dtype = a.mask_dtype;
  p.mask_offset = a.mask_offset;
  for (int d = 0; d < 4; ++d) p.mask_strides[d] = a.mask_strides[d];
  p.out = a.out;
  const bool packed = a.out_strides[0] == 0 && a.out_strides[1] == 0 && a.out_strides[2] == 0;
  p.out_sb = packed ? a.heads * a.tq * HD : a.out_strides[0];
  p.out_sh = packed ? a.tq * HD : a.out_strides[1];
  p.out_st = packed ? HD : a.out_strides[2];
  p.heads = static_cast<int>(a.heads);
  p.kv_heads = static_cast<int>(a.kv_heads);
  p.tq = static_cast<int>(a.tq);
  p.tk = static_cast<int>(a.tk);
  p.tq_pad = tq_pad;
  p.tk_pad = tk_pad;
  p.divisor = a.divisor;
  int exponent = 0;
  p.div_pow2 = std::frexp(a.divisor, &exponent) == 0.5f;
  p.inv_divisor = 1.0f / a.divisor;
  p.causal_offset = (causal & CB_CAUSAL_SKIP) ? static_cast<int>(a.tk - a.tq) : static_cast<int>(a.tk);
  p.zero_below = (causal & CB_CAUSAL_SKIP) && (causal & CB_CAUSAL_ZERO_BELOW);
  p.error_flag = error_flag;

  auto kernel = attn_tc_kernel<HD>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmem);
  if (e == cudaSuccess) {
    const dim3 grid(static_cast<unsigned>(tq_pad / kBQ), static_cast<unsigned>(a.heads),
                    static_cast<unsigned>(a.batch));
    kernel<<<grid, kAttnTcThreads, Sh::kSmem, s>>>(m_qh, m_ql, m_kh, m_kl, m_vh, m_vl, p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_error("cb_sdpa_tc: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_sdpa_tc");
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

long long cb_sdpa_tc_scratch(const cb_sdpa_args* a) {
  if (a == nullptr || a->batch <= 0 || a->heads <= 0 || a->kv_heads <= 0 || a->tq <= 0 || a->tk <= 0) return 0;
  const Planes n = planes_of(*a);
  return (2 * n.q + 4 * n.k) * 2;
}

int cb_sdpa_tc(const cb_sdpa_args* a, int causal, void* scratch, int* error_flag, cb_stream_t stream) {
  CB_REQUIRE(a != nullptr && a->q != nullptr && a->k != nullptr && a->v != nullptr && a->out != nullptr,
             "sdpa_tc: q, k, v and out are required");
  CB_REQUIRE(a->head_size == 64 || a->head_size == 128, "sdpa_tc: head_size %lld (64 or 128 supported)",
             a->head_size);
  CB_REQUIRE(a->batch > 0 && a->heads > 0 && a->kv_heads > 0 && a->heads % a->kv_heads == 0,
             "sdpa_tc: heads %lld must be a multiple of kv_heads %lld", a->heads, a->kv_heads);
  CB_REQUIRE(a->tq > 0 && a->tk > 0 && a->tk < (1LL << 24) && a->tq < (1LL << 24), "sdpa_tc: bad sequence lengths");
  CB_REQUIRE(a->batch * a->heads * round_up(a->tq, kBQ) < (1LL << 31) &&
                 a->batch * a->kv_heads * round_up(a->tk, kBQ) < (1LL << 31) && a->batch < 65536 && a->heads < 65536,
             "sdpa_tc: problem too large");
  CB_REQUIRE(a->divisor != 0.0f && std::isfinite(a->divisor), "sdpa_tc: bad divisor");
  CB_REQUIRE(scratch != nullptr && aligned16(scratch) && aligned16(a->out), "sdpa_tc: scratch and out must be 16-byte aligned");
  CB_REQUIRE((a->out_strides[3] == 0 || a->out_strides[3] == 1) && a->out_strides[0] % 4 == 0 &&
                 a->out_strides[1] % 4 == 0 && a->out_strides[2] % 4 == 0,
             "sdpa_tc: out rows must be contiguous and 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return a->head_size == 64 ? launch_sdpa_tc<64>(*a, causal, scratch, error_flag, s)
                            : launch_sdpa_tc<128>(*a, causal, scratch, error_flag, s);
}

}  // extern "C"

// GEMV building blocks shared by the streaming GEMV kernel (gemv.cu) and the
// decode-step megakernel (decode_step.cu): weight-row addressing, the x
// "planes" chunk reader and the multi-row shared-memory dot product.
#pragma once

#include "norm.cuh"
#include "sync.cuh"

namespace cb {

constexpr int kMaxStageRows = 8;  // rows multiplied together per stage

// Weight row of logical unit u.  SwiGLU interleaves gate (even) / up (odd).
__device__ __forceinline__ const char* unit_row(const cb_gemv_args& a, long long u, long long row_bytes) {
  if (a.epilogue == CB_EPI_SILU_MUL)
    return static_cast<const char*>(a.w[u & 1]) + (u >> 1) * row_bytes;
  if (u < a.w_rows[0]) return static_cast<const char*>(a.w[0]) + u * row_bytes;
  u -= a.w_rows[0];
  if (u < a.w_rows[1]) return static_cast<const char*>(a.w[1]) + u * row_bytes;
  u -= a.w_rows[1];
  return static_cast<const char*>(a.w[2]) + u * row_bytes;
}


// x for chunk c (VE elements) from the two planes: xa = elements 0..3 of each
// chunk, xb = 4..7 (bf16 chunks only).  Consecutive lanes read consecutive
// 16-byte words: no bank conflicts.
template <typename WT>
struct Chunk;
template <>
struct Chunk<uint16_t> {
  static constexpr int kElems = 8;
  float4 a, b;
  __device__ void load(const float4* xa, const float4* xb, long long c) {
    a = xa[c];
    b = xb[c];
  }
  __device__ float dot(const uint4& w, float acc) const {
    acc = fmaf(__uint_as_float(w.x << 16), a.x, acc);
    acc = fmaf(__uint_as_float(w.x & 0xffff0000u), a.y, acc);
    acc = fmaf(__uint_as_float(w.y << 16), a.z, acc);
    acc = fmaf(__uint_as_float(w.y & 0xffff0000u), a.w, acc);
    acc = fmaf(__uint_as_float(w.z << 16), b.x, acc);
    acc = fmaf(__uint_as_float(w.z & 0xffff0000u), b.y, acc);
    acc = fmaf(__uint_as_float(w.w << 16), b.z, acc);
    acc = fmaf(__uint_as_float(w.w & 0xffff0000u), b.w, acc);
    return acc;
  }
};
template <>
struct Chunk<float> {
  static constexpr int kElems = 4;
  float4 a;
  __device__ void load(const float4* xa, const float4*, long long c) { a = xa[c]; }
  __device__ float dot(const uint4& w, float acc) const {
    acc = fmaf(__uint_as_float(w.x), a.x, acc);
    acc = fmaf(__uint_as_float(w.y), a.y, acc);
    acc = fmaf(__uint_as_float(w.z), a.z, acc);
    acc = fmaf(__uint_as_float(w.w), a.w, acc);
    return acc;
  }
};

__device__ __forceinline__ void consumers_sync(int n) {
  asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory");
}

// Winner of the per-block argmax partials [0, n) (written by other blocks,
// read through L2), merged by all `nthreads` consumer threads: strided
// loads, warp shuffles, then thread 0 over the warps.  argmax_better is a
// total order (NaN first, then the larger value, then the lower index), so
// the merge order does not change the result.  Valid in thread 0; red_v and
// red_i hold nthreads / 32 entries.
__device__ __forceinline__ long long argmax_merge(const float* vals, const long long* idx, int n, int tid,
                                                  int nthreads, float* red_v, long long* red_i) {
  float bv = 0.0f;
  long long bi = -1;
  for (int c = tid; c < n; c += nthreads) {
    const long long ci = __ldcg(idx + c);
    const float cv = __ldcg(vals + c);
    if (ci >= 0 && (bi < 0 || argmax_better(cv, ci, bv, bi))) {
      bv = cv;
      bi = ci;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, off);
    const long long oi = __shfl_down_sync(0xffffffffu, bi, off);
    if (oi >= 0 && (bi < 0 || argmax_better(ov, oi, bv, bi))) {
      bv = ov;
      bi = oi;
    }
  }
  if ((tid & 31) == 0) {
    red_v[tid >> 5] = bv;
    red_i[tid >> 5] = bi;
  }
  consumers_sync(nthreads);
  if (tid == 0) {
    bv = 0.0f;
    bi = -1;
    for (int w = 0; w < nthreads / 32; ++w) {
      if (red_i[w] >= 0 && (bi < 0 || argmax_better(red_v[w], red_i[w], bv, bi))) {
        bv = red_v[w];
        bi = red_i[w];
      }
    }
  }
  return bi;
}

// R rows of one stage against x: totals[r] (valid on every lane).
template <typename WT, int R>
__device__ __forceinline__ void stage_dot(const unsigned char* stage, const long long* row_at,
                                          long long row_bytes, const float4* xa, const float4* xb,
                                          long long chunks, int lane, float* totals) {
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.0f;
  const uint4* rows[R];
#pragma unroll
  for (int r = 0; r < R; ++r) rows[r] = reinterpret_cast<const uint4*>(stage + row_at[r] * row_bytes);
  long long c = lane;
  // two chunks per iteration: twice the shared loads in flight
  for (; c + 32 < chunks; c += 64) {
    Chunk<WT> x0, x1;
    x0.load(xa, xb, c);
    x1.load(xa, xb, c + 32);
    uint4 w0[R], w1[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      w0[r] = rows[r][c];
      w1[r] = rows[r][c + 32];
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = x1.dot(w1[r], x0.dot(w0[r], acc[r]));
  }
  if (c < chunks) {
    Chunk<WT> x;
    x.load(xa, xb, c);
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = x.dot(rows[r][c], acc[r]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) totals[r] = warp_sum(acc[r]);
}


}  // namespace cb

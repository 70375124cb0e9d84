// RMSNorm arithmetic shared by the standalone rms_norm kernel and the fused
// GEMV prologue.
//
// The reference builds rms_norm from portable ops (llama.py:279-287):
//   sq   = x * x                (dtype dt_sq)
//   s    = sum(sq, axis=-1)     (dt_sum; NumPy accumulates bf16/f16 in order,
//                                rounding after every add)
//   mean = s / divisor          (dt_mean; divisor is a constant leaf)
//   t    = mean + eps           (dt_t;    eps is a constant leaf)
//   d    = sqrt(t)              (dt_d)
//   y    = x / d                (dt_y)
//   out  = y * w                (output dtype)
// Each function below reproduces one stage with the same roundings.
#pragma once

#include "common.cuh"

namespace cb {

struct NormSpec {
  float divisor, eps;
  int dt_sq, dt_sum, dt_mean, dt_t, dt_d, dt_y;
};

__device__ __forceinline__ float norm_finish_d(const NormSpec& n, float sum) {
  const float mean = round_to(__fdiv_rn(sum, n.divisor), n.dt_mean);
  const float t = round_to(__fadd_rn(mean, n.eps), n.dt_t);
  return round_to(__fsqrt_rn(t), n.dt_d);
}

__device__ __forceinline__ float norm_apply(const NormSpec& n, float x, float d, float w, int dt_out) {
  const float y = round_to(__fdiv_rn(x, d), n.dt_y);
  return round_to(__fmul_rn(y, w), dt_out);
}

// Sum of squares of row[0:width) (float32 values already in shared memory)
// for the whole block; returns the sum to every thread.  `red` needs
// blockDim.x/32 floats.  Sequential (index order, rounded) when dt_sum is a
// 16-bit float, else a tree reduction.
__device__ __forceinline__ float norm_block_sum(const NormSpec& n, const float* row, int width,
                                                float* red) {
  __shared__ float result;
  if (n.dt_sum != CB_F32) {
    if (threadIdx.x == 0) {
      float acc = round_to(__fmul_rn(row[0], row[0]), n.dt_sq);
      for (int i = 1; i < width; ++i) {
        const float sq = round_to(__fmul_rn(row[i], row[i]), n.dt_sq);
        acc = round_to(__fadd_rn(acc, sq), n.dt_sum);
      }
      result = acc;
    }
    __syncthreads();
    return result;
  }
  float part = 0.0f;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float sq = round_to(__fmul_rn(row[i], row[i]), n.dt_sq);
    part = __fadd_rn(part, sq);
  }
  part = warp_sum(part);
  const int warp = threadIdx.x >> 5, lanes = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.0f;
    for (int w = 0; w < lanes; ++w) acc += red[w];
    result = acc;
  }
  __syncthreads();
  return result;
}

}  // namespace cb

// Generic batched matmul with broadcasting and arbitrary (strided) operands.
// SIMT float32 accumulation: this is the correctness path for any MATMUL the
// plugin does not pattern-match onto a fused kernel.
#include "common.cuh"

namespace cb {
namespace {

constexpr int kTileM = 64, kTileN = 64, kTileK = 16, kThreads = 256;

__device__ __forceinline__ void batch_offsets(const cb_matmul_args& a, long long batch,
                                              long long* ao, long long* bo) {
  long long oa = a.a_offset, ob = a.b_offset;
  for (int d = a.batch_ndim - 1; d >= 0; --d) {
    const long long c = batch % a.batch_shape[d];
    batch /= a.batch_shape[d];
    oa += c * a.a_bstride[d];
    ob += c * a.b_bstride[d];
  }
  *ao = oa;
  *bo = ob;
}

__global__ void __launch_bounds__(kThreads) matmul_kernel(const cb_matmul_args a, long long batches) {
  __shared__ float As[kTileK][kTileM + 4];
  __shared__ float Bs[kTileK][kTileN + 4];
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const long long m0 = static_cast<long long>(blockIdx.y) * kTileM;
  const long long n0 = static_cast<long long>(blockIdx.x) * kTileN;
  for (long long batch = blockIdx.z; batch < batches; batch += gridDim.z) {
    long long ao, bo;
    batch_offsets(a, batch, &ao, &bo);
    float acc[4][4] = {};
    for (long long k0 = 0; k0 < a.k; k0 += kTileK) {
#pragma unroll
      for (int i = 0; i < (kTileM * kTileK) / kThreads; ++i) {
        const int e = tid + i * kThreads;
        const int row = e / kTileK, col = e % kTileK;
        const long long gm = m0 + row, gk = k0 + col;
        As[col][row] = (gm < a.m && gk < a.k) ? load_as_f32(a.a, ao + gm * a.a_rs + gk * a.a_cs, a.a_dtype)
                                              : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < (kTileN * kTileK) / kThreads; ++i) {
        const int e = tid + i * kThreads;
        const int row = e / kTileN, col = e % kTileN;
        const long long gk = k0 + row, gn = n0 + col;
        Bs[row][col] = (gk < a.k && gn < a.n) ? load_as_f32(a.b, bo + gk * a.b_rs + gn * a.b_cs, a.b_dtype)
                                              : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kTileK; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      __syncthreads();
    }
    const long long cbase = batch * a.m * a.n;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const long long gm = m0 + ty * 4 + i;
      if (gm >= a.m) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const long long gn = n0 + tx * 4 + j;
        if (gn < a.n) store_from_f32(a.c, cbase + gm * a.n + gn, a.c_dtype, acc[i][j]);
      }
    }
  }
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_matmul(const cb_matmul_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->batch_ndim >= 0 && a->batch_ndim <= CB_MM_MAX_BATCH, "matmul: too many batch dims");
  CB_REQUIRE(a->m >= 0 && a->n >= 0 && a->k >= 0, "matmul: negative size");
  long long batches = 1;
  for (int d = 0; d < a->batch_ndim; ++d) batches *= a->batch_shape[d];
  if (batches == 0 || a->m == 0 || a->n == 0) return CB_OK;
  const long long gx = (a->n + kTileN - 1) / kTileN, gy = (a->m + kTileM - 1) / kTileM;
  CB_REQUIRE(gy <= 65535 && gx <= 0x7fffffffLL, "matmul: matrix too large for the generic kernel");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy),
            static_cast<unsigned>(batches < 65535 ? batches : 65535));
  matmul_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(*a, batches);
  return check_launch("cb_matmul");
}

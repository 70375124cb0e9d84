// Standalone rms_norm and rope lowerings (prefill, block decode, and any
// graph whose norm/rope cannot be fused into a neighbouring kernel).
#include "norm.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ long long row_base(const cb_rmsnorm_args& a, long long r) {
  const long long src = a.x_index != nullptr ? load_index(a.x_index, r, a.x_index_dtype) : r;
  return a.x_offset + src * a.x_row_stride;
}

// One block per row; the row is staged as float32 in dynamic shared memory.
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const cb_rmsnorm_args a, NormSpec n) {
  extern __shared__ float row[];
  __shared__ float red[kThreads / 32];
  const long long r = blockIdx.x;
  const long long base = row_base(a, r);
  const int width = static_cast<int>(a.width);
  for (int i = threadIdx.x; i < width; i += blockDim.x) row[i] = load_as_f32(a.x, base + i, a.x_dtype);
  __syncthreads();
  float d;
  if (a.d_table != nullptr) {
    const long long src = a.x_index != nullptr ? load_index(a.x_index, r, a.x_index_dtype) : r;
    d = a.d_table[src];
  } else {
    d = norm_finish_d(n, norm_block_sum(n, row, width, red));
  }
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float w = load_as_f32(a.w, i, a.w_dtype);
    store_from_f32(a.out, r * a.width + i, a.out_dtype, norm_apply(n, row[i], d, w, a.out_dtype));
  }
}

// d for every row of a constant table; sequential sums run one row per thread.
__global__ void rmsnorm_table_seq_kernel(const cb_rmsnorm_args a, NormSpec n, float* d_out) {
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < a.rows;
       r += (long long)gridDim.x * blockDim.x) {
    const long long base = a.x_offset + r * a.x_row_stride;
    float x0 = load_as_f32(a.x, base, a.x_dtype);
    float acc = round_to(__fmul_rn(x0, x0), n.dt_sq);
    for (long long i = 1; i < a.width; ++i) {
      const float x = load_as_f32(a.x, base + i, a.x_dtype);
      acc = round_to(__fadd_rn(acc, round_to(__fmul_rn(x, x), n.dt_sq)), n.dt_sum);
    }
    d_out[r] = norm_finish_d(n, acc);
  }
}

__global__ void __launch_bounds__(kThreads) rmsnorm_table_par_kernel(const cb_rmsnorm_args a, NormSpec n,
                                                                    float* d_out) {
  extern __shared__ float row[];
  __shared__ float red[kThreads / 32];
  const long long r = blockIdx.x;
  const long long base = a.x_offset + r * a.x_row_stride;
  const int width = static_cast<int>(a.width);
  for (int i = threadIdx.x; i < width; i += blockDim.x) row[i] = load_as_f32(a.x, base + i, a.x_dtype);
  __syncthreads();
  const float d = norm_finish_d(n, norm_block_sum(n, row, width, red));
  if (threadIdx.x == 0) d_out[r] = d;
}

__global__ void rope_kernel(const cb_rope_args a) {
  const long long half = a.head_size / 2;
  const long long total = a.batch * a.heads * a.tokens * half;
  long long offset = 0;
  if (a.offset != nullptr) offset = load_index(a.offset, 0, a.offset_dtype);
  if (offset < 0 || offset >= a.n_offsets) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_POSITION);
    offset = offset < 0 ? 0 : a.n_offsets - 1;
  }
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long j = i % half;
    long long rest = i / half;
    const long long t = rest % a.tokens;
    rest /= a.tokens;
    const long long h = rest % a.heads;
    const long long b = rest / a.heads;
    const long long src = a.x_offset + b * a.x_strides[0] + h * a.x_strides[1] + t * a.x_strides[2];
    const float lo = load_as_f32(a.x, src + j * a.x_strides[3], a.x_dtype);
    const float hi = load_as_f32(a.x, src + (j + half) * a.x_strides[3], a.x_dtype);
    const long long tab = (offset * a.tokens + t) * half + j;
    const float c = a.cos_table[tab], s = a.sin_table[tab];
    const long long dst = ((b * a.heads + h) * a.tokens + t) * a.head_size;
    store_from_f32(a.out, dst + j, a.out_dtype, fmaf(-hi, s, __fmul_rn(lo, c)));
    store_from_f32(a.out, dst + j + half, a.out_dtype, fmaf(hi, c, __fmul_rn(lo, s)));
  }
}

inline NormSpec spec_of(const cb_rmsnorm_args& a) {
  return NormSpec{a.divisor, a.eps, a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y};
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_rmsnorm(const cb_rmsnorm_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->width > 0 && a->width <= 49152, "rms_norm: unsupported row width %lld", a->width);
  if (a->rows == 0) return CB_OK;
  CB_REQUIRE(a->rows < (1LL << 31), "rms_norm: too many rows");
  const size_t smem = static_cast<size_t>(a->width) * sizeof(float);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
  rmsnorm_kernel<<<static_cast<unsigned>(a->rows), kThreads, smem, s>>>(*a, spec_of(*a));
  return check_launch("cb_rmsnorm");
}

int cb_rmsnorm_row_table(const cb_rmsnorm_args* a, float* d_out, cb_stream_t stream) {
  CB_REQUIRE(a->width > 0 && a->width <= 49152, "rms_norm table: unsupported row width");
  if (a->rows == 0) return CB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const NormSpec n = spec_of(*a);
  if (a->dt_sum != CB_F32) {
    const long long blocks = (a->rows + 127) / 128;
    rmsnorm_table_seq_kernel<<<static_cast<unsigned>(blocks), 128, 0, s>>>(*a, n, d_out);
  } else {
    const size_t smem = static_cast<size_t>(a->width) * sizeof(float);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(rmsnorm_table_par_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    rmsnorm_table_par_kernel<<<static_cast<unsigned>(a->rows), kThreads, smem, s>>>(*a, n, d_out);
  }
  return check_launch("cb_rmsnorm_row_table");
}

int cb_rope(const cb_rope_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->head_size > 0 && a->head_size % 2 == 0, "rope: head size must be even");
  CB_REQUIRE(a->n_offsets >= 1, "rope: empty cos/sin table");
  const long long total = a->batch * a->heads * a->tokens * (a->head_size / 2);
  if (total == 0) return CB_OK;
  long long blocks = (total + kThreads - 1) / kThreads;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  rope_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_launch("cb_rope");
}

}  // extern "C"

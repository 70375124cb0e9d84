// Training kernels: the reference's fused lowerings for compiled training
// steps, and the grouped SGD update behind Compiler.update_native_parameters.
//
// The reference marks these subgraphs with lowering hints
// (chomikgrad/tensor.py:316-450): softmax and log_softmax over an axis, their
// backward contributions, layer_norm and its three backward contributions
// (input, weight, bias).  Each kernel computes what the hinted portable
// subgraph computes, in float32, with the same operations per element:
//   softmax      y = exp(x - max) / sum(exp(x - max))
//   log_softmax  y = (x - max) - log(sum(exp(x - max)))
//   softmax'     dx = y * (g - sum(g * y))
//   log_softmax' dx = g - exp(y) * sum(g)
//   layer_norm   c = x - mean(x), s = sqrt(mean(c * c) + eps), y = c / s * w + b
//   layer_norm'  n = c / s, gw = g * w,
//                dx = (gw - mean(gw) - n * mean(gw * n)) / s,
//                dw = sum over rows of g * n, db = sum over rows of g
// over the last axis of a contiguous (rows, width) float32 matrix.  Sums
// over a row run in a fixed tree order (NumPy's is pairwise; the results
// agree to float32 rounding).  One warp per row: the rows are short (the
// models' hidden sizes and vocabularies) and independent; the weight and
// bias gradients are column sums over the rows, one thread per column
// walking the rows in order (deterministic, coalesced).
//
// SGD (chomikgrad/optim.py:28-64 and the CUDA backend's grouped update):
// out = p - lr * g, the product rounded to float32 first as NumPy computes
// `storage - lr * gradient` on float32 storage.
#include "common.cuh"

namespace cb {
namespace {

constexpr int kRowWarps = 8;  // rows per block (one warp each)

__device__ __forceinline__ float row_max(const float* x, long long width, int lane) {
  float m = -INFINITY;
  for (long long j = lane; j < width; j += 32) m = fmaxf(m, x[j]);
  return warp_max(m);
}

__global__ void __launch_bounds__(kRowWarps * 32) softmax_rows_kernel(const float* x, long long rows,
                                                                      long long width, int log_form, float* out) {
  const long long row = static_cast<long long>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * width;
  float* yr = out + row * width;
  const float m = row_max(xr, width, lane);
  float sum = 0.0f;
  for (long long j = lane; j < width; j += 32) sum += expf(__fsub_rn(xr[j], m));
  sum = warp_sum(sum);
  if (log_form) {
    const float lse = logf(sum);
    for (long long j = lane; j < width; j += 32) yr[j] = __fsub_rn(__fsub_rn(xr[j], m), lse);
  } else {
    for (long long j = lane; j < width; j += 32) yr[j] = __fdiv_rn(expf(__fsub_rn(xr[j], m)), sum);
  }
}

__global__ void __launch_bounds__(kRowWarps * 32) softmax_backward_rows_kernel(const float* g, const float* y,
                                                                               long long rows, long long width,
                                                                               int log_form, float* out) {
  const long long row = static_cast<long long>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* gr = g + row * width;
  const float* yr = y + row * width;
  float* dr = out + row * width;
  float proj = 0.0f;
  if (log_form) {
    for (long long j = lane; j < width; j += 32) proj += gr[j];
  } else {
    for (long long j = lane; j < width; j += 32) proj += __fmul_rn(gr[j], yr[j]);
  }
  proj = warp_sum(proj);
  if (log_form) {
    for (long long j = lane; j < width; j += 32) dr[j] = __fsub_rn(gr[j], __fmul_rn(expf(yr[j]), proj));
  } else {
    for (long long j = lane; j < width; j += 32) dr[j] = __fmul_rn(yr[j], __fsub_rn(gr[j], proj));
  }
}

// Per row: mean and standard deviation (the forward's), into stats[row] = (mean, s).
__device__ __forceinline__ float2 row_moments(const float* xr, long long width, float eps, int lane) {
  float sum = 0.0f;
  for (long long j = lane; j < width; j += 32) sum += xr[j];
  const float mean = __fdiv_rn(warp_sum(sum), static_cast<float>(width));
  float sq = 0.0f;
  for (long long j = lane; j < width; j += 32) {
    const float c = __fsub_rn(xr[j], mean);
    sq = __fadd_rn(sq, __fmul_rn(c, c));
  }
  const float var = __fdiv_rn(warp_sum(sq), static_cast<float>(width));
  return make_float2(mean, __fsqrt_rn(__fadd_rn(var, eps)));
}

__global__ void __launch_bounds__(kRowWarps * 32) layer_norm_rows_kernel(const float* x, const float* w,
                                                                         const float* b, long long rows,
                                                                         long long width, float eps, float* out) {
  const long long row = static_cast<long long>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * width;
  float* yr = out + row * width;
  const float2 ms = row_moments(xr, width, eps, lane);
  for (long long j = lane; j < width; j += 32) {
    const float n = __fdiv_rn(__fsub_rn(xr[j], ms.x), ms.y);
    yr[j] = __fadd_rn(__fmul_rn(n, w[j]), b[j]);
  }
}

__global__ void __launch_bounds__(kRowWarps * 32) layer_norm_backward_rows_kernel(
    const float* g, const float* x, const float* w, long long rows, long long width, float eps, float* dx,
    float2* stats) {
  const long long row = static_cast<long long>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * width;
  const float* gr = g + row * width;
  const float2 ms = row_moments(xr, width, eps, lane);
  if (lane == 0 && stats != nullptr) stats[row] = ms;
  if (dx == nullptr) return;
  float wsum = 0.0f, corr = 0.0f;
  for (long long j = lane; j < width; j += 32) {
    const float n = __fdiv_rn(__fsub_rn(xr[j], ms.x), ms.y);
    const float gw = __fmul_rn(gr[j], w[j]);
    wsum += gw;
    corr = __fadd_rn(corr, __fmul_rn(gw, n));
  }
  const float wmean = __fdiv_rn(warp_sum(wsum), static_cast<float>(width));
  const float cmean = __fdiv_rn(warp_sum(corr), static_cast<float>(width));
  float* dr = dx + row * width;
  for (long long j = lane; j < width; j += 32) {
    const float n = __fdiv_rn(__fsub_rn(xr[j], ms.x), ms.y);
    const float gw = __fmul_rn(gr[j], w[j]);
    dr[j] = __fdiv_rn(__fsub_rn(__fsub_rn(gw, wmean), __fmul_rn(n, cmean)), ms.y);
  }
}

// dw[j] = sum_r g[r, j] * n[r, j], db[j] = sum_r g[r, j], rows in order.
__global__ void layer_norm_param_grads_kernel(const float* g, const float* x, const float2* stats, long long rows,
                                              long long width, float* dw, float* db) {
  const long long j = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j >= width) return;
  float sw = 0.0f, sb = 0.0f;
  for (long long r = 0; r < rows; ++r) {
    const float gv = g[r * width + j];
    if (dw != nullptr) {
      const float2 ms = stats[r];
      sw = __fadd_rn(sw, __fmul_rn(gv, __fdiv_rn(__fsub_rn(x[r * width + j], ms.x), ms.y)));
    }
    sb = __fadd_rn(sb, gv);
  }
  if (dw != nullptr) dw[j] = sw;
  if (db != nullptr) db[j] = sb;
}

__global__ void sgd_group_kernel(const cb_sgd_group g) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long first = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int t = 0; t < g.n; ++t) {
    const float* p = g.param[t];
    const float* d = g.grad[t];
    float* o = g.out[t];
    const long long n = g.count[t];
    const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(d) |
                       reinterpret_cast<uintptr_t>(o)) & 15) == 0;
    long long tail = 0;
    if (vec) {
      const long long n4 = n / 4;
      for (long long i = first; i < n4; i += stride) {
        const float4 pv = reinterpret_cast<const float4*>(p)[i];
        const float4 dv = reinterpret_cast<const float4*>(d)[i];
        float4 r;
        r.x = __fsub_rn(pv.x, __fmul_rn(g.lr, dv.x));
        r.y = __fsub_rn(pv.y, __fmul_rn(g.lr, dv.y));
        r.z = __fsub_rn(pv.z, __fmul_rn(g.lr, dv.z));
        r.w = __fsub_rn(pv.w, __fmul_rn(g.lr, dv.w));
        reinterpret_cast<float4*>(o)[i] = r;
      }
      tail = n4 * 4;
    }
    for (long long i = tail + first; i < n; i += stride) o[i] = __fsub_rn(p[i], __fmul_rn(g.lr, d[i]));
  }
}

unsigned row_blocks(long long rows) { return static_cast<unsigned>((rows + kRowWarps - 1) / kRowWarps); }

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_softmax_rows(const float* x, long long rows, long long width, int log_form, float* out, cb_stream_t stream) {
  CB_REQUIRE(rows >= 0 && width >= 0, "softmax: negative size");
  if (rows == 0 || width == 0) return CB_OK;
  CB_REQUIRE(x != nullptr && out != nullptr, "softmax: null pointer");
  CB_REQUIRE(rows / kRowWarps < (1LL << 31), "softmax: too many rows");
  softmax_rows_kernel<<<row_blocks(rows), kRowWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(x, rows, width,
                                                                                                  log_form, out);
  return check_launch("cb_softmax_rows");
}

int cb_softmax_backward_rows(const float* grad, const float* y, long long rows, long long width, int log_form,
                             float* out, cb_stream_t stream) {
  CB_REQUIRE(rows >= 0 && width >= 0, "softmax backward: negative size");
  if (rows == 0 || width == 0) return CB_OK;
  CB_REQUIRE(grad != nullptr && y != nullptr && out != nullptr, "softmax backward: null pointer");
  CB_REQUIRE(rows / kRowWarps < (1LL << 31), "softmax backward: too many rows");
  softmax_backward_rows_kernel<<<row_blocks(rows), kRowWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      grad, y, rows, width, log_form, out);
  return check_launch("cb_softmax_backward_rows");
}

int cb_layer_norm_rows(const float* x, const float* w, const float* b, long long rows, long long width, float eps,
                       float* out, cb_stream_t stream) {
  CB_REQUIRE(rows >= 0 && width >= 0, "layer_norm: negative size");
  if (rows == 0 || width == 0) return CB_OK;
  CB_REQUIRE(x != nullptr && w != nullptr && b != nullptr && out != nullptr, "layer_norm: null pointer");
  CB_REQUIRE(eps > 0.0f, "layer_norm: epsilon must be positive");
  CB_REQUIRE(rows / kRowWarps < (1LL << 31), "layer_norm: too many rows");
  layer_norm_rows_kernel<<<row_blocks(rows), kRowWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      x, w, b, rows, width, eps, out);
  return check_launch("cb_layer_norm_rows");
}

int cb_layer_norm_backward_rows(const float* grad, const float* x, const float* w, long long rows, long long width,
                                float eps, float* dx, float* dw, float* db, float* row_stats, cb_stream_t stream) {
  CB_REQUIRE(rows >= 0 && width >= 0, "layer_norm backward: negative size");
  CB_REQUIRE(dx != nullptr || dw != nullptr || db != nullptr, "layer_norm backward: no output requested");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (width == 0) return CB_OK;
  if (rows == 0) {  // empty sums: zero parameter gradients
    if (dw != nullptr && cudaMemsetAsync(dw, 0, static_cast<size_t>(width) * 4, s) != cudaSuccess)
      return check_launch("cb_layer_norm_backward_rows");
    if (db != nullptr && cudaMemsetAsync(db, 0, static_cast<size_t>(width) * 4, s) != cudaSuccess)
      return check_launch("cb_layer_norm_backward_rows");
    return CB_OK;
  }
  CB_REQUIRE(grad != nullptr && x != nullptr && w != nullptr, "layer_norm backward: null input");
  CB_REQUIRE(dw == nullptr || row_stats != nullptr, "layer_norm backward: the weight gradient needs row_stats");
  CB_REQUIRE(eps > 0.0f, "layer_norm backward: epsilon must be positive");
  CB_REQUIRE(rows / kRowWarps < (1LL << 31), "layer_norm backward: too many rows");
  layer_norm_backward_rows_kernel<<<row_blocks(rows), kRowWarps * 32, 0, s>>>(
      grad, x, w, rows, width, eps, dx, reinterpret_cast<float2*>(row_stats));
  int r = check_launch("cb_layer_norm_backward_rows");
  if (r != CB_OK || (dw == nullptr && db == nullptr)) return r;
  layer_norm_param_grads_kernel<<<static_cast<unsigned>((width + 255) / 256), 256, 0, s>>>(
      grad, x, reinterpret_cast<const float2*>(row_stats), rows, width, dw, db);
  return check_launch("cb_layer_norm_backward_rows (parameter gradients)");
}

int cb_sgd_update(const cb_sgd_group* group, cb_stream_t stream) {
  CB_REQUIRE(group != nullptr, "sgd: no group");
  CB_REQUIRE(group->n >= 0 && group->n <= CB_SGD_GROUP, "sgd: %d tensors (at most %d per launch)", group->n,
             CB_SGD_GROUP);
  long long total = 0;
  for (int t = 0; t < group->n; ++t) {
    CB_REQUIRE(group->count[t] >= 0, "sgd: negative size");
    if (group->count[t] > 0)
      CB_REQUIRE(group->param[t] != nullptr && group->grad[t] != nullptr && group->out[t] != nullptr,
                 "sgd: null pointer");
    total += group->count[t];
  }
  if (total == 0) return CB_OK;
  const int sms = sm_count();
  long long blocks = (total / 4 + 255) / 256;
  if (blocks > 4LL * sms) blocks = 4LL * sms;  // grid-stride beyond four waves
  if (blocks < 1) blocks = 1;
  sgd_group_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(*group);
  return check_launch("cb_sgd_update");
}

}  // extern "C"

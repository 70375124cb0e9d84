// Generic six-op kernels: fused elementwise, reductions, strided copies,
// gather and row argmax.  These carry any graph the plugin cannot pattern-
// match; the Llama hot path uses the fused kernels in gemv.cu/attention.cu.
#include "common.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;

inline int grid_for(long long n, int per_block = kThreads) {
  long long blocks = (n + per_block - 1) / per_block;
  long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

__device__ __forceinline__ float apply_op(int op, float a, float b) {
  switch (op) {
    case CB_OP_ADD: return __fadd_rn(a, b);
    case CB_OP_SUB: return __fsub_rn(a, b);
    case CB_OP_MUL: return __fmul_rn(a, b);
    case CB_OP_DIV: return __fdiv_rn(a, b);
    case CB_OP_EQUAL: return a == b ? 1.0f : 0.0f;
    case CB_OP_NEG: return -a;
    case CB_OP_EXP: return expf(a);
    case CB_OP_LOG: return logf(a);
    case CB_OP_SQRT: return __fsqrt_rn(a);
    case CB_OP_RELU: return (a >= 0.0f || a != a) ? a : 0.0f;  // np.maximum(a, 0)
    case CB_OP_STEP: return a > 0.0f ? 1.0f : 0.0f;
    default: return 0.0f;
  }
}

__global__ void elementwise_kernel(const cb_elementwise_args a, long long total) {
  float reg[CB_EW_MAX_INPUTS + CB_EW_MAX_INSTR];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long offs[CB_EW_MAX_INPUTS];
    for (int j = 0; j < a.n_inputs; ++j) offs[j] = a.in_offset[j];
    long long rest = i;
    for (int d = a.ndim - 1; d >= 0; --d) {
      const long long c = rest % a.shape[d];
      rest /= a.shape[d];
      for (int j = 0; j < a.n_inputs; ++j) offs[j] += c * a.in_strides[j][d];
    }
    for (int j = 0; j < a.n_inputs; ++j) reg[j] = load_as_f32(a.inputs[j], offs[j], a.in_dtype[j]);
    float result = reg[0];
    for (int t = 0; t < a.n_instr; ++t) {
      result = round_to(apply_op(a.op[t], reg[a.lhs[t]], a.rhs[t] >= 0 ? reg[a.rhs[t]] : 0.0f),
                        a.round[t]);
      reg[a.n_inputs + t] = result;
    }
    store_from_f32(a.out, i, a.out_dtype, result);
  }
}

// Every input is either laid out like the output (offset + i) or a scalar
// broadcast (bit j of `scalar` set): no per-element index arithmetic.  Each
// thread handles kFlatIlp elements a grid stride apart, loading all of them
// before computing, so their loads are in flight together.
constexpr int kFlatIlp = 4;

__global__ void elementwise_flat_kernel(const cb_elementwise_args a, long long total, unsigned scalar) {
  float reg[CB_EW_MAX_INPUTS + CB_EW_MAX_INSTR];
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long base = blockIdx.x * (long long)blockDim.x + threadIdx.x; base < total; base += stride * kFlatIlp) {
    float in[kFlatIlp][CB_EW_MAX_INPUTS];
#pragma unroll
    for (int e = 0; e < kFlatIlp; ++e) {
      const long long i = base + e * stride;
#pragma unroll
      for (int j = 0; j < CB_EW_MAX_INPUTS; ++j)
        if (j < a.n_inputs && i < total)
          in[e][j] = load_as_f32(a.inputs[j], a.in_offset[j] + (((scalar >> j) & 1u) ? 0 : i), a.in_dtype[j]);
    }
#pragma unroll
    for (int e = 0; e < kFlatIlp; ++e) {
      const long long i = base + e * stride;
      if (i >= total) break;
#pragma unroll
      for (int j = 0; j < CB_EW_MAX_INPUTS; ++j)
        if (j < a.n_inputs) reg[j] = in[e][j];
      float result = reg[0];
      for (int t = 0; t < a.n_instr; ++t) {
        result = round_to(apply_op(a.op[t], reg[a.lhs[t]], a.rhs[t] >= 0 ? reg[a.rhs[t]] : 0.0f), a.round[t]);
        reg[a.n_inputs + t] = result;
      }
      store_from_f32(a.out, i, a.out_dtype, result);
    }
  }
}

__device__ __forceinline__ float nan_max(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return fmaxf(a, b);
}

__device__ __forceinline__ long long red_offset(const cb_reduce_args& a, long long r) {
  long long off = 0;
  for (int d = a.n_red - 1; d >= 0; --d) {
    const long long c = r % a.red_shape[d];
    r /= a.red_shape[d];
    off += c * a.red_strides[d];
  }
  return off;
}

__device__ __forceinline__ long long keep_offset(const cb_reduce_args& a, long long o) {
  long long off = a.in_offset;
  for (int d = a.n_keep - 1; d >= 0; --d) {
    const long long c = o % a.keep_shape[d];
    o /= a.keep_shape[d];
    off += c * a.keep_strides[d];
  }
  return off;
}

// One thread per output, accumulating in index order (NumPy's reduce loop for
// non-native float types rounds the accumulator after every add).
__global__ void reduce_sequential_kernel(const cb_reduce_args a, long long n_out, long long n_red) {
  for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < n_out;
       o += (long long)gridDim.x * blockDim.x) {
    const long long base = keep_offset(a, o);
    float acc = load_as_f32(a.in, base + red_offset(a, 0), a.in_dtype);
    for (long long r = 1; r < n_red; ++r) {
      const float v = load_as_f32(a.in, base + red_offset(a, r), a.in_dtype);
      acc = a.kind == CB_REDUCE_SUM ? round_to(__fadd_rn(acc, v), a.acc_dtype) : nan_max(acc, v);
    }
    store_from_f32(a.out, o, a.out_dtype, acc);
  }
}

// One warp per output, tree order (float32 sums; any max).
__global__ void reduce_warp_kernel(const cb_reduce_args a, long long n_out, long long n_red) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long o = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); o < n_out;
       o += warps) {
    const long long base = keep_offset(a, o);
    float acc = a.kind == CB_REDUCE_SUM ? 0.0f : -INFINITY;
    for (long long r = lane; r < n_red; r += 32) {
      const float v = load_as_f32(a.in, base + red_offset(a, r), a.in_dtype);
      acc = a.kind == CB_REDUCE_SUM ? acc + v : nan_max(acc, v);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, acc, s);
      acc = a.kind == CB_REDUCE_SUM ? acc + other : nan_max(acc, other);
    }
    if (lane == 0) store_from_f32(a.out, o, a.out_dtype, acc);
  }
}

struct CopyShape {
  long long shape[CB_MAX_DIMS];
  long long strides[CB_MAX_DIMS];
};

template <typename T>
__global__ void copy_strided_kernel(const T* in, T* out, int ndim, CopyShape s, long long total) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long rest = i, off = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      const long long c = rest % s.shape[d];
      rest /= s.shape[d];
      off += c * s.strides[d];
    }
    out[i] = in[off];
  }
}

__global__ void place_columns_kernel(const void* in, int in_dtype, int ndim, CopyShape s, const int* cols,
                                     long long n, long long total, void* out, int out_dtype) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / n, j = i - r * n;
    const int c = cols[j];
    float v = 0.0f;
    if (c >= 0) {
      long long rest = r, off = c * s.strides[ndim - 1];
      for (int d = ndim - 2; d >= 0; --d) {
        off += (rest % s.shape[d]) * s.strides[d];
        rest /= s.shape[d];
      }
      v = load_as_f32(in, off, in_dtype);
    }
    store_from_f32(out, i, out_dtype, v);
  }
}

// Grid (units / 256, batch * heads): one thread per (row, 4 dims) of a
// head's cache; rows whose write mask is 0 are left alone (the blend is the
// cache itself there), so only the written row costs more than a mask read.
__global__ void kv_write_kernel(float* cache, long long heads, long long ctx, long long hd, const void* row,
                                int row_dtype, long long rs_b, long long rs_h, long long rs_d, const void* wm,
                                int wm_dtype, int one_minus_dtype) {
  const long long bh = blockIdx.y;
  const long long b = bh / heads, h = bh % heads;
  const long long groups = (hd + 3) / 4;
  const long long u = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= ctx * groups) return;
  const long long r = u / groups, d0 = (u % groups) * 4;
  const float w = load_as_f32(wm, r, wm_dtype);
  if (w == 0.0f) return;
  const float keep = round_to(__fsub_rn(1.0f, w), one_minus_dtype);
  float* base = cache + (bh * ctx + r) * hd;
  const long long rbase = b * rs_b + h * rs_h;
  for (long long d = d0; d < d0 + 4 && d < hd; ++d) {
    const float x = load_as_f32(row, rbase + d * rs_d, row_dtype);
    base[d] = __fadd_rn(__fmul_rn(base[d], keep), __fmul_rn(x, w));
  }
}

template <typename T>
__global__ void gather_kernel(const T* table, long long rows, long long row_units, const void* idx,
                              int idx_dtype, long long n, T* out, int* error_flag) {
  const long long total = n * row_units;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long which = i / row_units;
    const long long unit = i - which * row_units;
    long long row = load_index(idx, which, idx_dtype);
    if (row < 0) row += rows;
    if (row < 0 || row >= rows) {
      if (error_flag != nullptr) atomicExch(error_flag, CB_FLAG_INDEX);
      out[i] = T{};
      continue;
    }
    out[i] = table[row * row_units + unit];
  }
}

__global__ void argmax_rows_kernel(const void* x, int dtype, long long width, long long* out) {
  __shared__ float best_v[kThreads];
  __shared__ long long best_i[kThreads];
  const long long row = blockIdx.x;
  float bv = -INFINITY;
  long long bi = width;  // sentinel: loses to any real index
  for (long long j = threadIdx.x; j < width; j += blockDim.x) {
    const float v = load_as_f32(x, row * width + j, dtype);
    if (bi == width || argmax_better(v, j, bv, bi)) {
      bv = v;
      bi = j;
    }
  }
  best_v[threadIdx.x] = bv;
  best_i[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      const float ov = best_v[threadIdx.x + s];
      const long long oi = best_i[threadIdx.x + s];
      if (oi != width && (best_i[threadIdx.x] == width ||
                          argmax_better(ov, oi, best_v[threadIdx.x], best_i[threadIdx.x]))) {
        best_v[threadIdx.x] = ov;
        best_i[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[row] = best_i[0] == width ? 0 : best_i[0];
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_elementwise(const cb_elementwise_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->ndim >= 0 && a->ndim <= CB_MAX_DIMS, "elementwise: bad ndim %d", a->ndim);
  CB_REQUIRE(a->n_inputs >= 1 && a->n_inputs <= CB_EW_MAX_INPUTS, "elementwise: bad input count");
  CB_REQUIRE(a->n_instr >= 0 && a->n_instr <= CB_EW_MAX_INSTR, "elementwise: bad instruction count");
  for (int t = 0; t < a->n_instr; ++t) {
    const int limit = a->n_inputs + t;
    CB_REQUIRE(a->lhs[t] >= 0 && a->lhs[t] < limit && a->rhs[t] < limit,
               "elementwise: instruction %d reads an undefined register", t);
  }
  long long total = 1;
  for (int d = 0; d < a->ndim; ++d) total *= a->shape[d];
  if (total == 0) return CB_OK;
  // flat path: every input contiguous like the output, or a scalar
  unsigned scalar = 0;
  bool flat = true;
  for (int j = 0; j < a->n_inputs && flat; ++j) {
    bool zero = true, contig = true;
    long long expect = 1;
    for (int d = a->ndim - 1; d >= 0; --d) {
      if (a->shape[d] == 1) continue;
      zero = zero && a->in_strides[j][d] == 0;
      contig = contig && a->in_strides[j][d] == expect;
      expect *= a->shape[d];
    }
    if (zero) scalar |= 1u << j;
    flat = zero || contig;
  }
  if (flat) {
    elementwise_flat_kernel<<<grid_for((total + kFlatIlp - 1) / kFlatIlp), kThreads, 0,
                              static_cast<cudaStream_t>(stream)>>>(*a, total, scalar);
    return check_launch("cb_elementwise");
  }
  elementwise_kernel<<<grid_for(total), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(*a, total);
  return check_launch("cb_elementwise");
}

int cb_reduce(const cb_reduce_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->n_keep >= 0 && a->n_keep <= CB_MAX_DIMS && a->n_red >= 0 && a->n_red <= CB_MAX_DIMS,
             "reduce: bad dims");
  long long n_out = 1, n_red = 1;
  for (int d = 0; d < a->n_keep; ++d) n_out *= a->keep_shape[d];
  for (int d = 0; d < a->n_red; ++d) n_red *= a->red_shape[d];
  if (n_out == 0) return CB_OK;
  CB_REQUIRE(n_red > 0 || a->kind == CB_REDUCE_SUM,
             "zero-size array to reduction operation maximum which has no identity");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_red == 0) {
    cudaMemsetAsync(a->out, 0, n_out * (a->out_dtype == CB_F32 ? 4 : 2), s);
    return check_launch("cb_reduce(empty)");
  }
  if (a->sequential) {
    reduce_sequential_kernel<<<grid_for(n_out), kThreads, 0, s>>>(*a, n_out, n_red);
  } else {
    reduce_warp_kernel<<<grid_for(n_out * 32), kThreads, 0, s>>>(*a, n_out, n_red);
  }
  return check_launch("cb_reduce");
}

int cb_copy_strided(const void* in, long long in_offset, void* out, int elem_bytes, int ndim,
                    const long long* shape, const long long* in_strides, cb_stream_t stream) {
  CB_REQUIRE(ndim >= 0 && ndim <= CB_MAX_DIMS, "copy: bad ndim %d", ndim);
  CopyShape s{};
  long long total = 1;
  for (int d = 0; d < ndim; ++d) {
    s.shape[d] = shape[d];
    s.strides[d] = in_strides[d];
    total *= shape[d];
  }
  if (total == 0) return CB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int g = grid_for(total);
  switch (elem_bytes) {
    case 1: copy_strided_kernel<<<g, kThreads, 0, st>>>(static_cast<const uint8_t*>(in) + in_offset,
                                                         static_cast<uint8_t*>(out), ndim, s, total); break;
    case 2: copy_strided_kernel<<<g, kThreads, 0, st>>>(static_cast<const uint16_t*>(in) + in_offset,
                                                         static_cast<uint16_t*>(out), ndim, s, total); break;
    case 4: copy_strided_kernel<<<g, kThreads, 0, st>>>(static_cast<const uint32_t*>(in) + in_offset,
                                                         static_cast<uint32_t*>(out), ndim, s, total); break;
    case 8: copy_strided_kernel<<<g, kThreads, 0, st>>>(static_cast<const uint64_t*>(in) + in_offset,
                                                         static_cast<uint64_t*>(out), ndim, s, total); break;
    default: CB_REQUIRE(false, "copy: unsupported element size %d", elem_bytes);
  }
  return check_launch("cb_copy_strided");
}

int cb_place_columns(const void* in, int in_dtype, int ndim, const long long* shape, const long long* in_strides,
                     const int* cols, long long n, void* out, int out_dtype, cb_stream_t stream) {
  CB_REQUIRE(ndim >= 1 && ndim <= CB_MAX_DIMS, "place: bad ndim %d", ndim);
  CB_REQUIRE(n >= 0, "place: negative width");
  CopyShape s{};
  long long rows = 1;
  for (int d = 0; d < ndim; ++d) {
    s.shape[d] = shape[d];
    s.strides[d] = in_strides[d];
    if (d < ndim - 1) rows *= shape[d];
  }
  const long long total = rows * n;
  if (total == 0) return CB_OK;
  place_columns_kernel<<<grid_for(total), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      in, in_dtype, ndim, s, cols, n, total, out, out_dtype);
  return check_launch("cb_place_columns");
}

int cb_kv_write(float* cache, long long batch, long long heads, long long ctx, long long head_size,
                const void* row, int row_dtype, const long long* row_strides, const void* write_mask,
                int write_mask_dtype, int one_minus_dtype, cb_stream_t stream) {
  CB_REQUIRE(cache != nullptr && row != nullptr && write_mask != nullptr, "kv_write: null pointer");
  CB_REQUIRE(batch >= 0 && heads >= 0 && ctx >= 0 && head_size >= 0, "kv_write: negative size");
  if (batch * heads == 0 || ctx == 0) return CB_OK;
  CB_REQUIRE(batch * heads < 65536 && ctx * ((head_size + 3) / 4) < (1LL << 40), "kv_write: too many heads");
  const long long units = ctx * ((head_size + 3) / 4);
  const dim3 grid(static_cast<unsigned>((units + 255) / 256), static_cast<unsigned>(batch * heads));
  kv_write_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      cache, heads, ctx, head_size, row, row_dtype, row_strides[0], row_strides[1], row_strides[3], write_mask,
      write_mask_dtype, one_minus_dtype);
  return check_launch("cb_kv_write");
}

int cb_gather(const void* table, long long rows, long long row_bytes, const void* idx, int idx_dtype,
              long long n, void* out, int* error_flag, cb_stream_t stream) {
  CB_REQUIRE(idx_dtype == CB_I32 || idx_dtype == CB_I64, "gather: indices must be int32/int64");
  CB_REQUIRE(rows >= 0 && row_bytes >= 0 && n >= 0, "gather: negative size");
  if (n == 0 || row_bytes == 0) return CB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uintptr_t align = reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out) |
                          static_cast<uintptr_t>(row_bytes);
  if ((align & 15) == 0) {
    const long long units = row_bytes / 16;
    gather_kernel<<<grid_for(n * units), kThreads, 0, s>>>(static_cast<const uint4*>(table), rows, units,
                                                           idx, idx_dtype, n, static_cast<uint4*>(out),
                                                           error_flag);
  } else if ((align & 3) == 0) {
    const long long units = row_bytes / 4;
    gather_kernel<<<grid_for(n * units), kThreads, 0, s>>>(static_cast<const uint32_t*>(table), rows,
                                                           units, idx, idx_dtype, n,
                                                           static_cast<uint32_t*>(out), error_flag);
  } else {
    gather_kernel<<<grid_for(n * row_bytes), kThreads, 0, s>>>(static_cast<const uint8_t*>(table), rows,
                                                               row_bytes, idx, idx_dtype, n,
                                                               static_cast<uint8_t*>(out), error_flag);
  }
  return check_launch("cb_gather");
}

int cb_argmax_rows(const void* x, int dtype, long long rows, long long width, long long* out_index,
                   cb_stream_t stream) {
  CB_REQUIRE(width > 0, "attempt to get argmax of an empty sequence");
  if (rows == 0) return CB_OK;
  CB_REQUIRE(rows < (1LL << 31), "argmax: too many rows");
  argmax_rows_kernel<<<static_cast<unsigned>(rows), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, dtype, width, out_index);
  return check_launch("cb_argmax_rows");
}

}  // extern "C"

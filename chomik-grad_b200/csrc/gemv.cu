// Streaming GEMV for single-token decode: y = x W^T, W row-major (out, in).
//
// Decode is bound by reading every weight byte once from HBM.  Design:
//  * one CTA per SM; each CTA owns a contiguous range of "units" (weight
//    rows); the whole CTA cooperates on R rows at a time, every thread
//    issuing R x CPT independent 16-byte loads (L1 no-allocate) so a CTA
//    keeps 32 KiB of weight loads in flight;
//  * the input row x (optionally gathered by a device index and rms-normed
//    with the reference's roundings) is staged once per CTA in shared memory;
//  * epilogues fuse the consumers the reference graph applies next:
//    residual add, SwiGLU silu(gate)*up (rows of gate/up interleaved as unit
//    pairs), or logits + greedy argmax (last-CTA merge, deterministic);
//  * before waiting on its producer (programmatic dependent launch) every CTA
//    issues an L2 prefetch of its share of the NEXT kernel's weights, so HBM
//    keeps streaming across kernel boundaries.
#include "norm.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <typename WT>
struct Vec;
template <>
struct Vec<uint16_t> {  // bfloat16 weights: 8 per 16-byte chunk
  static constexpr int kElems = 8;
  __device__ static float dot(const uint4& w, const float* x) {
    float f[8];
    unpack_bf16x8(w, f);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = fmaf(f[i], x[i], s);
    return s;
  }
};
template <>
struct Vec<float> {  // float32 weights: 4 per chunk
  static constexpr int kElems = 4;
  __device__ static float dot(const uint4& w, const float* x) {
    float s = __uint_as_float(w.x) * x[0];
    s = fmaf(__uint_as_float(w.y), x[1], s);
    s = fmaf(__uint_as_float(w.z), x[2], s);
    s = fmaf(__uint_as_float(w.w), x[3], s);
    return s;
  }
};

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

template <typename WT, int CPT, int R>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const cb_gemv_args a, long long units,
                                                        long long units_per_cta) {
  extern __shared__ float xs[];  // k floats
  __shared__ float red[kWarps][R];
  __shared__ float tot[R];
  __shared__ float norm_red[kWarps];
  __shared__ float best_v;
  __shared__ long long best_i;
  __shared__ int is_last;
  constexpr int VE = Vec<WT>::kElems;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long K = a.k;
  const long long chunks = K / VE;
  const long long row_bytes = K * static_cast<long long>(sizeof(WT));
  const long long u0 = static_cast<long long>(blockIdx.x) * units_per_cta;
  const long long u1 = u0 + units_per_cta < units ? u0 + units_per_cta : units;

  prefetch_share(a.prefetch_ptr, a.prefetch_bytes, blockIdx.x, gridDim.x);
  pdl_wait();
  pdl_launch_dependents();

  // ---- stage (and normalise) the input row ----
  long long xrow = a.x_index != nullptr ? load_index(a.x_index, 0, a.x_index_dtype) : 0;
  if (a.x_index != nullptr && (xrow < 0 || xrow >= a.index_rows)) {
    if (tid == 0 && blockIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, 1);
    xrow = 0;
  }
  for (long long i = tid; i < K; i += kThreads) xs[i] = load_as_f32(a.x, xrow * K + i, a.x_dtype);
  __syncthreads();
  if (a.norm != CB_NORM_NONE) {
    const NormSpec n{a.divisor, a.eps, a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y};
    const float d = a.norm == CB_NORM_RMS_TABLE ? a.norm_table[xrow]
                                                : norm_finish_d(n, norm_block_sum(n, xs, static_cast<int>(K), norm_red));
    __syncthreads();
    for (long long i = tid; i < K; i += kThreads)
      xs[i] = norm_apply(n, xs[i], d, load_as_f32(a.norm_w, i, a.norm_w_dtype), a.dt_norm_out);
    __syncthreads();
  }
  if (a.epilogue == CB_EPI_ARGMAX && tid == 0) {
    best_v = 0.0f;
    best_i = -1;
  }

  // ---- stream the weight rows ----
  for (long long ub = u0; ub < u1; ub += R) {
    uint4 wv[R][CPT];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const bool live = ub + r < u1;
      const char* row = live ? unit_row(a, ub + r, row_bytes) : nullptr;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const long long ch = tid + static_cast<long long>(c) * kThreads;
        wv[r][c] = (live && ch < chunks) ? ld_stream(row + ch * 16) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float part[R];
#pragma unroll
    for (int r = 0; r < R; ++r) part[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const long long ch = tid + static_cast<long long>(c) * kThreads;
      if (ch < chunks) {
        float xv[VE];
#pragma unroll
        for (int e = 0; e < VE; e += 4) {
          const float4 q = *reinterpret_cast<const float4*>(xs + ch * VE + e);
          xv[e] = q.x;
          xv[e + 1] = q.y;
          xv[e + 2] = q.z;
          xv[e + 3] = q.w;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) part[r] += Vec<WT>::dot(wv[r][c], xv);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float s = warp_sum(part[r]);
      if (lane == 0) red[warp][r] = s;
    }
    __syncthreads();
    if (tid < R) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += red[w][tid];
      tot[tid] = s;
    }
    __syncthreads();
    // ---- epilogue ----
    if (a.epilogue == CB_EPI_ARGMAX) {
      if (tid == 0) {
        for (int r = 0; r < R && ub + r < u1; ++r) {
          const long long u = ub + r;
          a.out[u] = tot[r];
          if (best_i < 0 || argmax_better(tot[r], u, best_v, best_i)) {
            best_v = tot[r];
            best_i = u;
          }
        }
      }
    } else if (tid < R && ub + tid < u1) {
      const long long u = ub + tid;
      const float v = tot[tid];
      if (a.epilogue == CB_EPI_STORE) {
        a.out[u] = v;
      } else if (a.epilogue == CB_EPI_RESIDUAL) {
        long long rrow = 0;
        if (a.residual_index != nullptr) {
          rrow = load_index(a.residual_index, 0, a.residual_index_dtype);
          if (rrow < 0 || rrow >= a.index_rows) {
            if (a.error_flag != nullptr) atomicExch(a.error_flag, 1);
            rrow = 0;
          }
          rrow *= units;
        }
        a.out[u] = __fadd_rn(load_as_f32(a.residual, rrow + u, a.residual_dtype), v);
      } else if ((tid & 1) == 0) {  // CB_EPI_SILU_MUL: even unit = gate, odd = up
        const float up = tot[tid + 1];
        const float silu = __fdiv_rn(v, __fadd_rn(expf(-v), 1.0f));
        a.out[u >> 1] = __fmul_rn(silu, up);
      }
    }
  }

  if (a.epilogue != CB_EPI_ARGMAX) return;
  // ---- argmax: per-CTA best -> scratch; the last CTA merges in CTA order ----
  if (tid == 0) {
    a.scratch_val[blockIdx.x] = best_v;
    a.scratch_idx[blockIdx.x] = best_i;
    __threadfence();
    const unsigned ticket = atomicAdd(a.counter, 1u);
    is_last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last || tid != 0) return;
  __threadfence();
  float bv = 0.0f;
  long long bi = -1;
  for (unsigned c = 0; c < gridDim.x; ++c) {
    const long long ci = __ldcg(a.scratch_idx + c);
    const float cv = __ldcg(a.scratch_val + c);
    if (ci >= 0 && (bi < 0 || argmax_better(cv, ci, bv, bi))) {
      bv = cv;
      bi = ci;
    }
  }
  a.argmax_out[0] = bi;
  *a.counter = 0u;
}

struct Plan {
  long long units, per_cta;
  int grid, cpt, rows;
  size_t smem;
};

int plan_gemv(const cb_gemv_args& a, Plan* p) {
  CB_REQUIRE(a.w_dtype == CB_BF16 || a.w_dtype == CB_F32, "gemv: weights must be bf16 or f32");
  CB_REQUIRE(a.n_w >= 1 && a.n_w <= 3, "gemv: 1..3 weight matrices");
  const int ve = a.w_dtype == CB_BF16 ? 8 : 4;
  CB_REQUIRE(a.k > 0 && a.k % ve == 0, "gemv: k=%lld must be a multiple of %d", a.k, ve);
  const long long chunks = a.k / ve;
  int cpt = 1;
  while (cpt * kThreads < chunks) cpt *= 2;
  CB_REQUIRE(cpt <= 8, "gemv: k=%lld too large", a.k);
  long long units = 0;
  if (a.epilogue == CB_EPI_SILU_MUL) {
    CB_REQUIRE(a.n_w == 2 && a.w_rows[0] == a.w_rows[1], "gemv: SwiGLU needs gate/up of equal rows");
    units = 2 * a.w_rows[0];
  } else {
    for (int i = 0; i < a.n_w; ++i) units += a.w_rows[i];
  }
  CB_REQUIRE(units > 0, "gemv: no rows");
  int rows = 8 / cpt;
  if (a.epilogue == CB_EPI_SILU_MUL && rows < 2) rows = 2;
  int grid = a.grid > 0 ? a.grid : sm_count();
  long long per = (units + grid - 1) / grid;
  per = (per + rows - 1) / rows * rows;
  grid = static_cast<int>((units + per - 1) / per);
  p->units = units;
  p->per_cta = per;
  p->grid = grid;
  p->cpt = cpt;
  p->rows = rows;
  p->smem = static_cast<size_t>(a.k) * sizeof(float);
  CB_REQUIRE(p->smem <= 200 * 1024, "gemv: k too large for shared memory");
  if (a.epilogue == CB_EPI_ARGMAX)
    CB_REQUIRE(a.scratch_val && a.scratch_idx && a.counter && a.argmax_out, "gemv: argmax needs scratch");
  if (a.epilogue == CB_EPI_RESIDUAL) CB_REQUIRE(a.residual != nullptr, "gemv: residual missing");
  if (a.norm != CB_NORM_NONE) CB_REQUIRE(a.norm_w != nullptr, "gemv: norm weight missing");
  if (a.norm == CB_NORM_RMS_TABLE) CB_REQUIRE(a.norm_table && a.x_index, "gemv: norm table needs x_index");
  if (a.x_index != nullptr || a.residual_index != nullptr)
    CB_REQUIRE(a.index_rows > 0, "gemv: indexed rows need index_rows");
  return CB_OK;
}

template <typename WT, int CPT, int R>
cudaError_t launch_gemv(const cb_gemv_args& a, const Plan& p, cudaStream_t s) {
  auto kernel = gemv_kernel<WT, CPT, R>;
  if (p.smem > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p.smem));
  return launch(kernel, dim3(p.grid), dim3(kThreads), p.smem, s, a.pdl != 0, a, p.units, p.per_cta);
}

template <typename WT>
cudaError_t dispatch(const cb_gemv_args& a, const Plan& p, cudaStream_t s) {
  switch (p.cpt) {
    case 1: return launch_gemv<WT, 1, 8>(a, p, s);
    case 2: return launch_gemv<WT, 2, 4>(a, p, s);
    case 4: return launch_gemv<WT, 4, 2>(a, p, s);
    default: return p.rows == 2 ? launch_gemv<WT, 8, 2>(a, p, s) : launch_gemv<WT, 8, 1>(a, p, s);
  }
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_gemv_grid(const cb_gemv_args* a, int* grid) {
  Plan p;
  const int st = plan_gemv(*a, &p);
  if (st != CB_OK) return st;
  *grid = p.grid;
  return CB_OK;
}

int cb_gemv(const cb_gemv_args* a, cb_stream_t stream) {
  Plan p;
  const int st = plan_gemv(*a, &p);
  if (st != CB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = a->w_dtype == CB_BF16 ? dispatch<uint16_t>(*a, p, s) : dispatch<float>(*a, p, s);
  if (e != cudaSuccess) {
    set_error("cb_gemv: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_gemv");
}

}  // extern "C"

// Streaming GEMV for single-token decode: y = x W^T, W row-major (out, in).
//
// Decode is bound by reading every weight byte once from HBM.  Design:
//  * one CTA per SM owns a contiguous range of "units" (weight rows); a
//    producer warp streams them with bulk copies (TMA engine,
//    cp.async.bulk + mbarrier transaction counts) into a ring of ~8 KiB
//    shared-memory stages -- up to ~96 KiB per SM in flight without any
//    register cost;
//  * the producer starts streaming BEFORE the kernel waits on its producer
//    kernel (programmatic dependent launch: weights never depend on it), and
//    the CTA also issues an L2 prefetch of its share of the NEXT kernel's
//    weights, so HBM keeps streaming across kernel boundaries;
//  * eight consumer warps each own whole stages (round robin), so a row's dot
//    product is reduced inside one warp -- no block-wide barrier in the loop
//    and a fixed summation order (deterministic results);
//  * the input row x (optionally gathered by a device index and rms-normed
//    with the reference's roundings) is staged once per CTA in shared memory;
//  * epilogues fuse the consumers the reference graph applies next:
//    residual add, SwiGLU silu(gate)*up (gate/up rows interleaved in a
//    stage), or logits + greedy argmax (last-CTA merge in CTA order).
#include "norm.cuh"
#include "sync.cuh"

namespace cb {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + producer warp
constexpr int kStageTarget = 8 * 1024;                // bytes per ring stage
constexpr int kRingTarget = 96 * 1024;                // bytes in flight per CTA

template <typename WT>
struct Vec;
template <>
struct Vec<uint16_t> {  // bfloat16 weights: 8 per 16-byte chunk
  static constexpr int kElems = 8;
  __device__ static float dot(const uint4& w, const float* xs, float acc) {
    const float4 x0 = *reinterpret_cast<const float4*>(xs);
    const float4 x1 = *reinterpret_cast<const float4*>(xs + 4);
    acc = fmaf(__uint_as_float(w.x << 16), x0.x, acc);
    acc = fmaf(__uint_as_float(w.x & 0xffff0000u), x0.y, acc);
    acc = fmaf(__uint_as_float(w.y << 16), x0.z, acc);
    acc = fmaf(__uint_as_float(w.y & 0xffff0000u), x0.w, acc);
    acc = fmaf(__uint_as_float(w.z << 16), x1.x, acc);
    acc = fmaf(__uint_as_float(w.z & 0xffff0000u), x1.y, acc);
    acc = fmaf(__uint_as_float(w.w << 16), x1.z, acc);
    acc = fmaf(__uint_as_float(w.w & 0xffff0000u), x1.w, acc);
    return acc;
  }
};
template <>
struct Vec<float> {  // float32 weights: 4 per chunk
  static constexpr int kElems = 4;
  __device__ static float dot(const uint4& w, const float* xs, float acc) {
    const float4 x0 = *reinterpret_cast<const float4*>(xs);
    acc = fmaf(__uint_as_float(w.x), x0.x, acc);
    acc = fmaf(__uint_as_float(w.y), x0.y, acc);
    acc = fmaf(__uint_as_float(w.z), x0.z, acc);
    acc = fmaf(__uint_as_float(w.w), x0.w, acc);
    return acc;
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

struct Layout {
  long long units, per_cta;
  int grid, stage_units, slots;
  long long row_bytes, stage_bytes;
  size_t ring_bytes, smem;
};

template <typename WT>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const cb_gemv_args a, const Layout L) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  float* xs = reinterpret_cast<float*>(smem + L.ring_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.ring_bytes + ((a.k * 4 + 15) & ~15LL));
  uint64_t* empty = full + L.slots;
  __shared__ float norm_red[kConsumerWarps + 1];
  __shared__ float warp_best_v[kConsumerWarps];
  __shared__ long long warp_best_i[kConsumerWarps];
  __shared__ int is_last;

  constexpr int VE = Vec<WT>::kElems;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long K = a.k;
  const long long chunks = K / VE;
  const long long u0 = static_cast<long long>(blockIdx.x) * L.per_cta;
  const long long u1 = u0 + L.per_cta < L.units ? u0 + L.per_cta : L.units;
  const long long n_units = u1 > u0 ? u1 - u0 : 0;
  const long long n_stages = (n_units + L.stage_units - 1) / L.stage_units;

  if (tid == 0) {
    for (int s = 0; s < L.slots; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer: stream this CTA's rows into the ring ----
    pdl_launch_dependents();
    if (lane == 0) {
      for (long long s = 0; s < n_stages; ++s) {
        const int slot = static_cast<int>(s % L.slots);
        const long long round = s / L.slots;
        if (s == L.slots)  // ring primed: now ask L2 for the next kernel's weights
          prefetch_share(a.prefetch_ptr, a.prefetch_bytes, blockIdx.x, gridDim.x, 0, 1);
        if (round > 0 && !mbar_wait(empty + slot, static_cast<uint32_t>((round - 1) & 1))) {
          if (a.error_flag != nullptr) atomicExch(a.error_flag, 4);
          break;
        }
        const long long first = u0 + s * L.stage_units;
        const long long last = first + L.stage_units < u1 ? first + L.stage_units : u1;
        mbar_arrive_expect_tx(full + slot, static_cast<uint32_t>((last - first) * L.row_bytes));
        unsigned char* dst = ring + slot * L.stage_bytes;
        for (long long u = first; u < last; ++u)
          bulk_load(dst + (u - first) * L.row_bytes, unit_row(a, u, L.row_bytes),
                    static_cast<uint32_t>(L.row_bytes), full + slot);
      }
      if (n_stages <= L.slots)
        prefetch_share(a.prefetch_ptr, a.prefetch_bytes, blockIdx.x, gridDim.x, 0, 1);
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  pdl_launch_dependents();
  const int ctid = tid;  // 0 .. 255
  constexpr int kConsumers = kConsumerWarps * 32;
  long long xrow = a.x_index != nullptr ? load_index(a.x_index, 0, a.x_index_dtype) : 0;
  if (a.x_index != nullptr && (xrow < 0 || xrow >= a.index_rows)) {
    if (ctid == 0 && blockIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, 1);
    xrow = 0;
  }
  for (long long i = ctid; i < K; i += kConsumers) xs[i] = load_as_f32(a.x, xrow * K + i, a.x_dtype);
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
  if (a.norm != CB_NORM_NONE) {
    const NormSpec n{a.divisor, a.eps, a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y};
    float d;
    if (a.norm == CB_NORM_RMS_TABLE) {
      d = a.norm_table[xrow];
    } else {
      // consumer-only version of norm_block_sum (named barrier 1)
      __shared__ float total_sq;
      if (n.dt_sum != CB_F32) {
        if (ctid == 0) {
          float acc = round_to(__fmul_rn(xs[0], xs[0]), n.dt_sq);
          for (long long i = 1; i < K; ++i)
            acc = round_to(__fadd_rn(acc, round_to(__fmul_rn(xs[i], xs[i]), n.dt_sq)), n.dt_sum);
          total_sq = acc;
        }
      } else {
        float part = 0.0f;
        for (long long i = ctid; i < K; i += kConsumers)
          part = __fadd_rn(part, round_to(__fmul_rn(xs[i], xs[i]), n.dt_sq));
        part = warp_sum(part);
        if (lane == 0) norm_red[warp] = part;
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
        if (ctid == 0) {
          float acc = 0.0f;
          for (int w = 0; w < kConsumerWarps; ++w) acc += norm_red[w];
          total_sq = acc;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
      d = norm_finish_d(n, total_sq);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
    for (long long i = ctid; i < K; i += kConsumers)
      xs[i] = norm_apply(n, xs[i], d, load_as_f32(a.norm_w, i, a.norm_w_dtype), a.dt_norm_out);
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
  }
  long long rrow = 0;
  if (a.epilogue == CB_EPI_RESIDUAL && a.residual_index != nullptr) {
    rrow = load_index(a.residual_index, 0, a.residual_index_dtype);
    if (rrow < 0 || rrow >= a.index_rows) {
      if (ctid == 0 && blockIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, 1);
      rrow = 0;
    }
    rrow *= L.units;
  }

  float best_v = 0.0f, gate = 0.0f;
  long long best_i = -1;
  for (long long s = warp; s < n_stages; s += kConsumerWarps) {
    const int slot = static_cast<int>(s % L.slots);
    if (!mbar_wait(full + slot, static_cast<uint32_t>((s / L.slots) & 1))) {
      if (lane == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, 4);
      break;
    }
    const unsigned char* stage = ring + slot * L.stage_bytes;
    const long long first = u0 + s * L.stage_units;
    const long long last = first + L.stage_units < u1 ? first + L.stage_units : u1;
    for (long long u = first; u < last; ++u) {
      const uint4* row = reinterpret_cast<const uint4*>(stage + (u - first) * L.row_bytes);
      float acc = 0.0f;
      for (long long c = lane; c < chunks; c += 32) acc = Vec<WT>::dot(row[c], xs + c * VE, acc);
      const float total = warp_sum(acc);
      if (lane == 0) {
        switch (a.epilogue) {
          case CB_EPI_STORE: a.out[u] = total; break;
          case CB_EPI_RESIDUAL:
            a.out[u] = __fadd_rn(load_as_f32(a.residual, rrow + u, a.residual_dtype), total);
            break;
          case CB_EPI_SILU_MUL:
            if ((u & 1) == 0) {
              gate = total;
            } else {
              const float silu = __fdiv_rn(gate, __fadd_rn(expf(-gate), 1.0f));
              a.out[u >> 1] = __fmul_rn(silu, total);
            }
            break;
          default:  // CB_EPI_ARGMAX
            a.out[u] = total;
            if (best_i < 0 || argmax_better(total, u, best_v, best_i)) {
              best_v = total;
              best_i = u;
            }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  }

  if (a.epilogue != CB_EPI_ARGMAX) return;
  // ---- argmax: warp -> CTA -> scratch; the last CTA merges in CTA order ----
  if (lane == 0) {
    warp_best_v[warp] = best_v;
    warp_best_i[warp] = best_i;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
  if (ctid == 0) {
    float bv = 0.0f;
    long long bi = -1;
    for (int w = 0; w < kConsumerWarps; ++w) {
      if (warp_best_i[w] >= 0 && (bi < 0 || argmax_better(warp_best_v[w], warp_best_i[w], bv, bi))) {
        bv = warp_best_v[w];
        bi = warp_best_i[w];
      }
    }
    a.scratch_val[blockIdx.x] = bv;
    a.scratch_idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned ticket = atomicAdd(a.counter, 1u);
    is_last = ticket == gridDim.x - 1;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
  if (!is_last || ctid != 0) return;
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

int plan_gemv(const cb_gemv_args& a, Layout* L) {
  CB_REQUIRE(a.w_dtype == CB_BF16 || a.w_dtype == CB_F32, "gemv: weights must be bf16 or f32");
  CB_REQUIRE(a.n_w >= 1 && a.n_w <= 3, "gemv: 1..3 weight matrices");
  const int ve = a.w_dtype == CB_BF16 ? 8 : 4;
  CB_REQUIRE(a.k > 0 && a.k % ve == 0, "gemv: k=%lld must be a multiple of %d", a.k, ve);
  for (int i = 0; i < a.n_w; ++i)
    CB_REQUIRE((reinterpret_cast<uintptr_t>(a.w[i]) & 15) == 0, "gemv: weights must be 16-byte aligned");
  long long units = 0;
  if (a.epilogue == CB_EPI_SILU_MUL) {
    CB_REQUIRE(a.n_w == 2 && a.w_rows[0] == a.w_rows[1], "gemv: SwiGLU needs gate/up of equal rows");
    units = 2 * a.w_rows[0];
  } else {
    for (int i = 0; i < a.n_w; ++i) units += a.w_rows[i];
  }
  CB_REQUIRE(units > 0, "gemv: no rows");
  const long long row_bytes = a.k * (a.w_dtype == CB_BF16 ? 2 : 4);
  CB_REQUIRE(row_bytes <= 64 * 1024, "gemv: rows longer than 64 KiB are not supported");
  int stage_units = static_cast<int>(kStageTarget / row_bytes);
  if (stage_units < 1) stage_units = 1;
  if (a.epilogue == CB_EPI_SILU_MUL) stage_units = stage_units < 2 ? 2 : stage_units & ~1;
  const long long stage_bytes = stage_units * row_bytes;
  const size_t x_bytes = (static_cast<size_t>(a.k) * 4 + 15) & ~size_t(15);
  // two CTAs (this kernel + the next one, launched early) must fit an SM
  long long ring = kRingTarget;
  const long long budget = 110 * 1024 - static_cast<long long>(x_bytes);
  if (ring > budget) ring = budget;
  int slots = static_cast<int>(ring / stage_bytes);
  if (slots < 2) slots = 2;
  int grid = a.grid > 0 ? a.grid : sm_count();
  long long per = (units + grid - 1) / grid;
  if (a.epilogue == CB_EPI_SILU_MUL) per += per & 1;  // whole gate/up pairs per CTA
  grid = static_cast<int>((units + per - 1) / per);
  L->units = units;
  L->per_cta = per;
  L->grid = grid;
  L->stage_units = stage_units;
  L->slots = slots;
  L->row_bytes = row_bytes;
  L->stage_bytes = stage_bytes;
  L->ring_bytes = static_cast<size_t>(slots) * stage_bytes;
  L->smem = L->ring_bytes + x_bytes + 2 * slots * sizeof(uint64_t);
  CB_REQUIRE(L->smem <= 220 * 1024, "gemv: k too large for shared memory");
  if (a.epilogue == CB_EPI_ARGMAX)
    CB_REQUIRE(a.scratch_val && a.scratch_idx && a.counter && a.argmax_out, "gemv: argmax needs scratch");
  if (a.epilogue == CB_EPI_RESIDUAL) CB_REQUIRE(a.residual != nullptr, "gemv: residual missing");
  if (a.norm != CB_NORM_NONE) CB_REQUIRE(a.norm_w != nullptr, "gemv: norm weight missing");
  if (a.norm == CB_NORM_RMS_TABLE) CB_REQUIRE(a.norm_table && a.x_index, "gemv: norm table needs x_index");
  if (a.x_index != nullptr || a.residual_index != nullptr)
    CB_REQUIRE(a.index_rows > 0, "gemv: indexed rows need index_rows");
  return CB_OK;
}

template <typename WT>
cudaError_t launch_gemv(const cb_gemv_args& a, const Layout& L, cudaStream_t s) {
  auto kernel = gemv_kernel<WT>;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem));
  return launch(kernel, dim3(L.grid), dim3(kThreads), L.smem, s, a.pdl != 0, a, L);
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_gemv_grid(const cb_gemv_args* a, int* grid) {
  Layout L;
  const int st = plan_gemv(*a, &L);
  if (st != CB_OK) return st;
  *grid = L.grid;
  return CB_OK;
}

int cb_gemv(const cb_gemv_args* a, cb_stream_t stream) {
  Layout L;
  const int st = plan_gemv(*a, &L);
  if (st != CB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = a->w_dtype == CB_BF16 ? launch_gemv<uint16_t>(*a, L, s) : launch_gemv<float>(*a, L, s);
  if (e != cudaSuccess) {
    set_error("cb_gemv: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_gemv");
}

}  // extern "C"

// Streaming GEMV for single-token decode: y = x W^T, W row-major (out, in).
//
// Decode is bound by reading every weight byte once from HBM.  Design:
//  * one CTA per SM owns a contiguous range of "units" (weight rows); a
//    producer warp streams them with bulk copies (TMA engine,
//    cp.async.bulk + mbarrier transaction counts) into a shared-memory ring
//    of multi-row stages (>= 16 KiB each, ~128-180 KiB in flight per SM);
//  * the CTA also issues an L2 prefetch of its share of the NEXT kernel's
//    weights, so HBM keeps streaming across kernel boundaries;
//  * consumer warps own ring slots (slot s belongs to warp s % consumers, so
//    parity waits are never more than one phase behind) and multiply all R
//    rows of a stage at once: each 16-byte chunk of x is read from shared
//    memory once for R rows (x is stored as two conflict-free planes), R
//    independent FMA chains, one warp reduction per row, fixed order
//    (deterministic results);
//  * the input row x (optionally gathered by a device index and rms-normed
//    with the reference's roundings) is staged once per CTA;
//  * epilogues fuse the consumers the reference graph applies next:
//    residual add, SwiGLU silu(gate)*up (stage = [gate rows | up rows]), or
//    logits + greedy argmax (last-CTA merge in CTA order).
#include "gemv_core.cuh"

namespace cb {
namespace {

constexpr int kMaxConsumerWarps = 8;
constexpr int kThreads = (kMaxConsumerWarps + 1) * 32;  // + producer warp
constexpr int kMaxRows = kMaxStageRows;
constexpr long long kRingBudget = 180 * 1024;
constexpr long long kSmemBudget = 210 * 1024;

struct Layout {
  long long units, per_cta;
  int grid, rows, slots, consumers;
  long long row_bytes, stage_bytes;
  size_t ring_bytes, x_bytes, smem;
};

template <typename WT>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const cb_gemv_args a, const Layout L) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  float* xs = reinterpret_cast<float*>(smem + L.ring_bytes);  // staged x (k floats)
  float4* xa = reinterpret_cast<float4*>(smem + L.ring_bytes + L.x_bytes);
  float4* xb = xa + (a.k / 8 + 1);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.ring_bytes + 2 * L.x_bytes + 32);
  uint64_t* empty = full + L.slots;
  __shared__ float norm_red[kMaxConsumerWarps];
  __shared__ float total_sq;
  __shared__ float warp_best_v[kMaxConsumerWarps];
  __shared__ long long warp_best_i[kMaxConsumerWarps];
  __shared__ int is_last;

  constexpr int VE = Chunk<WT>::kElems;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ncons = L.consumers * 32;
  const long long K = a.k;
  const long long chunks = K / VE;
  const long long u0 = static_cast<long long>(blockIdx.x) * L.per_cta;
  const long long u1 = u0 + L.per_cta < L.units ? u0 + L.per_cta : L.units;
  const long long n_units = u1 > u0 ? u1 - u0 : 0;
  const long long n_stages = (n_units + L.rows - 1) / L.rows;
  const bool pairs = a.epilogue == CB_EPI_SILU_MUL;

  if (tid == 0) {
    for (int s = 0; s < L.slots; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kMaxConsumerWarps) {
    // ---------------- producer: stream this CTA's rows into the ring ----
    pdl_launch_dependents();
    // Producer lane j feeds consumer warp j: it issues stages j, j + C, ...
    // into the slots that warp owns, so C lanes issue copies in parallel.
    if (lane < L.consumers) {
      long long s = lane;
      for (; s < n_stages; s += L.consumers) {
        const int slot = static_cast<int>(s % L.slots);
        const long long round = s / L.slots;
        if (lane == 0 && s == L.slots)  // ring primed: ask L2 for the next kernel's weights
          prefetch_share(a.prefetch_ptr, a.prefetch_bytes, blockIdx.x, gridDim.x, 0, 1);
        if (round > 0 && !mbar_wait(empty + slot, static_cast<uint32_t>((round - 1) & 1))) {
          if (a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_WAIT_SLOT);
          break;
        }
        const long long first = u0 + s * L.rows;
        const long long last = first + L.rows < u1 ? first + L.rows : u1;
        mbar_arrive_expect_tx(full + slot, static_cast<uint32_t>((last - first) * L.row_bytes));
        unsigned char* dst = ring + slot * L.stage_bytes;
        if (pairs) {
          // [gate rows | up rows] of the stage's pairs: two contiguous copies
          const uint32_t bytes = static_cast<uint32_t>((last - first) / 2 * L.row_bytes);
          bulk_load(dst, unit_row(a, first, L.row_bytes), bytes, full + slot);
          bulk_load(dst + (L.rows / 2) * L.row_bytes, unit_row(a, first + 1, L.row_bytes), bytes, full + slot);
        } else {
          // one copy per run of rows inside the same weight matrix
          long long u = first;
          while (u < last) {
            long long end = a.w_rows[0];
            if (u >= end) end += a.w_rows[1];
            if (u >= end) end += a.w_rows[2];
            if (end > last) end = last;
            bulk_load(dst + (u - first) * L.row_bytes, unit_row(a, u, L.row_bytes),
                      static_cast<uint32_t>((end - u) * L.row_bytes), full + slot);
            u = end;
          }
        }
      }
      if (lane == 0 && n_stages <= L.slots)
        prefetch_share(a.prefetch_ptr, a.prefetch_bytes, blockIdx.x, gridDim.x, 0, 1);
      // Drain: this lane issued stages lane, lane + C, ..., s - C.  The last
      // one in each of its slots must have landed before the lane exits, so
      // no copy still writes this block's shared memory when it retires --
      // also after a consumer or producer wait gave up.  No later stage uses
      // these slots, so each wait is for exactly that copy's phase.
      const int per_lane = L.slots / L.consumers;
      for (int i = 1; i <= per_lane; ++i) {
        const long long t = s - static_cast<long long>(i) * L.consumers;
        if (t < lane) break;
        if (!mbar_wait(full + t % L.slots, static_cast<uint32_t>((t / L.slots) & 1))) {
          if (a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_WAIT_DRAIN);
          break;
        }
      }
    }
    return;
  }
  if (warp >= L.consumers) return;

  // ---------------- consumers: stage x (+ norm) ----------------
  pdl_wait();
  pdl_launch_dependents();
  long long xrow = a.x_index != nullptr ? load_index(a.x_index, 0, a.x_index_dtype) : 0;
  if (a.x_index != nullptr && (xrow < 0 || xrow >= a.index_rows)) {
    if (tid == 0 && blockIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_INDEX);
    xrow = 0;
  }
  for (long long i = tid; i < K; i += ncons) xs[i] = load_as_f32(a.x, xrow * K + i, a.x_dtype);
  consumers_sync(ncons);
  float d = 0.0f;
  NormSpec n{a.divisor, a.eps, a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y};
  if (a.norm == CB_NORM_RMS_TABLE) {
    d = a.norm_table[xrow];
  } else if (a.norm == CB_NORM_RMS) {
    if (n.dt_sum != CB_F32) {  // NumPy's sequential 16-bit-float sum
      if (tid == 0) {
        float acc = round_to(__fmul_rn(xs[0], xs[0]), n.dt_sq);
        for (long long i = 1; i < K; ++i)
          acc = round_to(__fadd_rn(acc, round_to(__fmul_rn(xs[i], xs[i]), n.dt_sq)), n.dt_sum);
        total_sq = acc;
      }
    } else {
      float part = 0.0f;
      for (long long i = tid; i < K; i += ncons) part = __fadd_rn(part, round_to(__fmul_rn(xs[i], xs[i]), n.dt_sq));
      part = warp_sum(part);
      if (lane == 0) norm_red[warp] = part;
      consumers_sync(ncons);
      if (tid == 0) {
        float acc = 0.0f;
        for (int w = 0; w < L.consumers; ++w) acc += norm_red[w];
        total_sq = acc;
      }
    }
    consumers_sync(ncons);
    d = norm_finish_d(n, total_sq);
  }
  // normalise and split into the two x planes
  for (long long c = tid; c < chunks; c += ncons) {
    float v[8];
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      const long long i = c * VE + e;
      v[e] = a.norm != CB_NORM_NONE
                 ? norm_apply(n, xs[i], d, load_as_f32(a.norm_w, i, a.norm_w_dtype), a.dt_norm_out)
                 : xs[i];
    }
    xa[c] = make_float4(v[0], v[1], v[2], v[3]);
    if (VE == 8) xb[c] = make_float4(v[4], v[5], v[6], v[7]);
  }
  consumers_sync(ncons);

  long long rrow = 0;
  if (a.epilogue == CB_EPI_RESIDUAL && a.residual_index != nullptr) {
    rrow = load_index(a.residual_index, 0, a.residual_index_dtype);
    if (rrow < 0 || rrow >= a.index_rows) {
      if (tid == 0 && blockIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_INDEX);
      rrow = 0;
    }
    rrow *= L.units;
  }

  // ---------------- consumers: this warp's stages ----------------
  float best_v = 0.0f;
  long long best_i = -1;
  for (long long s = warp; s < n_stages; s += L.consumers) {
    const int slot = static_cast<int>(s % L.slots);
    const bool ok = mbar_wait(full + slot, static_cast<uint32_t>((s / L.slots) & 1));
    if (!__all_sync(0xffffffffu, ok)) {  // the warp leaves together (shuffles follow)
      if (lane == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_WAIT_DATA);
      break;
    }
    const unsigned char* stage = ring + slot * L.stage_bytes;
    const long long first = u0 + s * L.rows;
    const int in_stage = static_cast<int>(first + L.rows < u1 ? L.rows : u1 - first);
    long long row_at[kMaxRows];
    float totals[kMaxRows];
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) {
      const int i = r < in_stage ? r : 0;  // pad with row 0 (result unused)
      row_at[r] = pairs ? (i & 1) * (L.rows / 2) + (i >> 1) : i;
    }
    switch (L.rows) {
      case 1: stage_dot<WT, 1>(stage, row_at, L.row_bytes, xa, xb, chunks, lane, totals); break;
      case 2: stage_dot<WT, 2>(stage, row_at, L.row_bytes, xa, xb, chunks, lane, totals); break;
      case 4: stage_dot<WT, 4>(stage, row_at, L.row_bytes, xa, xb, chunks, lane, totals); break;
      default: stage_dot<WT, 8>(stage, row_at, L.row_bytes, xa, xb, chunks, lane, totals); break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);  // slot free: reads are done
    // epilogue: lane i finishes row i (every lane holds every total)
    float mine = totals[0], next = 0.0f;
#pragma unroll
    for (int r = 1; r < kMaxRows; ++r) {
      if (lane == r) mine = totals[r];
      if (lane + 1 == r) next = totals[r];
    }
    if (lane < in_stage) {
      const long long u = first + lane;
      switch (a.epilogue) {
        case CB_EPI_STORE: a.out[u] = mine; break;
        case CB_EPI_RESIDUAL:
          a.out[u] = __fadd_rn(load_as_f32(a.residual, rrow + u, a.residual_dtype), mine);
          break;
        case CB_EPI_SILU_MUL:
          if ((lane & 1) == 0) {
            const float silu = __fdiv_rn(mine, __fadd_rn(expf(-mine), 1.0f));
            a.out[u >> 1] = __fmul_rn(silu, next);
          }
          break;
        default:  // CB_EPI_ARGMAX
          a.out[u] = mine;
      }
    }
    if (a.epilogue == CB_EPI_ARGMAX && lane == 0) {
      for (int i = 0; i < in_stage; ++i) {
        const long long u = first + i;
        if (best_i < 0 || argmax_better(totals[i], u, best_v, best_i)) {
          best_v = totals[i];
          best_i = u;
        }
      }
    }
  }

  if (a.epilogue != CB_EPI_ARGMAX) return;
  // ---- argmax: warp -> CTA -> scratch; the last CTA merges in CTA order ----
  if (lane == 0) {
    warp_best_v[warp] = best_v;
    warp_best_i[warp] = best_i;
  }
  consumers_sync(ncons);
  if (tid == 0) {
    float bv = 0.0f;
    long long bi = -1;
    for (int w = 0; w < L.consumers; ++w) {
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
  consumers_sync(ncons);
  if (!is_last) return;  // block-uniform: the last block merges with all its consumer threads
  __threadfence();
  const long long bi = argmax_merge(a.scratch_val, a.scratch_idx, static_cast<int>(gridDim.x), tid, ncons,
                                    warp_best_v, warp_best_i);
  if (tid == 0) {
    a.argmax_out[0] = bi;
    *a.counter = 0u;
  }
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
  const size_t x_bytes = (static_cast<size_t>(a.k) * 4 + 15) & ~size_t(15);
  const bool pairs = a.epilogue == CB_EPI_SILU_MUL;
  long long ring = kRingBudget;
  if (ring + 2 * static_cast<long long>(x_bytes) + 1024 > kSmemBudget)
    ring = kSmemBudget - 2 * static_cast<long long>(x_bytes) - 1024;
  // Ring shape: C consumer warps, each owning m >= 2 slots (its next stage is
  // in flight while it multiplies the current one), stages of `rows` rows
  // (power of two <= 8, even for SwiGLU).  Pick the shape with the most bytes
  // in flight, preferring more consumer warps, then stages of >= 8 KiB.
  int rows = 0, consumers = 0, slots = 0;
  long long best = -1;
  for (int c = kMaxConsumerWarps; c >= 2; c /= 2) {
    for (int r = pairs ? 2 : 1; r <= kMaxRows; r *= 2) {
      const long long stage = r * row_bytes;
      long long m = ring / (c * stage);
      if (m > 4) m = 4;
      if (m < 2) continue;
      const long long score = c * m * stage * 4 + (stage >= 8 * 1024 ? 2 : 0) + (c >= 4 ? 1 : 0);
      if (score > best) {
        best = score;
        rows = r;
        consumers = c;
        slots = static_cast<int>(c * m);
      }
    }
  }
  if (best < 0) {  // very long rows: single-buffered fallback
    rows = pairs ? 2 : 1;
    consumers = 2;
    while (consumers > 1 && consumers * rows * row_bytes > ring) consumers /= 2;
    slots = consumers;
  }
  CB_REQUIRE(slots * rows * row_bytes <= ring, "gemv: rows of %lld bytes do not fit the ring", row_bytes);
  const long long stage_bytes = rows * row_bytes;
  int grid = a.grid > 0 ? a.grid : sm_count();
  long long per = (units + grid - 1) / grid;
  if (pairs) per += per & 1;  // whole gate/up pairs per CTA
  grid = static_cast<int>((units + per - 1) / per);
  L->units = units;
  L->per_cta = per;
  L->grid = grid;
  L->rows = rows;
  L->slots = slots;
  L->consumers = consumers;
  L->row_bytes = row_bytes;
  L->stage_bytes = stage_bytes;
  L->ring_bytes = static_cast<size_t>(slots) * stage_bytes;
  L->x_bytes = x_bytes;
  L->smem = L->ring_bytes + 2 * x_bytes + 32 + 2 * slots * sizeof(uint64_t);
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

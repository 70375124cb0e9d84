// A whole decode step in one persistent, cooperative launch: cb_decode_step.
//
// Single-token decode reads every weight byte once; what a chain of ~110
// separate launches loses is the time between them (ramp-up, x staging, the
// tail of each launch), during which HBM idles.  Here the step is ONE grid
// of one block per SM, and the step's kernels become phases:
//
//  * the producer warp of each block streams the block's rows of EVERY GEMV
//    phase, in phase order, through a 16-slot shared-memory ring (bulk
//    copies, mbarrier transaction counts).  Weights do not depend on
//    activations, so it never waits for a phase -- only for free slots --
//    and it prefetches the block's rows of the next GEMV phase into L2, so
//    HBM keeps streaming while the consumers wait at a phase boundary;
//  * the 8 consumer warps run the phases in order.  Before phase p they wait
//    (bounded) until every block has finished phase p-1 (a grid-wide arrival
//    counter per phase).  Whatever does not depend on phase p-1 is loaded
//    BEFORE that wait: norm weights and the norm-table value of a GEMV
//    phase, the K/V cache rows of an attention item.  After it they load x
//    (every load of a thread issued at once: one round trip), apply SwiGLU
//    of the previous phase's [gate | up] output or merge the attention
//    splits, RMSNorm it in registers, multiply the ring stages and apply the
//    epilogue (store, residual, logits + argmax);
//  * attention phases run decode-attention work items (one per context split
//    and KV head, attn_core.cuh) on the consumer warps of the first blocks
//    and leave split partials; the O-projection phase that reads the
//    attention output merges them while staging x.
//
// Counters: every block arrives at counters[p] after phase p; the last block
// to finish the last phase zeroes them all for the next launch.  Buffers
// other blocks write during the launch are each written once per launch
// (one [gate | up] buffer per layer, too), so x staging may read them through
// L1; values a phase may rewrite (counters, argmax scratch, caches) are read
// through L2 (ld.global.cg).
#include <cstring>
#include <vector>

#include "attn_core.cuh"
#include "gemv_core.cuh"

namespace cb {
namespace {

constexpr int kStepConsumers = 8;                        // = attention's 8 warps
constexpr int kStepThreads = (kStepConsumers + 1) * 32;  // + producer warp
constexpr int kStepSlots = 2 * kStepConsumers;           // slot s owned by warp s % 8
constexpr long long kStepSmemMax = 227 * 1024 - 3 * 1024;  // dynamic; the rest is static
constexpr int kRowValsMax = 256;  // per-block row values: staged residuals, or SwiGLU gate/up totals
constexpr long long kNormStageMax = 16 * 1024;             // largest norm-weight vector staged
constexpr long long kPrefetchDefault = 0;  // L2 lookahead per block and phase (measured: none is best)
constexpr int kThreadChunks = 3;                         // x chunks per consumer thread
constexpr int kXMerge = 2;                               // internal x mode: merge attention splits

static_assert(kStepConsumers * 32 == kAttnThreads, "attention items run on the consumer warps");
static_assert(kStepSlots % kStepConsumers == 0, "slot ownership needs slots % consumers == 0");

struct alignas(16) PhaseDesc {
  int kind, x_mode, rows, splits;
  int x_vec, nw_vec;         // 16-byte vector loads allowed for x / norm weights
  int merge_in_kernel;       // attention: merge splits in the phase (else a later x stage does)
  int merge_splits, merge_hd;
  long long merge_heads;
  const float* merge_parts;  // kXMerge: the attention phase's split partials
  long long units, per_cta, row_bytes, items;
  long long cta0;  // GEMV: blocks [0, cta0) have no rows of this phase (see the prepare step)
  // Norm weights staged in shared memory (two slots, bulk copies): this
  // phase's ordinal among such phases (-1: read from global memory), and the
  // copy this phase's start issues -- the NEXT staged phase's weights.
  int norm_ord, next_norm_slot;
  int paired;  // SwiGLU: units are gate/up pairs; a block streams its gate rows, then the same up rows
  const void* next_norm_w;
  long long next_norm_bytes;
  const void* first_norm_w;  // phase 0 only: the copy issued at kernel start
  long long first_norm_bytes;
  // L2 prefetch of the NEXT phase's attention cache rows (set on the phase
  // before an attention phase): item i = blockIdx.x reads rows
  // [split * kAttnSplit, ...) of KV head i / pf_splits in both caches.
  const void* pf_k;
  const void* pf_v;
  long long pf_context, pf_row_bytes;
  int pf_items, pf_splits;
  cb_gemv_args g;
  cb_decode_attention_args at;
};
static_assert(sizeof(PhaseDesc) % 16 == 0 && sizeof(PhaseDesc) <= 1024, "descriptor copies move 16-byte pieces");

// Asynchronous copy of a phase descriptor into shared memory by the consumer
// threads (cp.async, no registers held); desc_wait + a barrier make it visible.
__device__ __forceinline__ void desc_copy(const PhaseDesc* src, PhaseDesc* dst, int tid) {
  constexpr int kPieces = static_cast<int>(sizeof(PhaseDesc) / 16);
  const char* s = reinterpret_cast<const char*>(src);
  char* d = reinterpret_cast<char*>(dst);
  for (int i = tid; i < kPieces; i += kAttnThreads)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(d + 16 * i)), "l"(s + 16 * i)
                 : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void desc_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

struct StepParams {
  const PhaseDesc* __restrict__ phases;
  int n_phases, grid;
  long long slot_bytes, ring_bytes, x_bytes, norm_bytes;  // norm_bytes: one norm-weight slot
  unsigned int* counters;
  int* error_flag;
  unsigned long long* timeline;  // optional stamps, see cb_decode_step_config
  long long prefetch_bytes;      // L2 lookahead per block and phase
  int lane_inflight;             // ring copies in flight per producer lane (1 or 2)
  int quiet_window;              // pause ring copies from a phase's wait until its x is staged
  int test_withhold;             // see cb_decode_step_config
};

enum {
  kStampWait = 0,    // consumers: phase begins (pre-wait loads issued next)
  kStampReady = 1,   // previous phase complete grid-wide
  kStampStaged = 2,  // x staged
  kStampDone = 3,    // phase done in this block
  kStampIssued = 4,  // producer issued the phase's last stage
  kStampLoaded = 5,  // thread 0's own x loads returned
  kStampFirst = 6,   // warp 0's first stage of the phase had landed
  kStampLastLoad = 7,  // the last warp's x loads returned (latest over warps)
  kStampNormed = 8,    // thread 0 normalised its x values
  kStampLastArrive = 9,  // the last warp reached the end of x staging
  kStampW0First = 10,    // warp 0's first stage of the phase had landed
  kStampW0Last = 11,     // warp 0 finished its last stage of the phase
  kStamps = 12
};

__device__ __forceinline__ void stamp(const StepParams& S, int p, int which) {
  if (S.timeline != nullptr)
    S.timeline[(static_cast<long long>(blockIdx.x) * S.n_phases + p) * kStamps + which] = global_ns();
}

__device__ __forceinline__ void raise_flag(int* flag, int code) {
  if (flag != nullptr) atomicCAS(flag, 0, code);
}

// Wait-type errors stop the step; index/position errors only flag results.
__device__ __forceinline__ bool step_failed(const int* flag) {
  return flag != nullptr && *reinterpret_cast<const volatile int*>(flag) >= CB_FLAG_WAIT_DATA;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Until *c >= target: bounded by time and polls, and abandoned once the
// step has failed elsewhere.
// The waits below read the clock (%globaltimer) only every few polls and
// start it at the first such read, so a wait that finds its condition met
// costs one poll.  `limit_ns` bounds a wait in time: the producer's waits on
// the consumers get twice the consumers' limit, so when a consumer wait runs
// out, it is the one that reports.
__device__ __forceinline__ bool waited_too_long(uint64_t* start, uint64_t limit_ns) {
  const uint64_t now = global_ns();
  if (*start == 0) {
    *start = now;
    return false;
  }
  return now - *start > limit_ns;
}

__device__ bool wait_counter(const unsigned* c, unsigned target, const int* flag) {
  uint64_t start = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (ld_acquire(c) >= target) return true;
    if ((i & 15u) == 15u && (step_failed(flag) || waited_too_long(&start, kWaitNs))) return false;
    __nanosleep(32);
  }
  return false;
}

// mbarrier wait that also gives up when this block has stopped (*stop != 0).
__device__ bool wait_or_stop(uint64_t* bar, uint32_t parity, const volatile int* stop,
                             uint64_t limit_ns = kWaitNs) {
  uint64_t start = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && (*stop != 0 || waited_too_long(&start, limit_ns))) return false;
  }
  return false;
}

// Producer side of the quiet window: until *quiet == 0 (bounded; false on
// timeout or once the block has stopped).
__device__ bool wait_loud(const int* quiet, const int* stop) {
  const volatile int* q = quiet;
  const volatile int* s = stop;
  if (*q == 0) return true;
  uint64_t start = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (*q == 0) return true;
    if (*s != 0 || ((i & 15u) == 15u && waited_too_long(&start, 2 * kWaitNs))) return false;
    __nanosleep(64);
  }
  return false;
}

__device__ __forceinline__ void unit_range(const PhaseDesc& P, long long cta, long long* u0, long long* u1) {
  const long long c = cta - P.cta0;
  const long long a = c < 0 ? P.units : c * P.per_cta, b = a + P.per_cta;
  *u0 = a < P.units ? a : P.units;
  *u1 = b < P.units ? b : P.units;
}

__device__ __forceinline__ long long block_stages(const PhaseDesc& P, long long cta) {
  long long u0, u1;
  unit_range(P, cta, &u0, &u1);
  const long long n_local = P.paired ? 2 * (u1 - u0) : u1 - u0;
  return (n_local + P.rows - 1) / P.rows;
}

// End of the run of rows starting at u that lies inside one weight matrix.
__device__ __forceinline__ long long run_end(const cb_gemv_args& a, long long u, long long last) {
  long long end = a.w_rows[0];
  if (u >= end) end += a.w_rows[1];
  if (u >= end) end += a.w_rows[2];
  return end < last ? end : last;
}

// L2 prefetch of this block's rows of phase P (up to `budget` bytes).
__device__ void prefetch_rows(const PhaseDesc& P, long long cta, long long budget) {
  long long u0, u1;
  unit_range(P, cta, &u0, &u1);
  for (long long u = u0; u < u1 && budget > 0;) {
    const long long end = run_end(P.g, u, u1);
    const char* src = unit_row(P.g, u, P.row_bytes);
    long long bytes = (end - u) * P.row_bytes;
    if (bytes > budget) bytes = budget;
    for (long long off = 0; off < bytes; off += 64 * 1024) {
      const long long piece = bytes - off < 64 * 1024 ? bytes - off : 64 * 1024;
      prefetch_l2(src + off, static_cast<uint32_t>(piece));
    }
    budget -= bytes;
    u = end;
  }
}

// x element i from the two planes (see Chunk in gemv_core.cuh).
template <int VE>
__device__ __forceinline__ float& plane_at(float4* xa, float4* xb, long long i) {
  const long long c = i / VE;
  const int e = static_cast<int>(i % VE);
  return e < 4 ? (&xa[c].x)[e] : (&xb[c].x)[e - 4];
}

// VE consecutive elements from element i0 as floats; `vec` = 16-byte vector
// loads (checked by prepare).  FRESH: data another block wrote earlier in
// this launch -- loaded through L1 (ld.global.ca), which is safe because
// every such buffer is written once per launch and this SM reads it only
// after the phase that wrote it (so L1 holds no older copy); the L1 also
// merges the lanes' partial-sector requests.  Otherwise read-only constants.
template <int VE, bool FRESH>
__device__ __forceinline__ void load_elems(const void* base, int dtype, long long i0, bool vec, float* v) {
  if (vec && dtype == CB_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i0);
    const float4 a = FRESH ? __ldca(p) : __ldg(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    if (VE == 8) {
      const float4 b = FRESH ? __ldca(p + 1) : __ldg(p + 1);
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
  } else if (vec && dtype == CB_BF16) {
    const uint16_t* q = static_cast<const uint16_t*>(base) + i0;
    if (VE == 8) {
      const uint4 w = FRESH ? __ldca(reinterpret_cast<const uint4*>(q)) : __ldg(reinterpret_cast<const uint4*>(q));
      unpack_bf16x8(w, v);
    } else {
      const uint2 w = FRESH ? __ldca(reinterpret_cast<const uint2*>(q)) : __ldg(reinterpret_cast<const uint2*>(q));
      v[0] = __uint_as_float(w.x << 16); v[1] = __uint_as_float(w.x & 0xffff0000u);
      v[2] = __uint_as_float(w.y << 16); v[3] = __uint_as_float(w.y & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int e = 0; e < VE; ++e) v[e] = load_as_f32(base, i0 + e, dtype);
  }
}

struct StepShared {
  float norm_red[kStepConsumers];
  float total_sq;
  float warp_best_v[kStepConsumers];
  long long warp_best_i[kStepConsumers];
  int last;
  int stop;
  // Quiet window: set from the start of a phase's wait until its x is
  // staged.  The producer issues no new ring copies meanwhile, so the
  // latency-critical loads of the window (phase counter, x, residual) do not
  // queue behind up to a ring of bulk data on the way to this SM.
  int quiet;
  float row_vals[kRowValsMax];  // this block's residual values, or its SwiGLU gate | up totals
};

// A load issued before the phase wait and consumed after it.  As volatile
// asm it keeps its place before the wait's barrier (the compiler may not
// sink it to its first use), so its latency hides behind the wait.
__device__ __forceinline__ float ld_early_f32(const float* p) {
  float r;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}

// What a GEMV phase's x staging can load before the phase wait.
template <int VE>
struct StagePre {
  float d;  // norm-table divisor of the row
  long long xrow;
};

// Norm weights of elements [i0, i0 + VE): from the phase's shared-memory slot
// (staged) or from global memory.  Generic loads serve both.
template <int VE>
__device__ __forceinline__ void norm_weights(const void* base, int dtype, long long i0, bool vec, float* w) {
  if (vec && dtype == CB_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i0);
    const float4 a = p[0];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    if (VE == 8) {
      const float4 b = p[1];
      w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
  } else if (vec && dtype == CB_BF16) {
    const uint16_t* q = static_cast<const uint16_t*>(base) + i0;
    if (VE == 8) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(q), w);
    } else {
      const uint2 a = *reinterpret_cast<const uint2*>(q);
      w[0] = __uint_as_float(a.x << 16); w[1] = __uint_as_float(a.x & 0xffff0000u);
      w[2] = __uint_as_float(a.y << 16); w[3] = __uint_as_float(a.y & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int e = 0; e < VE; ++e) w[e] = load_as_f32(base, i0 + e, dtype);
  }
}

template <typename WT>
__device__ void stage_pre(const PhaseDesc& P, StagePre<Chunk<WT>::kElems>& pre, int* flag, int tid) {
  constexpr int VE = Chunk<WT>::kElems;
  const cb_gemv_args& a = P.g;
  const long long chunks = a.k / VE;
  pre.xrow = 0;
  pre.d = 0.0f;
  if (a.x_index != nullptr) {
    pre.xrow = load_index(a.x_index, 0, a.x_index_dtype);
    if (pre.xrow < 0 || pre.xrow >= a.index_rows) {
      if (tid == 0 && blockIdx.x == 0) raise_flag(flag, CB_FLAG_INDEX);
      pre.xrow = 0;
    }
  }
  if (a.norm == CB_NORM_RMS_TABLE) pre.d = ld_early_f32(a.norm_table + pre.xrow);
  (void)chunks;
}

// x (+ SwiGLU / attention merge, + RMSNorm) into the planes; all consumer threads.
template <typename WT>
__device__ void stage_x(const PhaseDesc& P, const StagePre<Chunk<WT>::kElems>& pre, float4* xa, float4* xb,
                        StepShared& sh, int tid, long long res_first, int n_res, const StepParams& S, int p,
                        const unsigned char* norm_smem, uint64_t* norm_bar) {
  constexpr int VE = Chunk<WT>::kElems;
  constexpr int N = kAttnThreads;
  const cb_gemv_args& a = P.g;
  const long long K = a.k, chunks = K / VE;
  const int warp = tid >> 5, lane = tid & 31;
  const bool vec = P.x_vec != 0;
  // the block's residual values ride along with the x loads
  float res[kRowValsMax / kAttnThreads];
#pragma unroll
  for (int j = 0; j < kRowValsMax / kAttnThreads; ++j) {
    const int i = tid + j * N;
    if (i < n_res) res[j] = load_cg_f32(a.residual, res_first + i, a.residual_dtype);
  }
  float v[kThreadChunks][VE];
  if (P.x_mode == CB_X_SILU_MUL) {  // the SwiGLU epilogue's arithmetic
    float u[kThreadChunks][VE];
#pragma unroll
    for (int j = 0; j < kThreadChunks; ++j) {
      const long long c = tid + static_cast<long long>(j) * N;
      if (c < chunks) {
        load_elems<VE, true>(a.x, CB_F32, c * VE, vec, v[j]);
        load_elems<VE, true>(a.x, CB_F32, K + c * VE, vec, u[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kThreadChunks; ++j)
#pragma unroll
      for (int e = 0; e < VE; ++e)
        v[j][e] = __fmul_rn(__fdiv_rn(v[j][e], __fadd_rn(expf(-v[j][e]), 1.0f)), u[j][e]);
  } else if (P.x_mode == kXMerge) {
#pragma unroll
    for (int j = 0; j < kThreadChunks; ++j) {
      const long long c = tid + static_cast<long long>(j) * N;
      if (c < chunks)
        attention_merge_chunk(P.merge_parts, P.merge_heads, P.merge_hd, P.merge_splits, c * VE, VE, v[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kThreadChunks; ++j) {
      const long long c = tid + static_cast<long long>(j) * N;
      if (c < chunks) load_elems<VE, true>(a.x, a.x_dtype, pre.xrow * K + c * VE, vec, v[j]);
    }
  }
  if (lane == 0 && S.timeline != nullptr) {  // once this lane's values have arrived
    asm volatile("" ::"f"(v[0][0]));
    if (tid == 0) stamp(S, p, kStampLoaded);
    atomicMax(S.timeline + (static_cast<long long>(blockIdx.x) * S.n_phases + p) * kStamps + kStampLastLoad,
              static_cast<unsigned long long>(global_ns()));
  }
  if (a.norm != CB_NORM_NONE) {
    const NormSpec n{a.divisor, a.eps, a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y};
    float d = pre.d;
    if (a.norm == CB_NORM_RMS) {
      if (n.dt_sum != CB_F32) {  // NumPy's sequential 16-bit-float sum, over the raw planes
#pragma unroll
        for (int j = 0; j < kThreadChunks; ++j) {
          const long long c = tid + static_cast<long long>(j) * N;
          if (c < chunks) {
            xa[c] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
            if (VE == 8) xb[c] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
          }
        }
        consumers_sync(N);
        if (tid == 0) {
          const float x0 = plane_at<VE>(xa, xb, 0);
          float acc = round_to(__fmul_rn(x0, x0), n.dt_sq);
          for (long long i = 1; i < K; ++i) {
            const float xi = plane_at<VE>(xa, xb, i);
            acc = round_to(__fadd_rn(acc, round_to(__fmul_rn(xi, xi), n.dt_sq)), n.dt_sum);
          }
          sh.total_sq = acc;
        }
      } else {
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < kThreadChunks; ++j) {
          const long long c = tid + static_cast<long long>(j) * N;
          if (c < chunks)
#pragma unroll
            for (int e = 0; e < VE; ++e) part = __fadd_rn(part, round_to(__fmul_rn(v[j][e], v[j][e]), n.dt_sq));
        }
        part = warp_sum(part);
        if (lane == 0) sh.norm_red[warp] = part;
      }
      consumers_sync(N);
      if (tid == 0) stamp(S, p, kStampFirst);
      if (n.dt_sum != CB_F32) {
        d = norm_finish_d(n, sh.total_sq);
      } else {  // every thread adds the warp partials in the same order: no second barrier
        float acc = 0.0f;
        for (int w = 0; w < kStepConsumers; ++w) acc += sh.norm_red[w];
        d = norm_finish_d(n, acc);
      }
    }
    const void* wbase = a.norm_w;
    bool wvec = P.nw_vec != 0;
    if (P.norm_ord >= 0) {  // staged by a bulk copy issued phases ago
      const int slot = P.norm_ord & 1;
      if (!wait_or_stop(norm_bar + slot, static_cast<uint32_t>((P.norm_ord >> 1) & 1), &sh.stop)) {
        raise_flag(S.error_flag, CB_FLAG_WAIT_DATA);  // results invalid; the step stops next phase
        sh.stop = 1;
      }
      wbase = norm_smem + slot * S.norm_bytes;
      wvec = true;
    }
#pragma unroll
    for (int j = 0; j < kThreadChunks; ++j) {
      const long long c = tid + static_cast<long long>(j) * N;
      if (c >= chunks) continue;
      float w[VE];
      norm_weights<VE>(wbase, a.norm_w_dtype, c * VE, wvec, w);
#pragma unroll
      for (int e = 0; e < VE; ++e) v[j][e] = norm_apply(n, v[j][e], d, w[e], a.dt_norm_out);
    }
    if (tid == 0 && S.timeline != nullptr) {
      asm volatile("" ::"f"(v[0][0]));
      stamp(S, p, kStampNormed);
    }
  }
#pragma unroll
  for (int j = 0; j < kThreadChunks; ++j) {
    const long long c = tid + static_cast<long long>(j) * N;
    if (c < chunks) {
      xa[c] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      if (VE == 8) xb[c] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
    }
  }
#pragma unroll
  for (int j = 0; j < kRowValsMax / kAttnThreads; ++j) {
    const int i = tid + j * N;
    if (i < n_res) sh.row_vals[i] = res[j];
  }
  if (lane == 0 && S.timeline != nullptr)
    atomicMax(S.timeline + (static_cast<long long>(blockIdx.x) * S.n_phases + p) * kStamps + kStampLastArrive,
              static_cast<unsigned long long>(global_ns()));
  consumers_sync(N);
}

// One GEMV phase on the consumer warps; g = this block's first ring stage.
template <typename WT>
__device__ void gemv_phase(const PhaseDesc& P, const StagePre<Chunk<WT>::kElems>& pre, const StepParams& S,
                           int p, long long g, unsigned char* ring, uint64_t* full, uint64_t* empty, float4* xa,
                           const unsigned char* norm_smem, uint64_t* norm_bar, StepShared& sh, int tid) {
  constexpr int VE = Chunk<WT>::kElems;
  constexpr int N = kAttnThreads;
  constexpr int C = kStepConsumers;
  const cb_gemv_args& a = P.g;
  const int warp = tid >> 5, lane = tid & 31;
  long long u0, u1;
  unit_range(P, blockIdx.x, &u0, &u1);
  // the block's rows in stream order: its units, or for SwiGLU its gate rows
  // then the same up rows (block-local index j)
  const long long n_units = u1 - u0;
  const long long n_local = P.paired ? 2 * n_units : n_units;
  const long long n_stages = (n_local + P.rows - 1) / P.rows;
  const long long chunks = a.k / VE;
  float4* xb = xa + (chunks + 1);
  float best_v = 0.0f;
  long long best_i = -1;

  if (n_stages > 0) {
    long long rrow = 0;
    if (a.epilogue == CB_EPI_RESIDUAL && a.residual_index != nullptr) {
      rrow = load_index(a.residual_index, 0, a.residual_index_dtype);
      if (rrow < 0 || rrow >= a.index_rows) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(S.error_flag, CB_FLAG_INDEX);
        rrow = 0;
      }
      rrow *= P.units;
    }
    // residual values of this block's rows, staged with x when they fit
    const bool res_staged = a.epilogue == CB_EPI_RESIDUAL && n_units <= kRowValsMax;
    stage_x<WT>(P, pre, xa, xb, sh, tid, rrow + u0, res_staged ? static_cast<int>(n_units) : 0, S, p, norm_smem,
                norm_bar);
    if (tid == 0) {
      stamp(S, p, kStampStaged);
      *reinterpret_cast<volatile int*>(&sh.quiet) = 0;  // staged: the producer may stream again
    }
    for (long long s = ((warp - g) % C + C) % C; s < n_stages; s += C) {
      const long long gs = g + s;
      const int slot = static_cast<int>(gs % kStepSlots);
      bool ok = wait_or_stop(full + slot, static_cast<uint32_t>((gs / kStepSlots) & 1), &sh.stop);
      ok = __all_sync(0xffffffffu, ok);  // the warp leaves together
      if (!ok) {
        if (lane == 0) {
          raise_flag(S.error_flag, CB_FLAG_WAIT_DATA);
          sh.stop = 1;
        }
        break;
      }
      if (tid == 0 && s < C) stamp(S, p, kStampW0First);
      const unsigned char* stage = ring + slot * S.slot_bytes;
      const long long first = s * P.rows;  // block-local
      const int in_stage = static_cast<int>(first + P.rows < n_local ? P.rows : n_local - first);
      long long row_at[kMaxStageRows];
      float totals[kMaxStageRows];
#pragma unroll
      for (int r = 0; r < kMaxStageRows; ++r) row_at[r] = r < in_stage ? r : 0;
      switch (P.rows) {
        case 1: stage_dot<WT, 1>(stage, row_at, P.row_bytes, xa, xb, chunks, lane, totals); break;
        case 2: stage_dot<WT, 2>(stage, row_at, P.row_bytes, xa, xb, chunks, lane, totals); break;
        case 3: stage_dot<WT, 3>(stage, row_at, P.row_bytes, xa, xb, chunks, lane, totals); break;
        case 4: stage_dot<WT, 4>(stage, row_at, P.row_bytes, xa, xb, chunks, lane, totals); break;
        default: stage_dot<WT, 8>(stage, row_at, P.row_bytes, xa, xb, chunks, lane, totals); break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + slot);  // slot free: reads are done
      float mine = totals[0];
#pragma unroll
      for (int r = 1; r < kMaxStageRows; ++r)
        if (lane == r) mine = totals[r];
      if (lane < in_stage) {
        const long long j = first + lane;
        if (P.paired) {  // gate / up totals of the block's rows, combined below
          sh.row_vals[j] = mine;
        } else if (a.epilogue == CB_EPI_RESIDUAL) {
          const long long u = u0 + j;
          a.out[u] = __fadd_rn(res_staged ? sh.row_vals[j] : load_cg_f32(a.residual, rrow + u, a.residual_dtype),
                               mine);
        } else {  // CB_EPI_STORE, CB_EPI_ARGMAX (logits)
          a.out[u0 + j] = mine;
        }
      }
      if (a.epilogue == CB_EPI_ARGMAX && lane == 0) {
        for (int i = 0; i < in_stage; ++i) {
          const long long u = u0 + first + i;
          if (best_i < 0 || argmax_better(totals[i], u, best_v, best_i)) {
            best_v = totals[i];
            best_i = u;
          }
        }
      }
    }
    if (tid == 0) stamp(S, p, kStampW0Last);
    if (P.paired) {  // SwiGLU: silu(gate) * up, as the gemv epilogue computes it
      consumers_sync(N);
      for (long long t = tid; t < n_units; t += N) {
        const float gate = sh.row_vals[t], up = sh.row_vals[n_units + t];
        a.out[u0 + t] = __fmul_rn(__fdiv_rn(gate, __fadd_rn(expf(-gate), 1.0f)), up);
      }
    }
  }

  if (a.epilogue != CB_EPI_ARGMAX) return;
  // argmax: warp -> block -> scratch; the last block merges in block order
  if (lane == 0) {
    sh.warp_best_v[warp] = best_v;
    sh.warp_best_i[warp] = best_i;
  }
  consumers_sync(N);
  if (tid == 0) {
    float bv = 0.0f;
    long long bi = -1;
    for (int w = 0; w < C; ++w) {
      if (sh.warp_best_i[w] >= 0 && (bi < 0 || argmax_better(sh.warp_best_v[w], sh.warp_best_i[w], bv, bi))) {
        bv = sh.warp_best_v[w];
        bi = sh.warp_best_i[w];
      }
    }
    a.scratch_val[blockIdx.x] = bv;
    a.scratch_idx[blockIdx.x] = bi;
    const unsigned ticket = ticket_acq_rel(a.counter);  // releases this block's partial
    sh.last = ticket == gridDim.x - 1;
  }
  consumers_sync(N);
  if (!sh.last) return;  // block-uniform: the last block merges with all its consumer threads
  const long long bi = argmax_merge(a.scratch_val, a.scratch_idx, static_cast<int>(gridDim.x), tid, N,
                                    sh.warp_best_v, sh.warp_best_i);
  if (tid == 0) {
    a.argmax_out[0] = bi;
    *a.counter = 0u;
  }
}

template <typename WT, int HD>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepParams S) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ StepShared sh;
  __shared__ PhaseDesc sh_desc[2];
  unsigned char* ring = smem;
  float4* xa = reinterpret_cast<float4*>(smem + S.ring_bytes);
  unsigned char* norm_smem = smem + S.ring_bytes + S.x_bytes;  // two norm-weight slots
  uint64_t* full = reinterpret_cast<uint64_t*>(norm_smem + 2 * S.norm_bytes);
  uint64_t* empty = full + kStepSlots;
  uint64_t* norm_bar = empty + kStepSlots;  // one per norm-weight slot
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int C = kStepConsumers;
  constexpr int VE = Chunk<WT>::kElems;

  if (tid == 0) {
    for (int s = 0; s < kStepSlots; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(norm_bar, 1);
    mbar_init(norm_bar + 1, 1);
    mbar_fence_init();
    sh.stop = 0;
    sh.last = 0;
    sh.quiet = S.quiet_window;  // phase 0 stages x first
  }
  __syncthreads();

  if (warp == C) {
    // ---------------- producer: every GEMV phase's rows, in phase order ----
    if (lane < C) {
      long long g = 0, last = -1;
      bool stop = false;
      for (int p = 0; p < S.n_phases && !stop; ++p) {
        const PhaseDesc* Pp = S.phases + p;
        if (Pp->kind != CB_PHASE_GEMV) continue;
        // what the issue loop needs, in registers: the polls below clobber
        // memory, so fields read through Pp would be reloaded from the table
        const long long units = Pp->units, per_cta = Pp->per_cta, row_bytes = Pp->row_bytes;
        const long long rows = Pp->rows;
        const long long r0 = Pp->g.w_rows[0], r01 = r0 + Pp->g.w_rows[1];
        const char* w0 = static_cast<const char*>(Pp->g.w[0]);
        const char* w1 = static_cast<const char*>(Pp->g.w[1]);
        const char* w2 = static_cast<const char*>(Pp->g.w[2]);
        const bool paired = Pp->paired != 0;
        if (lane == 0 && S.prefetch_bytes > 0) {  // L2 lookahead: the next GEMV phase (wrapping)
          int q = p + 1;
          while (q < S.n_phases && S.phases[q].kind != CB_PHASE_GEMV) ++q;
          if (q == S.n_phases) {
            q = 0;
            while (S.phases[q].kind != CB_PHASE_GEMV) ++q;
          }
          prefetch_rows(S.phases[q], blockIdx.x, S.prefetch_bytes);
        }
        const long long c = static_cast<long long>(blockIdx.x) - Pp->cta0;
        const long long lo = c < 0 ? units : c * per_cta;
        const long long u0 = lo < units ? lo : units;
        const long long u1 = lo + per_cta < units ? lo + per_cta : units;
        // block-local rows j: its units in order, or (SwiGLU) its gate rows then its up rows
        const long long n_units = u1 - u0;
        const long long n_local = paired ? 2 * n_units : n_units;
        const long long n_stages = (n_local + rows - 1) / rows;
        for (long long s = ((lane - g) % C + C) % C; s < n_stages; s += C) {
          const long long gs = g + s;
          const int slot = static_cast<int>(gs % kStepSlots);
          const long long round = gs / kStepSlots;
          if (round > 0 &&
              !wait_or_stop(empty + slot, static_cast<uint32_t>((round - 1) & 1), &sh.stop, 2 * kWaitNs)) {
            if (!sh.stop) raise_flag(S.error_flag, CB_FLAG_WAIT_SLOT);
            stop = true;
            break;
          }
          // with one copy in flight per lane, the lane's previous copy lands first
          // (its slot is not reused before it is consumed, so the parity is exact)
          if (S.lane_inflight == 1 && last >= 0 &&
              !wait_or_stop(full + last % kStepSlots, static_cast<uint32_t>((last / kStepSlots) & 1), &sh.stop,
                            2 * kWaitNs)) {
            if (!sh.stop) raise_flag(S.error_flag, CB_FLAG_WAIT_SLOT);
            stop = true;
            break;
          }
          if (!wait_loud(&sh.quiet, &sh.stop)) {
            if (!sh.stop) raise_flag(S.error_flag, CB_FLAG_WAIT_SLOT);
            stop = true;
            break;
          }
          const long long first = s * rows;
          const long long end = first + rows < n_local ? first + rows : n_local;
          unsigned char* dst = ring + slot * S.slot_bytes;
          mbar_arrive_expect_tx(full + slot, static_cast<uint32_t>((end - first) * row_bytes));
          for (long long j = first; j < end;) {  // one copy per run of rows inside one matrix
            long long stop_j;
            const char* src;
            if (paired) {
              if (j < n_units) {
                stop_j = n_units < end ? n_units : end;
                src = w0 + (u0 + j) * row_bytes;
              } else {
                stop_j = end;
                src = w1 + (u0 + j - n_units) * row_bytes;
              }
            } else {
              const long long u = u0 + j;
              if (u < r0) {
                stop_j = r0 - u0 < end ? r0 - u0 : end;
                src = w0 + u * row_bytes;
              } else if (u < r01) {
                stop_j = r01 - u0 < end ? r01 - u0 : end;
                src = w1 + (u - r0) * row_bytes;
              } else {
                stop_j = end;
                src = w2 + (u - r01) * row_bytes;
              }
            }
            bulk_load(dst + (j - first) * row_bytes, src, static_cast<uint32_t>((stop_j - j) * row_bytes),
                      full + slot);
            j = stop_j;
          }
          last = gs;
        }
        g += n_stages;
        if (lane == 0) stamp(S, p, kStampIssued);
      }
      // Drain: this lane issued every stage gs == lane (mod C) up to `last`,
      // alternating between its kStepSlots / C slots.  Their last copies
      // must land before the lane exits (no copy may outlive the block);
      // nothing is issued after them, so each wait is for exactly that phase.
      for (int i = 0; i < kStepSlots / C; ++i) {
        const long long t = last - static_cast<long long>(i) * C;
        if (last < 0 || t < 0) break;
        if (!mbar_wait(full + t % kStepSlots, static_cast<uint32_t>((t / kStepSlots) & 1))) {
          raise_flag(S.error_flag, CB_FLAG_WAIT_DRAIN);
          break;
        }
      }
    }
    return;
  }

  // ---------------- consumers: the phases in order ----------------
  // Phase descriptors live in shared memory (double-buffered, phase p+1's
  // copied while phase p runs): the barriers' memory clobbers would otherwise
  // reload every field from the table in global memory.
  float* attn_smem = reinterpret_cast<float*>(xa);
  desc_copy(S.phases, &sh_desc[0], tid);
  desc_wait();
  consumers_sync(kAttnThreads);
  // Norm weights: thread 0 issues each staged phase's copy one staged phase
  // ahead (the first one now), into the slot its ordinal selects.
  int norm_issued = 0;
  if (tid == 0 && sh_desc[0].first_norm_w != nullptr) {
    mbar_arrive_expect_tx(norm_bar, static_cast<uint32_t>(sh_desc[0].first_norm_bytes));
    bulk_load(norm_smem, sh_desc[0].first_norm_w, static_cast<uint32_t>(sh_desc[0].first_norm_bytes), norm_bar);
    norm_issued = 1;
  }
  long long g = 0;
  for (int p = 0; p < S.n_phases; ++p) {
    const PhaseDesc& P = sh_desc[p & 1];
    if (p + 1 < S.n_phases) desc_copy(S.phases + p + 1, &sh_desc[(p + 1) & 1], tid);
    if (tid == 0 && P.next_norm_w != nullptr) {  // its slot's previous contents were used two staged phases ago
      const int slot = P.next_norm_slot;
      mbar_arrive_expect_tx(norm_bar + slot, static_cast<uint32_t>(P.next_norm_bytes));
      bulk_load(norm_smem + slot * S.norm_bytes, P.next_norm_w, static_cast<uint32_t>(P.next_norm_bytes),
                norm_bar + slot);
      ++norm_issued;
    }
    // the next phase's attention item reads its K/V cache rows right after
    // this phase: fetch them into L2 now, off every critical path
    if (tid == 32 && blockIdx.x < P.pf_items) {
      const long long grp = blockIdx.x / P.pf_splits, lo = (blockIdx.x % P.pf_splits) * kAttnSplit;
      const long long rows = P.pf_context - lo < kAttnSplit ? P.pf_context - lo : kAttnSplit;
      const long long off = (grp * P.pf_context + lo) * P.pf_row_bytes;
      prefetch_l2(static_cast<const char*>(P.pf_k) + off, static_cast<uint32_t>(rows * P.pf_row_bytes));
      prefetch_l2(static_cast<const char*>(P.pf_v) + off, static_cast<uint32_t>(rows * P.pf_row_bytes));
    }
    // before the wait: everything that does not depend on phase p-1
    if (tid == 0 && S.quiet_window) *reinterpret_cast<volatile int*>(&sh.quiet) = 1;
    StagePre<VE> pre;
    const bool gemv = P.kind == CB_PHASE_GEMV;
    if (gemv) {
      if (block_stages(P, blockIdx.x) > 0) stage_pre<WT>(P, pre, S.error_flag, tid);
    } else if (blockIdx.x < P.items) {
      attention_stage_cache<HD>(P.at, static_cast<int>(blockIdx.x / P.splits),
                                static_cast<int>(blockIdx.x % P.splits), attn_smem, tid);
    }
    if (tid == 0) stamp(S, p, kStampWait);
    if (p > 0) {
      if (tid == 0 && !wait_counter(S.counters + p - 1, static_cast<unsigned>(S.grid), S.error_flag)) {
        raise_flag(S.error_flag, CB_FLAG_WAIT_PHASE);
        sh.stop = 1;
      }
    }
    consumers_sync(kAttnThreads);  // also orders the attention staging before its use
    if (*reinterpret_cast<volatile int*>(&sh.stop) != 0) break;
    if (tid == 0) stamp(S, p, kStampReady);
    if (gemv) {
      if (tid == 0 && block_stages(P, blockIdx.x) == 0) *reinterpret_cast<volatile int*>(&sh.quiet) = 0;
      gemv_phase<WT>(P, pre, S, p, g, ring, full, empty, xa, norm_smem, norm_bar, sh, tid);  // ends the quiet window
      g += block_stages(P, blockIdx.x);
    } else {
      for (long long it = blockIdx.x; it < P.items; it += S.grid) {
        const int grp = static_cast<int>(it / P.splits), split = static_cast<int>(it % P.splits);
        if (it != blockIdx.x) {  // later items of this block: stage after the previous one
          attn_sync();
          attention_stage_cache<HD>(P.at, grp, split, attn_smem, tid);
          attn_sync();
        }
        unsigned long long* item_stamps =
            S.timeline != nullptr && it == blockIdx.x
                ? S.timeline + (static_cast<long long>(blockIdx.x) * S.n_phases + p) * kStamps + kStampLoaded
                : nullptr;
        attention_finish<HD>(P.at, grp, split, P.splits, attn_smem, &sh.last, tid, P.merge_in_kernel != 0,
                             item_stamps);
      }
      if (tid == 0) *reinterpret_cast<volatile int*>(&sh.quiet) = 0;
    }
    desc_wait();                   // phase p+1's descriptor has landed ...
    consumers_sync(kAttnThreads);  // ... and this block's phase-p writes are issued
    if (tid == 0) stamp(S, p, kStampDone);
    if (tid == 0 && *reinterpret_cast<volatile int*>(&sh.stop) == 0) {
      if (p < S.n_phases - 1) {
        if (!(p == 0 && S.test_withhold == static_cast<int>(blockIdx.x) + 1))
          arrive_release(S.counters + p);  // the barrier above ordered the block's writes
      } else if (ticket_acq_rel(S.counters + p) == static_cast<unsigned>(S.grid) - 1) {
        // every block has finished every phase: zero the counters for the next step
        for (int q = 0; q < S.n_phases; ++q) S.counters[q] = 0u;
        __threadfence();
      }
    }
  }
  // Drain: no norm-weight copy may outlive the block (after an early stop
  // the last two issued may still be in flight; waits on landed ones return).
  if (tid == 0) {
    for (int ord = norm_issued - 1; ord >= 0 && ord >= norm_issued - 2; --ord) {
      if (!mbar_wait(norm_bar + (ord & 1), static_cast<uint32_t>((ord >> 1) & 1))) {
        raise_flag(S.error_flag, CB_FLAG_WAIT_DRAIN);
        break;
      }
    }
  }
  (void)lane;
}

long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }

int launch_step(const StepParams& S, const cb_decode_step_config& c, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(c.grid));
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(c.smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all blocks resident: they wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
#define CB_STEP_CASE(WT, HD)                                                                          \
  {                                                                                                  \
    auto kernel = decode_step_kernel<WT, HD>;                                                         \
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(c.smem)); \
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, kernel, S);                                   \
  }
  const int hd = c.head_size == 0 ? 64 : c.head_size;
  if (c.w_dtype == CB_BF16) {
    switch (hd) {
      case 32: CB_STEP_CASE(uint16_t, 32) break;
      case 64: CB_STEP_CASE(uint16_t, 64) break;
      case 128: CB_STEP_CASE(uint16_t, 128) break;
      default: CB_STEP_CASE(uint16_t, 256) break;
    }
  } else {
    switch (hd) {
      case 32: CB_STEP_CASE(float, 32) break;
      case 64: CB_STEP_CASE(float, 64) break;
      case 128: CB_STEP_CASE(float, 128) break;
      default: CB_STEP_CASE(float, 256) break;
    }
  }
#undef CB_STEP_CASE
  if (e != cudaSuccess) {
    set_error("cb_decode_step: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_decode_step");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Whether [p, p + bytes) overlaps [q, q + qbytes).
bool overlaps(const void* p, long long bytes, const void* q, long long qbytes) {
  if (p == nullptr || q == nullptr) return false;
  const auto a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(q);
  return a < b + static_cast<uintptr_t>(qbytes) && b < a + static_cast<uintptr_t>(bytes);
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

long long cb_decode_step_table_bytes(int n_phases) {
  return n_phases > 0 ? static_cast<long long>(n_phases) * static_cast<long long>(sizeof(PhaseDesc)) : 0;
}

int cb_decode_step_prepare(const cb_step_phase* phases, int n_phases, void* table, long long table_bytes,
                           int flags, cb_decode_step_config* config) {
  CB_REQUIRE(phases != nullptr && n_phases > 0 && table != nullptr && config != nullptr,
             "decode step: phases, table and config are required");
  CB_REQUIRE(table_bytes >= cb_decode_step_table_bytes(n_phases), "decode step: table of %lld bytes is too small",
             table_bytes);
  CB_REQUIRE(aligned16(table), "decode step: table must be 16-byte aligned");
  const int grid = sm_count();
  std::vector<PhaseDesc> desc(static_cast<size_t>(n_phases));
  int w_dtype = -1, head_size = 0, n_gemv = 0;
  long long max_row = 0, x_bytes = 1024;
  for (int i = 0; i < n_phases; ++i) {
    const cb_step_phase& ph = phases[i];
    PhaseDesc& d = desc[static_cast<size_t>(i)];
    std::memset(&d, 0, sizeof(d));
    d.kind = ph.kind;
    d.x_mode = ph.x_mode;
    if (ph.kind == CB_PHASE_GEMV) {
      const cb_gemv_args& a = ph.gemv;
      CB_REQUIRE(a.w_dtype == CB_BF16 || a.w_dtype == CB_F32, "decode step phase %d: weights must be bf16 or f32", i);
      CB_REQUIRE(w_dtype < 0 || w_dtype == a.w_dtype, "decode step phase %d: mixed weight dtypes", i);
      w_dtype = a.w_dtype;
      CB_REQUIRE(a.n_w >= 1 && a.n_w <= 3, "decode step phase %d: 1..3 weight matrices", i);
      const int ve = a.w_dtype == CB_BF16 ? 8 : 4;
      CB_REQUIRE(a.k > 0 && a.k % ve == 0, "decode step phase %d: k=%lld must be a multiple of %d", i, a.k, ve);
      CB_REQUIRE(a.k / ve <= static_cast<long long>(kThreadChunks) * kAttnThreads,
                 "decode step phase %d: k=%lld exceeds the %d x staging elements", i, a.k,
                 kThreadChunks * kAttnThreads * ve);
      long long units = 0;
      for (int w = 0; w < a.n_w; ++w) {
        CB_REQUIRE(a.w[w] != nullptr && aligned16(a.w[w]), "decode step phase %d: weights must be 16-byte aligned",
                   i);
        CB_REQUIRE(a.w_rows[w] > 0, "decode step phase %d: empty weight matrix", i);
        units += a.w_rows[w];
      }
      for (int w = a.n_w; w < 3; ++w) CB_REQUIRE(a.w_rows[w] == 0, "decode step phase %d: unused w_rows must be 0", i);
      CB_REQUIRE(a.epilogue == CB_EPI_STORE || a.epilogue == CB_EPI_RESIDUAL || a.epilogue == CB_EPI_ARGMAX ||
                     a.epilogue == CB_EPI_SILU_MUL,
                 "decode step phase %d: unknown epilogue %d", i, a.epilogue);
      if (a.epilogue == CB_EPI_SILU_MUL) {  // gate/up pairs: units are pairs
        CB_REQUIRE(a.n_w == 2 && a.w_rows[0] == a.w_rows[1], "decode step phase %d: SwiGLU needs gate/up of equal rows",
                   i);
        units = a.w_rows[0];
        CB_REQUIRE((units + grid - 1) / grid * 2 <= kRowValsMax,
                   "decode step phase %d: %lld SwiGLU rows per block exceed %d", i, (units + grid - 1) / grid,
                   kRowValsMax / 2);
        d.paired = 1;
      }
      CB_REQUIRE(ph.x_mode == CB_X_PLAIN || ph.x_mode == CB_X_SILU_MUL, "decode step phase %d: bad x mode", i);
      CB_REQUIRE(a.x != nullptr && a.out != nullptr, "decode step phase %d: x and out are required", i);
      if (ph.x_mode == CB_X_SILU_MUL)
        CB_REQUIRE(a.x_dtype == CB_F32 && a.x_index == nullptr, "decode step phase %d: SwiGLU x is float32", i);
      if (a.epilogue == CB_EPI_ARGMAX)
        CB_REQUIRE(a.scratch_val && a.scratch_idx && a.counter && a.argmax_out,
                   "decode step phase %d: argmax needs scratch for %d blocks", i, grid);
      if (a.epilogue == CB_EPI_RESIDUAL) CB_REQUIRE(a.residual != nullptr, "decode step phase %d: residual missing", i);
      if (a.norm != CB_NORM_NONE) CB_REQUIRE(a.norm_w != nullptr, "decode step phase %d: norm weight missing", i);
      if (a.norm == CB_NORM_RMS_TABLE)
        CB_REQUIRE(a.norm_table && a.x_index, "decode step phase %d: norm table needs x_index", i);
      if (a.x_index != nullptr || a.residual_index != nullptr)
        CB_REQUIRE(a.index_rows > 0, "decode step phase %d: indexed rows need index_rows", i);
      d.g = a;
      d.units = units;
      d.per_cta = (units + grid - 1) / grid;
      d.row_bytes = a.k * (a.w_dtype == CB_BF16 ? 2 : 4);
      // vector loads: 16-byte aligned base; rows and chunks keep the alignment
      d.x_vec = aligned16(a.x) && (a.x_dtype == CB_F32 || a.x_dtype == CB_BF16);
      d.nw_vec = a.norm_w != nullptr && aligned16(a.norm_w) &&
                 (a.norm_w_dtype == CB_F32 || a.norm_w_dtype == CB_BF16);
      if (d.row_bytes > max_row) max_row = d.row_bytes;
      const long long planes = 4 * a.k + 64;
      if (planes > x_bytes) x_bytes = planes;
      ++n_gemv;
    } else if (ph.kind == CB_PHASE_ATTENTION) {
      const cb_decode_attention_args& t = ph.attention;
      CB_REQUIRE(t.head_size == 32 || t.head_size == 64 || t.head_size == 128 || t.head_size == 256,
                 "decode step phase %d: head size %lld unsupported", i, t.head_size);
      CB_REQUIRE(head_size == 0 || head_size == t.head_size, "decode step phase %d: mixed head sizes", i);
      head_size = static_cast<int>(t.head_size);
      CB_REQUIRE(t.kv_heads > 0 && t.heads % t.kv_heads == 0, "decode step phase %d: bad head grouping", i);
      CB_REQUIRE(t.context > 0, "decode step phase %d: empty context", i);
      CB_REQUIRE(t.mask && t.write_mask && t.position && t.scratch && t.counters && t.out,
                 "decode step phase %d: attention buffers missing", i);
      CB_REQUIRE(t.kv_dtype == CB_F32 || t.kv_dtype == CB_BF16,
                 "decode step phase %d: caches must be float32 or bfloat16", i);
      CB_REQUIRE(t.split == 0 || t.split == kAttnSplit, "decode step phase %d: split must be %d", i, kAttnSplit);
      const long long splits = (t.context + kAttnSplit - 1) / kAttnSplit;
      const long long bytes = attn_smem_floats(t.heads / t.kv_heads, t.head_size) * 4;
      if (bytes > x_bytes) x_bytes = bytes;
      d.at = t;
      d.splits = static_cast<int>(splits);
      d.items = splits * t.kv_heads;
      d.merge_in_kernel = 1;
    } else {
      CB_REQUIRE(false, "decode step phase %d: unknown kind %d", i, ph.kind);
    }
  }
  CB_REQUIRE(n_gemv > 0, "decode step: no GEMV phase");
  // The phase before an attention phase (its q/k/v projection): the blocks
  // that run attention items get none of its rows, so they stage their
  // items' cache rows while the other blocks multiply, and the attention
  // starts as soon as q/k/v are complete.  Its cache rows are prefetched
  // into L2 at that phase's start.
  for (int i = 1; i < n_phases; ++i) {
    const PhaseDesc& at = desc[static_cast<size_t>(i)];
    PhaseDesc& before = desc[static_cast<size_t>(i) - 1];
    if (at.kind != CB_PHASE_ATTENTION) continue;
    if (before.kind == CB_PHASE_GEMV && before.paired == 0 && at.items <= grid / 2) {
      before.cta0 = at.items;
      before.per_cta = (before.units + (grid - at.items) - 1) / (grid - at.items);
    }
    const long long row_bytes = at.at.head_size * (at.at.kv_dtype == CB_BF16 ? 2 : 4);
    if (row_bytes % 16 != 0 || !aligned16(at.at.k_cache) || !aligned16(at.at.v_cache)) continue;
    before.pf_k = at.at.k_cache;
    before.pf_v = at.at.v_cache;
    before.pf_context = at.at.context;
    before.pf_row_bytes = row_bytes;
    before.pf_items = at.items < grid ? static_cast<int>(at.items) : grid;
    before.pf_splits = at.splits;
  }
  // With CB_STEP_MERGE_IN_STAGE, an attention output read only by the next
  // phase's x (the O projection) is never materialised: that phase merges
  // the split partials while staging.  Otherwise the attention phase merges.
  for (int i = 0; (flags & CB_STEP_MERGE_IN_STAGE) != 0 && i + 1 < n_phases; ++i) {
    PhaseDesc& at = desc[static_cast<size_t>(i)];
    PhaseDesc& o = desc[static_cast<size_t>(i) + 1];
    if (at.kind != CB_PHASE_ATTENTION || o.kind != CB_PHASE_GEMV) continue;
    const long long out_bytes = at.at.heads * at.at.head_size * 4;
    if (o.x_mode != CB_X_PLAIN || o.g.x != at.at.out || o.g.x_dtype != CB_F32 || o.g.x_index != nullptr ||
        o.g.k != at.at.heads * at.at.head_size)
      continue;
    bool other_reader = false;
    for (int j = 0; j < n_phases && !other_reader; ++j) {
      const PhaseDesc& q = desc[static_cast<size_t>(j)];
      if (q.kind == CB_PHASE_GEMV) {
        other_reader = (j != i + 1 && overlaps(q.g.x, 4 * q.g.k, at.at.out, out_bytes)) ||
                       overlaps(q.g.residual, 4 * q.units, at.at.out, out_bytes);
      } else {
        other_reader = j != i && overlaps(q.at.qkv, 4 * (q.at.v_off + q.at.kv_heads * q.at.head_size), at.at.out,
                                          out_bytes);
      }
    }
    if (other_reader) continue;
    at.merge_in_kernel = 0;
    o.x_mode = kXMerge;
    o.merge_parts = at.at.scratch;
    o.merge_heads = at.at.heads;
    o.merge_hd = static_cast<int>(at.at.head_size);
    o.merge_splits = at.splits;
  }
  x_bytes = round_up(x_bytes, 128);
  // Norm weights staged in shared memory: every GEMV phase with a norm whose
  // weights allow 16-byte bulk copies, in order; phase k's copy is issued at
  // the start of staged phase k-1 (the first at kernel start) into slot k % 2.
  long long norm_bytes = 0;
  int norm_count = 0, prev_norm = -1;
  for (int i = 0; i < n_phases; ++i) {
    PhaseDesc& d = desc[static_cast<size_t>(i)];
    d.norm_ord = -1;
    if (d.kind != CB_PHASE_GEMV || d.g.norm == CB_NORM_NONE || !d.nw_vec) continue;
    const long long bytes = d.g.k * (d.g.norm_w_dtype == CB_BF16 ? 2 : 4);
    if (bytes % 16 != 0 || bytes > kNormStageMax) continue;
    d.norm_ord = norm_count;
    if (prev_norm < 0) {
      desc[0].first_norm_w = d.g.norm_w;
      desc[0].first_norm_bytes = bytes;
    } else {
      PhaseDesc& q = desc[static_cast<size_t>(prev_norm)];
      q.next_norm_w = d.g.norm_w;
      q.next_norm_bytes = bytes;
      q.next_norm_slot = norm_count & 1;
    }
    prev_norm = i;
    ++norm_count;
    if (round_up(bytes, 128) > norm_bytes) norm_bytes = round_up(bytes, 128);
  }
  const long long bar_bytes = (2LL * kStepSlots + 2) * 8;
  const long long slot_bytes = (kStepSmemMax - x_bytes - 2 * norm_bytes - bar_bytes) / kStepSlots / 128 * 128;
  CB_REQUIRE(slot_bytes >= max_row, "decode step: a %lld-byte weight row does not fit the %lld-byte ring slot",
             max_row, slot_bytes);
  for (PhaseDesc& d : desc) {
    if (d.kind != CB_PHASE_GEMV) continue;
    const long long fit = slot_bytes / d.row_bytes;
    d.rows = fit >= 8 ? 8 : fit >= 4 ? 4 : static_cast<int>(fit);
  }
  cudaError_t e = cudaMemcpy(table, desc.data(), desc.size() * sizeof(PhaseDesc), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    set_error("cb_decode_step_prepare: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  config->grid = grid;
  config->n_phases = n_phases;
  config->w_dtype = w_dtype;
  config->head_size = head_size;
  config->slot_bytes = slot_bytes;
  config->x_bytes = x_bytes;
  config->norm_bytes = norm_bytes;
  config->smem = kStepSlots * slot_bytes + x_bytes + 2 * norm_bytes + bar_bytes;
  config->prefetch_bytes = kPrefetchDefault;
  config->lane_inflight = 2;
  config->quiet_window = 0;  // measured: streaming on through the staging window is faster
  config->test_withhold = 0;
  config->timeline = nullptr;
  return CB_OK;
}

int cb_decode_step(const void* table, const cb_decode_step_config* config, unsigned int* counters, int* error_flag,
                   cb_stream_t stream) {
  CB_REQUIRE(table != nullptr && config != nullptr && counters != nullptr && error_flag != nullptr,
             "decode step: table, config, counters and error flag are required");
  CB_REQUIRE(config->n_phases > 0 && config->grid > 0 && config->smem > 0, "decode step: config not prepared");
  StepParams S;
  S.phases = static_cast<const PhaseDesc*>(table);
  S.n_phases = config->n_phases;
  S.grid = config->grid;
  S.slot_bytes = config->slot_bytes;
  S.ring_bytes = kStepSlots * config->slot_bytes;
  S.x_bytes = config->x_bytes;
  S.norm_bytes = config->norm_bytes;
  S.counters = counters;
  S.error_flag = error_flag;
  S.timeline = config->timeline;
  S.prefetch_bytes = config->prefetch_bytes < 0 ? 0 : config->prefetch_bytes;
  CB_REQUIRE(config->lane_inflight == 1 || config->lane_inflight == 2, "decode step: lane_inflight must be 1 or 2");
  S.lane_inflight = config->lane_inflight;
  S.quiet_window = config->quiet_window != 0;
  CB_REQUIRE(config->test_withhold >= 0 && config->test_withhold <= config->grid,
             "decode step: test_withhold must be 0 or 1 + a block index");
  CB_REQUIRE(config->test_withhold == 0 || config->n_phases > 1, "decode step: test_withhold needs two phases");
  S.test_withhold = config->test_withhold;
  return launch_step(S, *config, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

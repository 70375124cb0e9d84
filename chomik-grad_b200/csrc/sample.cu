// Temperature / top-k sampling of logit rows on the device: cb_sample_rows.
//
// The reference samples on the host (examples/generate_tinyllama.py:124-143,
// reached through sample_native_token :146-157 whenever temperature != 0):
// it copies the whole logit row to the host and computes, in float64,
//
//   v = logits[0] / temperature
//   top-k: every v outside the k largest (np.argpartition) becomes -inf
//   p = exp(v - max(v));  p /= p.sum()
//   token = rng.choice(V, p=p)
//
// and NumPy's Generator.choice with p draws ONE double u = rng.random() and
// returns cdf.searchsorted(u, side="right") for cdf = cumsum(p) / cumsum(p)[-1]
// (the first index whose cdf exceeds u).  Here the host draws the same u from
// the caller's generator (the generator advances exactly as in the
// reference) and passes it in; one block per row does the rest from L2:
//
//   1. max over the row (a NaN or a non-finite maximum makes the reference's
//      p NaN, which rng.choice rejects: error flag, token -1);
//   2. top-k: the k-th largest value by an 8-bit radix select over the
//      order-preserving integer image of the floats (4 histogram passes,
//      the first one fused with step 1; one shared atomic per distinct bin
//      of a warp);
//      every value above it is kept, and of the values equal to it the
//      lowest-index ones up to k in total (argpartition leaves that choice
//      unspecified);
//   3. each thread owns a contiguous index range: the per-thread sums of
//      e = exp(v - vmax) over the kept values (float64) are scanned across
//      the block;
//   4. the thread whose range holds the first cumulative sum above
//      u * sum(e) returns that index (cumsum(e) / sum(e) is the reference's
//      cdf, which divides by the sum first).
//
// The float64 sums are added in another order than NumPy's, so the chosen
// index differs from the reference's only when u falls within a few ulps of
// a cdf boundary.
#include <climits>

#include "common.cuh"

namespace cb {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kLoads = 8;  // independent loads a thread issues before using them

// Larger float <=> larger key (for non-NaN values).
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < kSampleWarps; ++w) r = fmaxf(r, red[w]);
  return r;
}

__device__ __forceinline__ double warp_inclusive_scan(double v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__device__ __forceinline__ long long warp_inclusive_scan(long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Exclusive scan over the block in thread order; *total receives the sum.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* red, T* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T incl = warp_inclusive_scan(v);
  const T prev = __shfl_up_sync(0xffffffffu, incl, 1);  // the lanes before this one, as added
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  T before = 0, all = 0;
  for (int w = 0; w < kSampleWarps; ++w) {
    if (w == warp) before = all;
    all += red[w];
  }
  *total = all;
  return lane == 0 ? before : before + prev;
}

// hist[bin] += 1 for the lanes with `valid`, one shared atomic per distinct
// bin of the warp (values cluster in a few bins: the exponent byte first).
// Every lane of the warp must call it.
__device__ __forceinline__ void hist_add(unsigned* hist, unsigned bin, bool valid) {
  const unsigned peers = __match_any_sync(0xffffffffu, valid ? bin : 0x100u);
  if (valid && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
}

// Warp 0 finds the bin holding the k-th largest of the counted values (bins
// counted from the top); sets *prefix's byte at `shift` and *rank to k's rank
// inside that bin.
__device__ __forceinline__ void select_bin(const unsigned* hist, unsigned k, uint32_t prefix, int shift,
                                           uint32_t* sel_prefix, unsigned* sel_rank) {
  const int lane = threadIdx.x;  // warp 0 only; lane l holds bins 255-8l .. 248-8l
  unsigned c[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = hist[255 - (lane * 8 + j)];
    s += c[j];
  }
  unsigned incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const unsigned excl = incl - s;
  if (excl < k && k <= incl) {
    unsigned acc = excl;
    for (int j = 0; j < 8; ++j) {
      if (acc + c[j] >= k) {
        *sel_prefix = prefix | (static_cast<uint32_t>(255 - (lane * 8 + j)) << shift);
        *sel_rank = k - acc;
        break;
      }
      acc += c[j];
    }
  }
}

__global__ void __launch_bounds__(kSampleThreads) sample_rows_kernel(const cb_sample_args a) {
  __shared__ float red_f[kSampleWarps];
  __shared__ double red_d[kSampleWarps];
  __shared__ long long red_l[kSampleWarps];
  __shared__ unsigned hist[256];
  __shared__ uint32_t sel_prefix;
  __shared__ unsigned sel_rank;
  __shared__ unsigned long long pick;
  __shared__ unsigned long long last_kept;

  const int tid = threadIdx.x;
  const long long row = blockIdx.x;
  const long long base = row * a.ld;
  const long long width = a.width;
  const void* x = a.logits;
  const int dt = a.logits_dtype;
  const bool topk = a.top_k > 0 && a.top_k < width;
  auto value = [&](long long i) -> float { return load_as_f32(x, base + i, dt); };

  // 1. maximum (and the reference's NaN rejection); with top-k, the
  // histogram of the keys' top byte as well
  for (int b = tid; b < 256; b += kSampleThreads) hist[b] = 0;
  __syncthreads();
  float m = -INFINITY;
  int bad = 0;
  for (long long i0 = 0; i0 < width; i0 += kLoads * kSampleThreads) {  // block-uniform trip count
    float v[kLoads];
#pragma unroll
    for (int j = 0; j < kLoads; ++j) {
      const long long i = i0 + j * kSampleThreads + tid;
      v[j] = i < width ? load_as_f32(x, base + i, dt) : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < kLoads; ++j) {
      bad |= v[j] != v[j];
      m = fmaxf(m, v[j]);
      if (topk) hist_add(hist, order_key(v[j]) >> 24, i0 + j * kSampleThreads + tid < width);
    }
  }
  m = block_max(m, red_f);
  bad = __syncthreads_or(bad);
  const double temperature = a.temperature;
  const double vmax = static_cast<double>(m) / temperature;
  if (bad || !isfinite(vmax)) {
    if (tid == 0) {
      a.out[row] = -1;
      if (a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_NAN);
    }
    return;
  }

  // 2. top-k threshold: key of the k-th largest value (radix select, one
  // byte per pass from the top), and how many values equal to it are kept
  uint32_t thr = 0;
  long long need_eq = 0;
  if (topk) {
    uint32_t prefix = 0, mask = 0;
    unsigned k = static_cast<unsigned>(a.top_k);
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (shift < 24) {
        for (int b = tid; b < 256; b += kSampleThreads) hist[b] = 0;
        __syncthreads();
        for (long long i0 = 0; i0 < width; i0 += kLoads * kSampleThreads) {
          float v[kLoads];
#pragma unroll
          for (int j = 0; j < kLoads; ++j) {
            const long long i = i0 + j * kSampleThreads + tid;
            v[j] = i < width ? value(i) : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < kLoads; ++j) {
            const uint32_t key = order_key(v[j]);
            hist_add(hist, (key >> shift) & 255u,
                     i0 + j * kSampleThreads + tid < width && (key & mask) == prefix);
          }
        }
      }
      __syncthreads();
      if (tid < 32) select_bin(hist, k, prefix, shift, &sel_prefix, &sel_rank);
      __syncthreads();
      prefix = sel_prefix;
      k = sel_rank;
      mask |= 255u << shift;
    }
    thr = prefix;
    need_eq = k;
  }

  // contiguous index range of this thread
  const long long seg = (width + kSampleThreads - 1) / kSampleThreads;
  const long long s0 = tid * seg < width ? tid * seg : width;
  const long long s1 = s0 + seg < width ? s0 + seg : width;

  long long eq_before = 0;
  if (topk) {
    long long count = 0;
    for (long long i0 = s0; i0 < s1; i0 += kLoads) {
      float v[kLoads];
#pragma unroll
      for (int j = 0; j < kLoads; ++j) v[j] = i0 + j < s1 ? value(i0 + j) : 0.0f;
#pragma unroll
      for (int j = 0; j < kLoads; ++j) count += i0 + j < s1 && order_key(v[j]) == thr;
    }
    long long all;
    eq_before = block_exclusive_scan(count, red_l, &all);
  }
  // whether value i is kept; eq counts the threshold-equal values seen so far
  auto kept = [&](float v, long long& eq) -> bool {
    if (!topk) return true;
    const uint32_t key = order_key(v);
    if (key > thr) return true;
    if (key != thr) return false;
    return eq++ < need_eq;
  };

  // 3. e = exp(v - vmax) of the kept values, summed per range and scanned
  // in index order: the cdf is cumsum(e) / sum(e) (the reference divides
  // by the sum first; the same ratios up to rounding)
  double part = 0.0;
  long long eq = eq_before;
  for (long long i0 = s0; i0 < s1; i0 += kLoads) {
    float v[kLoads];
#pragma unroll
    for (int j = 0; j < kLoads; ++j) v[j] = i0 + j < s1 ? value(i0 + j) : 0.0f;
#pragma unroll
    for (int j = 0; j < kLoads; ++j)
      if (i0 + j < s1 && kept(v[j], eq)) part += exp(static_cast<double>(v[j]) / temperature - vmax);
  }
  double total;
  const double before = block_exclusive_scan(part, red_d, &total);
  if (tid == 0) {
    pick = ULLONG_MAX;
    last_kept = 0;  // the maximum is always kept with e = 1, so some range raises it
  }
  __syncthreads();
  const double u = a.uniforms[row];
  // 4. The range whose running sum crosses u * total holds the token.  A
  // range that starts past it (its scanned prefix rounded above u) offers
  // its first positive-probability index; the smallest offer wins.  Ranges
  // that end well below u cannot hold it and skip the walk.
  const bool starts_before = before / total <= u;
  if (!starts_before || before + part >= u * total * (1.0 - 1e-9)) {
    double c = before;
    long long mine_last = -1;
    eq = eq_before;
    bool found = false;
    for (long long i0 = s0; i0 < s1 && !found; i0 += kLoads) {
      float v[kLoads];
#pragma unroll
      for (int j = 0; j < kLoads; ++j) v[j] = i0 + j < s1 ? value(i0 + j) : 0.0f;
      for (int j = 0; j < kLoads && i0 + j < s1; ++j) {
        if (!kept(v[j], eq)) continue;
        const double e = exp(static_cast<double>(v[j]) / temperature - vmax);
        if (e <= 0.0) continue;
        mine_last = i0 + j;
        c += e;
        if (!starts_before || c / total > u) {
          atomicMin(&pick, static_cast<unsigned long long>(i0 + j));
          found = true;
          break;
        }
      }
    }
    if (mine_last >= 0) atomicMax(&last_kept, static_cast<unsigned long long>(mine_last));
  }
  __syncthreads();
  if (tid == 0) a.out[row] = static_cast<long long>(pick != ULLONG_MAX ? pick : last_kept);
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_sample_rows(const cb_sample_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->width > 0, "sample: empty logit rows");
  CB_REQUIRE(a->width < (1LL << 31), "sample: rows wider than 2^31 - 1");
  CB_REQUIRE(a->logits_dtype == CB_F32 || a->logits_dtype == CB_BF16 || a->logits_dtype == CB_F16,
             "sample: logits must be float32, bfloat16 or float16");
  CB_REQUIRE(a->temperature > 0.0, "sample: temperature must be positive (temperature 0 is argmax)");
  CB_REQUIRE(a->ld >= a->width, "sample: row stride below the row width");
  if (a->rows == 0) return CB_OK;
  CB_REQUIRE(a->rows < (1LL << 31), "sample: too many rows");
  CB_REQUIRE(a->logits != nullptr && a->uniforms != nullptr && a->out != nullptr, "sample: null pointer");
  sample_rows_kernel<<<static_cast<unsigned>(a->rows), kSampleThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      *a);
  return check_launch("cb_sample_rows");
}

}  // extern "C"

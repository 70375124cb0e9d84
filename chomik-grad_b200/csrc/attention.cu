// Attention kernels.
//
//  * cb_sdpa: generic grouped-query attention (prefill, verify blocks, any
//    graph) -- one warp per query row, online softmax, float32.
//  * cb_decode_attention: the single-token decode step.  One CTA per
//    (context split, KV head) ropes the new q/k rows, stages its split's K/V
//    rows in shared memory (applying the write-mask blend to the rows it owns
//    on the way), computes all (query head, position) scores in one pass,
//    and the last CTA of each KV group merges the splits.
//
// Score arithmetic follows the reference graph: s = q.k, x = s / divisor +
// mask, softmax over the whole context, then p @ v.
#include "common.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxLaneDims = 8;  // head_size <= 256

__device__ __forceinline__ long long idx4(const long long* st, long long a, long long b, long long c,
                                          long long d) {
  return a * st[0] + b * st[1] + c * st[2] + d * st[3];
}

__global__ void __launch_bounds__(kThreads) sdpa_kernel(const cb_sdpa_args a) {
  extern __shared__ float qs[];  // (warps, head_size)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const long long rows = a.batch * a.heads * a.tq;
  const long long D = a.head_size;
  const int lane_dims = static_cast<int>((D + 31) / 32);
  const long long group = a.heads / a.kv_heads;
  float* q = qs + warp * D;
  for (long long row = blockIdx.x * (long long)warps + warp; row < rows;
       row += (long long)gridDim.x * warps) {
    const long long t = row % a.tq;
    const long long h = (row / a.tq) % a.heads;
    const long long b = row / (a.tq * a.heads);
    const long long kh = h / group;
    for (long long d = lane; d < D; d += 32) q[d] = load_as_f32(a.q, a.q_offset + idx4(a.q_strides, b, h, t, d), a.q_dtype);
    __syncwarp();
    float m = -INFINITY, l = 0.0f;
    float acc[kMaxLaneDims];
#pragma unroll
    for (int i = 0; i < kMaxLaneDims; ++i) acc[i] = 0.0f;
    for (long long base = 0; base < a.tk; base += 32) {
      const long long j = base + lane;
      float x = -INFINITY;
      if (j < a.tk) {
        float s = 0.0f;
        const long long kb = a.k_offset + idx4(a.k_strides, b, kh, j, 0);
        for (long long d = 0; d < D; ++d) s = fmaf(q[d], load_as_f32(a.k, kb + d * a.k_strides[3], a.k_dtype), s);
        x = __fdiv_rn(s, a.divisor);
        if (a.mask != nullptr)
          x = __fadd_rn(x, load_as_f32(a.mask, a.mask_offset + idx4(a.mask_strides, b, h, t, j), a.mask_dtype));
      }
      const float m_new = fmaxf(m, warp_max(x));
      const float p = j < a.tk ? expf(x - m_new) : 0.0f;
      const float alpha = expf(m - m_new);
      l = l * alpha + warp_sum(p);
#pragma unroll
      for (int i = 0; i < kMaxLaneDims; ++i) acc[i] *= alpha;
      const int count = static_cast<int>(a.tk - base < 32 ? a.tk - base : 32);
      for (int jj = 0; jj < count; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        const long long vb = a.v_offset + idx4(a.v_strides, b, kh, base + jj, 0);
#pragma unroll
        for (int i = 0; i < kMaxLaneDims; ++i) {
          const long long d = lane + 32 * i;
          if (i < lane_dims && d < D) acc[i] = fmaf(pj, load_as_f32(a.v, vb + d * a.v_strides[3], a.v_dtype), acc[i]);
        }
      }
      m = m_new;
    }
    const long long ob = row * D;
#pragma unroll
    for (int i = 0; i < kMaxLaneDims; ++i) {
      const long long d = lane + 32 * i;
      if (i < lane_dims && d < D) a.out[ob + d] = __fdiv_rn(acc[i], l);
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Decode.  grid (splits, kv_heads), 256 threads, SPLIT (= 32) positions per
// CTA.  Dynamic shared memory:
//   q_rot[group][HD] | k_new[HD] | v_new[HD] | ks[SPLIT][HD+1] | vs[SPLIT][HD]
//   | probs[group][SPLIT] | stats[group][2]
// ks rows are padded by one float so lane j reading row j is conflict-free.
constexpr int kSplit = 32;

template <int HD>
__global__ void __launch_bounds__(kThreads) decode_attention_kernel(const cb_decode_attention_args a) {
  extern __shared__ float smem[];
  __shared__ int s_last;
  const int g = blockIdx.y;
  const int split = blockIdx.x;
  const int splits = gridDim.x;
  const int group = static_cast<int>(a.heads / a.kv_heads);
  constexpr int half = HD / 2;
  constexpr int KS = HD + 1;
  float* q_rot = smem;
  float* k_new = q_rot + group * HD;
  float* v_new = k_new + HD;
  float* ks = v_new + HD;
  float* vs = ks + kSplit * KS;
  float* probs = vs + kSplit * HD;
  float* stats = probs + group * kSplit;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int warps = kThreads / 32;

  prefetch_share(a.prefetch_ptr, a.prefetch_bytes, static_cast<long long>(g) * splits + split,
                 static_cast<long long>(splits) * gridDim.y, tid, kThreads);
  pdl_wait();
  pdl_launch_dependents();

  long long pos = load_index(a.position, 0, a.position_dtype);
  if (pos < 0 || pos >= a.n_positions) {
    if (tid == 0 && split == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, 2);
    pos = pos < 0 ? 0 : a.n_positions - 1;
  }
  const float* cs = a.cos_table + pos * half;
  const float* sn = a.sin_table + pos * half;
  for (int i = tid; i < group * half; i += kThreads) {
    const int h = i / half, j = i % half;
    const float* src = a.qkv + a.q_off + (static_cast<long long>(g) * group + h) * HD;
    const float lo = src[j], hi = src[j + half], c = cs[j], s = sn[j];
    q_rot[h * HD + j] = fmaf(-hi, s, __fmul_rn(lo, c));
    q_rot[h * HD + j + half] = fmaf(hi, c, __fmul_rn(lo, s));
  }
  for (int j = tid; j < half; j += kThreads) {
    const float* src = a.qkv + a.k_off + static_cast<long long>(g) * HD;
    const float lo = src[j], hi = src[j + half], c = cs[j], s = sn[j];
    k_new[j] = fmaf(-hi, s, __fmul_rn(lo, c));
    k_new[j + half] = fmaf(hi, c, __fmul_rn(lo, s));
  }
  for (int d = tid; d < HD; d += kThreads) v_new[d] = a.qkv[a.v_off + static_cast<long long>(g) * HD + d];
  __syncthreads();

  // ---- stage this split's K/V rows; rows with wm != 0 get the blend
  //      cache*(1-wm) + new*wm (float32, written back to the cache) ----
  const long long lo_pos = static_cast<long long>(split) * kSplit;
  const int n = static_cast<int>(a.context - lo_pos < kSplit ? a.context - lo_pos : kSplit);
  float* kc = a.k_cache + (static_cast<long long>(g) * a.context + lo_pos) * HD;
  float* vc = a.v_cache + (static_cast<long long>(g) * a.context + lo_pos) * HD;
  for (int e = tid; e < n * (HD / 4); e += kThreads) {
    const int r = e / (HD / 4), d4 = (e % (HD / 4)) * 4;
    float4 kv = reinterpret_cast<const float4*>(kc)[e];
    float4 vv = reinterpret_cast<const float4*>(vc)[e];
    const float wm = load_as_f32(a.write_mask, lo_pos + r, a.write_mask_dtype);
    if (wm != 0.0f) {
      const float keep = round_to(__fsub_rn(1.0f, wm), a.one_minus_dtype);
      float* kf = &kv.x;
      float* vf = &vv.x;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kf[i] = __fadd_rn(__fmul_rn(kf[i], keep), __fmul_rn(k_new[d4 + i], wm));
        vf[i] = __fadd_rn(__fmul_rn(vf[i], keep), __fmul_rn(v_new[d4 + i], wm));
      }
      reinterpret_cast<float4*>(kc)[e] = kv;
      reinterpret_cast<float4*>(vc)[e] = vv;
    }
    float* kd = ks + r * KS + d4;
    kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
    *reinterpret_cast<float4*>(vs + r * HD + d4) = vv;
  }
  __syncthreads();

  // ---- scores: warp = query head (looping), lane = position ----
  for (int h = warp; h < group; h += warps) {
    float x = -INFINITY;
    if (lane < n) {
      const float* q = q_rot + h * HD;
      const float* k = ks + lane * KS;
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int d = 0; d < HD; d += 2) {
        s0 = fmaf(q[d], k[d], s0);
        s1 = fmaf(q[d + 1], k[d + 1], s1);
      }
      x = __fadd_rn(__fdiv_rn(s0 + s1, a.divisor), load_as_f32(a.mask, lo_pos + lane, a.mask_dtype));
    }
    const float m = warp_max(x);
    const float p = lane < n ? expf(x - m) : 0.0f;
    const float l = warp_sum(p);
    probs[h * kSplit + lane] = p;
    if (lane == 0) {
      stats[2 * h] = m;
      stats[2 * h + 1] = l;
    }
  }
  __syncthreads();

  // ---- p @ v for every (head, dim) of the group; partials to scratch ----
  for (int i = tid; i < group * HD; i += kThreads) {
    const int h = i / HD, d = i % HD;
    const float* p = probs + h * kSplit;
    float acc0 = 0.0f, acc1 = 0.0f;
    int j = 0;
    for (; j + 1 < n; j += 2) {
      acc0 = fmaf(p[j], vs[j * HD + d], acc0);
      acc1 = fmaf(p[j + 1], vs[(j + 1) * HD + d], acc1);
    }
    if (j < n) acc0 = fmaf(p[j], vs[j * HD + d], acc0);
    float* part = a.scratch + (static_cast<long long>(split) * a.heads + g * group + h) * (HD + 2);
    part[2 + d] = acc0 + acc1;
    if (d == 0) {
      part[0] = stats[2 * h];
      part[1] = stats[2 * h + 1];
    }
  }

  // ---- merge the splits of this KV group in split order (deterministic) ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned ticket = atomicAdd(a.counters + g, 1u);
    s_last = ticket == static_cast<unsigned>(splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < group * HD; i += kThreads) {
    const int h = i / HD, d = i % HD;
    const long long head = static_cast<long long>(g) * group + h;
    const float* base = a.scratch + head * (HD + 2);
    const long long stride = a.heads * (HD + 2);
    float mmax = -INFINITY;
    for (int sp = 0; sp < splits; ++sp) mmax = fmaxf(mmax, __ldcg(base + sp * stride));
    float lsum = 0.0f, acc = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
      const float* part = base + sp * stride;
      const float scale = expf(__ldcg(part) - mmax);
      lsum = fmaf(__ldcg(part + 1), scale, lsum);
      acc = fmaf(__ldcg(part + 2 + d), scale, acc);
    }
    a.out[head * HD + d] = __fdiv_rn(acc, lsum);
  }
  if (tid == 0) a.counters[g] = 0u;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_sdpa(const cb_sdpa_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->head_size > 0 && a->head_size <= 32 * kMaxLaneDims, "sdpa: head size %lld unsupported",
             a->head_size);
  CB_REQUIRE(a->kv_heads > 0 && a->heads % a->kv_heads == 0, "sdpa: heads must be a multiple of KV heads");
  const long long rows = a->batch * a->heads * a->tq;
  if (rows == 0) return CB_OK;
  const int warps = kThreads / 32;
  long long blocks = (rows + warps - 1) / warps;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  const size_t smem = static_cast<size_t>(warps) * a->head_size * sizeof(float);
  sdpa_kernel<<<static_cast<unsigned>(blocks), kThreads, smem, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_launch("cb_sdpa");
}

long long cb_decode_attention_scratch(const cb_decode_attention_args* a) {
  const long long splits = (a->context + kSplit - 1) / kSplit;
  return splits * a->heads * (a->head_size + 2);
}

int cb_decode_attention(const cb_decode_attention_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->head_size == 32 || a->head_size == 64 || a->head_size == 128 || a->head_size == 256,
             "decode attention: head size %lld unsupported (32/64/128/256)", a->head_size);
  CB_REQUIRE(a->kv_heads > 0 && a->heads % a->kv_heads == 0, "decode attention: bad head grouping");
  CB_REQUIRE(a->context > 0, "decode attention: empty context");
  CB_REQUIRE(a->mask != nullptr && a->write_mask != nullptr && a->position != nullptr,
             "decode attention: mask, write mask and position are required");
  CB_REQUIRE(a->split == 0 || a->split == kSplit, "decode attention: split must be %d", kSplit);
  const long long splits = (a->context + kSplit - 1) / kSplit;
  CB_REQUIRE(splits < 65536 && a->kv_heads < 65536, "decode attention: grid too large");
  const long long group = a->heads / a->kv_heads;
  const long long hd = a->head_size;
  const size_t smem = static_cast<size_t>((group + 2) * hd + kSplit * (hd + 1) + kSplit * hd +
                                          group * kSplit + 2 * group) * sizeof(float);
  CB_REQUIRE(smem <= 200 * 1024, "decode attention: too many query heads per KV head");
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(a->kv_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define CB_DECODE_CASE(HD)                                                                          \
  case HD:                                                                                          \
    cudaFuncSetAttribute(decode_attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                         static_cast<int>(smem));                                                   \
    e = launch(decode_attention_kernel<HD>, grid, dim3(kThreads), smem, s, a->pdl != 0, *a);         \
    break;
  switch (a->head_size) {
    CB_DECODE_CASE(32)
    CB_DECODE_CASE(64)
    CB_DECODE_CASE(128)
    CB_DECODE_CASE(256)
  }
#undef CB_DECODE_CASE
  if (e != cudaSuccess) {
    set_error("cb_decode_attention: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_decode_attention");
}

}  // extern "C"

// Attention kernels.
//
//  * cb_sdpa: generic grouped-query attention (prefill, verify blocks, any
//    graph) -- one warp per query row, online softmax, float32.
//  * cb_decode_attention: the single-token decode step.  One CTA per
//    (context split, KV head) ropes the new q/k rows, applies the write-mask
//    blend to the cache rows it owns, attends its split for the group's query
//    heads, and the last CTA of each KV group merges the splits.
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
// Decode: grid (splits, kv_heads), 256 threads.  Dynamic smem layout:
//   q_rot[group][hd] | k_new[hd] | v_new[hd]
template <int LANE_DIMS>
__global__ void __launch_bounds__(kThreads) decode_attention_kernel(const cb_decode_attention_args a,
                                                                   int split_len) {
  constexpr int HD = LANE_DIMS * 32;
  extern __shared__ float smem[];
  __shared__ int s_last;
  const int g = blockIdx.y;
  const int split = blockIdx.x;
  const int splits = gridDim.x;
  const int group = static_cast<int>(a.heads / a.kv_heads);
  const int half = HD / 2;
  float* q_rot = smem;
  float* k_new = q_rot + group * HD;
  float* v_new = k_new + HD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, warps = blockDim.x >> 5;

  prefetch_share(a.prefetch_ptr, a.prefetch_bytes, static_cast<long long>(g) * splits + split,
                 static_cast<long long>(splits) * gridDim.y, tid, blockDim.x);
  pdl_wait();
  pdl_launch_dependents();

  long long pos = load_index(a.position, 0, a.position_dtype);
  if (pos < 0 || pos >= a.n_positions) {
    if (tid == 0 && split == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, 2);
    pos = pos < 0 ? 0 : a.n_positions - 1;
  }
  const float* cs = a.cos_table + pos * half;
  const float* sn = a.sin_table + pos * half;
  for (int i = tid; i < group * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    const float* src = a.qkv + a.q_off + (static_cast<long long>(g) * group + h) * HD;
    const float lo = src[j], hi = src[j + half], c = cs[j], s = sn[j];
    q_rot[h * HD + j] = fmaf(-hi, s, __fmul_rn(lo, c));
    q_rot[h * HD + j + half] = fmaf(hi, c, __fmul_rn(lo, s));
  }
  for (int j = tid; j < half; j += blockDim.x) {
    const float* src = a.qkv + a.k_off + static_cast<long long>(g) * HD;
    const float lo = src[j], hi = src[j + half], c = cs[j], s = sn[j];
    k_new[j] = fmaf(-hi, s, __fmul_rn(lo, c));
    k_new[j + half] = fmaf(hi, c, __fmul_rn(lo, s));
  }
  for (int d = tid; d < HD; d += blockDim.x) v_new[d] = a.qkv[a.v_off + static_cast<long long>(g) * HD + d];
  __syncthreads();

  const long long lo_pos = static_cast<long long>(split) * split_len;
  const long long hi_pos = lo_pos + split_len < a.context ? lo_pos + split_len : a.context;
  float* kc = a.k_cache + static_cast<long long>(g) * a.context * HD;
  float* vc = a.v_cache + static_cast<long long>(g) * a.context * HD;
  // Write-mask blend: cache*(1-wm) + new*wm on the rows this CTA owns.
  for (long long r = lo_pos; r < hi_pos; ++r) {
    const float wm = load_as_f32(a.write_mask, r, a.write_mask_dtype);
    if (wm == 0.0f) continue;
    const float keep = round_to(__fsub_rn(1.0f, wm), a.one_minus_dtype);
    for (int d = tid; d < HD; d += blockDim.x) {
      kc[r * HD + d] = __fadd_rn(__fmul_rn(kc[r * HD + d], keep), __fmul_rn(k_new[d], wm));
      vc[r * HD + d] = __fadd_rn(__fmul_rn(vc[r * HD + d], keep), __fmul_rn(v_new[d], wm));
    }
  }
  __syncthreads();

  for (int h = warp; h < group; h += warps) {
    const float* q = q_rot + h * HD;
    float m = -INFINITY, l = 0.0f;
    float acc[LANE_DIMS];
#pragma unroll
    for (int i = 0; i < LANE_DIMS; ++i) acc[i] = 0.0f;
    for (long long base = lo_pos; base < hi_pos; base += 32) {
      const long long j = base + lane;
      float x = -INFINITY;
      if (j < hi_pos) {
        const float4* krow = reinterpret_cast<const float4*>(kc + j * HD);
        float s = 0.0f;
#pragma unroll
        for (int d4 = 0; d4 < HD / 4; ++d4) {
          const float4 kv = krow[d4];
          s = fmaf(q[4 * d4 + 0], kv.x, s);
          s = fmaf(q[4 * d4 + 1], kv.y, s);
          s = fmaf(q[4 * d4 + 2], kv.z, s);
          s = fmaf(q[4 * d4 + 3], kv.w, s);
        }
        x = __fadd_rn(__fdiv_rn(s, a.divisor), load_as_f32(a.mask, j, a.mask_dtype));
      }
      const float m_new = fmaxf(m, warp_max(x));
      const float p = j < hi_pos ? expf(x - m_new) : 0.0f;
      const float alpha = expf(m - m_new);
      l = l * alpha + warp_sum(p);
#pragma unroll
      for (int i = 0; i < LANE_DIMS; ++i) acc[i] *= alpha;
      const int count = static_cast<int>(hi_pos - base < 32 ? hi_pos - base : 32);
      for (int jj = 0; jj < count; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        const float* vrow = vc + (base + jj) * HD;
#pragma unroll
        for (int i = 0; i < LANE_DIMS; ++i) acc[i] = fmaf(pj, vrow[lane + 32 * i], acc[i]);
      }
      m = m_new;
    }
    float* part = a.scratch + (static_cast<long long>(split) * a.heads + g * group + h) * (HD + 2);
    if (lane == 0) {
      part[0] = m;
      part[1] = l;
    }
#pragma unroll
    for (int i = 0; i < LANE_DIMS; ++i) part[2 + lane + 32 * i] = acc[i];
  }

  // Merge the splits of this KV group in split order (deterministic).
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned ticket = atomicAdd(a.counters + g, 1u);
    s_last = ticket == static_cast<unsigned>(splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int h = warp; h < group; h += warps) {
    const long long head = static_cast<long long>(g) * group + h;
    float mmax = -INFINITY;
    for (int sp = 0; sp < splits; ++sp)
      mmax = fmaxf(mmax, __ldcg(a.scratch + (static_cast<long long>(sp) * a.heads + head) * (HD + 2)));
    float lsum = 0.0f;
    float acc[LANE_DIMS];
#pragma unroll
    for (int i = 0; i < LANE_DIMS; ++i) acc[i] = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
      const float* part = a.scratch + (static_cast<long long>(sp) * a.heads + head) * (HD + 2);
      const float scale = expf(__ldcg(part) - mmax);
      lsum = fmaf(__ldcg(part + 1), scale, lsum);
#pragma unroll
      for (int i = 0; i < LANE_DIMS; ++i) acc[i] = fmaf(__ldcg(part + 2 + lane + 32 * i), scale, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < LANE_DIMS; ++i) a.out[head * HD + lane + 32 * i] = __fdiv_rn(acc[i], lsum);
  }
  if (tid == 0) a.counters[g] = 0u;
}

inline int decode_split(const cb_decode_attention_args& a) {
  return a.split > 0 ? a.split : 32;
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
  const long long split = decode_split(*a);
  const long long splits = (a->context + split - 1) / split;
  return splits * a->heads * (a->head_size + 2);
}

int cb_decode_attention(const cb_decode_attention_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->head_size % 32 == 0 && a->head_size >= 32 && a->head_size <= 256,
             "decode attention: head size %lld must be a multiple of 32 up to 256", a->head_size);
  CB_REQUIRE(a->kv_heads > 0 && a->heads % a->kv_heads == 0, "decode attention: bad head grouping");
  CB_REQUIRE(a->context > 0, "decode attention: empty context");
  CB_REQUIRE(a->mask != nullptr && a->write_mask != nullptr && a->position != nullptr,
             "decode attention: mask, write mask and position are required");
  const int split = decode_split(*a);
  const long long splits = (a->context + split - 1) / split;
  CB_REQUIRE(splits < 65536 && a->kv_heads < 65536, "decode attention: grid too large");
  const int group = static_cast<int>(a->heads / a->kv_heads);
  const size_t smem = static_cast<size_t>(group + 2) * a->head_size * sizeof(float);
  CB_REQUIRE(smem <= 200 * 1024, "decode attention: too many query heads per KV head");
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(a->kv_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define CB_DECODE_CASE(LD)                                                                          \
  case LD:                                                                                          \
    if (smem > 48 * 1024)                                                                           \
      cudaFuncSetAttribute(decode_attention_kernel<LD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           static_cast<int>(smem));                                                 \
    e = launch(decode_attention_kernel<LD>, grid, dim3(kThreads), smem, s, a->pdl != 0, *a, split);  \
    break;
  switch (a->head_size / 32) {
    CB_DECODE_CASE(1)
    CB_DECODE_CASE(2)
    CB_DECODE_CASE(4)
    CB_DECODE_CASE(8)
    default:
      CB_REQUIRE(false, "decode attention: head size %lld unsupported", a->head_size);
  }
#undef CB_DECODE_CASE
  if (e != cudaSuccess) {
    set_error("cb_decode_attention: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_decode_attention");
}

}  // extern "C"

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
#include "attn_core.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxLaneDims = 8;  // head_size <= 256

__device__ __forceinline__ long long idx4(const long long* st, long long a, long long b, long long c,
                                          long long d) {
  return a * st[0] + b * st[1] + c * st[2] + d * st[3];
}

// Offset of out[b, h, t, 0]: contiguous (B, H, T, D) unless out_strides are given.
__device__ __forceinline__ long long out_index(const cb_sdpa_args& a, long long b, long long h, long long t) {
  if (a.out_strides[0] == 0 && a.out_strides[1] == 0 && a.out_strides[2] == 0)
    return ((b * a.heads + h) * a.tq + t) * a.head_size;
  return b * a.out_strides[0] + h * a.out_strides[1] + t * a.out_strides[2];
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
    const long long ob = out_index(a, b, h, t);
#pragma unroll
    for (int i = 0; i < kMaxLaneDims; ++i) {
      const long long d = lane + 32 * i;
      if (i < lane_dims && d < D) a.out[ob + d] = __fdiv_rn(acc[i], l);
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Single-query attention (tq == 1) over float32 K/V rows, split over keys:
// the batched decode step's attention (every sequence's one new query
// against its own cache).  Pass 1, grid (splits, kv_heads, batch): a block
// stages the split's K/V rows with 16-byte loads (coalesced: rows are
// contiguous), loads the group's q rows and mask values, and one warp per
// query head computes the split's scores (lane = key), its max, sum and
// unnormalised p @ v.  Pass 2 merges the splits of each (batch, head) in
// split order, so results are deterministic.
constexpr int kQSplit = 32;  // keys per split = lanes

__host__ __device__ inline long long qsplit_smem_floats(long long group, long long hd) {
  return kQSplit * (hd + 4) + kQSplit * hd + group * hd + group * kQSplit;
}

template <int HD>
__global__ void __launch_bounds__(kThreads) sdpa_query_kernel(const cb_sdpa_args a, float* parts, int splits) {
  extern __shared__ float sm[];
  constexpr int KS = HD + 4;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = static_cast<int>(a.heads / a.kv_heads);
  float* ks = sm;                          // [kQSplit][KS]
  float* vs = ks + kQSplit * KS;           // [kQSplit][HD]
  float* qs = vs + kQSplit * HD;           // [group][HD]
  float* ms = qs + group * HD;             // [group][kQSplit]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long lo = static_cast<long long>(split) * kQSplit;
  const int n = static_cast<int>(a.tk - lo < kQSplit ? a.tk - lo : kQSplit);
  const float* kb = static_cast<const float*>(a.k) + a.k_offset + b * a.k_strides[0] + kvh * a.k_strides[1];
  const float* vb = static_cast<const float*>(a.v) + a.v_offset + b * a.v_strides[0] + kvh * a.v_strides[1];
  for (int e = tid; e < n * (HD / 4); e += kThreads) {
    const int r = e / (HD / 4), d4 = (e % (HD / 4)) * 4;
    const float4 kv = __ldg(reinterpret_cast<const float4*>(kb + (lo + r) * a.k_strides[2] + d4));
    const float4 vv = __ldg(reinterpret_cast<const float4*>(vb + (lo + r) * a.v_strides[2] + d4));
    *reinterpret_cast<float4*>(ks + r * KS + d4) = kv;
    *reinterpret_cast<float4*>(vs + r * HD + d4) = vv;
  }
  for (int e = tid; e < group * HD; e += kThreads) {
    const int h = kvh * group + e / HD, d = e % HD;
    qs[e] = load_as_f32(a.q, a.q_offset + idx4(a.q_strides, b, h, 0, d), a.q_dtype);
  }
  for (int e = tid; e < group * kQSplit; e += kThreads) {
    const int h = kvh * group + e / kQSplit, j = e % kQSplit;
    ms[e] = (a.mask != nullptr && j < n)
                ? load_as_f32(a.mask, a.mask_offset + idx4(a.mask_strides, b, h, 0, lo + j), a.mask_dtype)
                : 0.0f;
  }
  __syncthreads();
  for (int hl = warp; hl < group; hl += kThreads / 32) {
    const int h = kvh * group + hl;
    float x = -INFINITY;
    if (lane < n) {
      const float4* q = reinterpret_cast<const float4*>(qs + hl * HD);
      const float4* k = reinterpret_cast<const float4*>(ks + lane * KS);
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll
      for (int d = 0; d < HD / 4; ++d) {
        const float4 qa = q[d], ka = k[d];
        s0 = fmaf(qa.x, ka.x, s0);
        s1 = fmaf(qa.y, ka.y, s1);
        s2 = fmaf(qa.z, ka.z, s2);
        s3 = fmaf(qa.w, ka.w, s3);
      }
      x = __fadd_rn(__fdiv_rn((s0 + s1) + (s2 + s3), a.divisor), ms[hl * kQSplit + lane]);
    }
    const float m = warp_max(x);
    const float p = lane < n ? expf(x - m) : 0.0f;
    const float l = warp_sum(p);
    float* part = parts + ((static_cast<long long>(b) * a.heads + h) * splits + split) * (HD + 2);
#pragma unroll
    for (int d0 = 0; d0 < HD; d0 += 64) {
      const int d = d0 + 2 * lane;
      const bool mine = d < HD;
      float2 acc = make_float2(0.0f, 0.0f);
      for (int j = 0; j < n; ++j) {  // every lane shuffles; rows j < n only are read
        const float pj = __shfl_sync(0xffffffffu, p, j);
        if (mine) {
          const float2 v = *reinterpret_cast<const float2*>(vs + j * HD + d);
          acc.x = fmaf(pj, v.x, acc.x);
          acc.y = fmaf(pj, v.y, acc.y);
        }
      }
      if (mine) *reinterpret_cast<float2*>(part + 2 + d) = acc;
    }
    if (lane == 0) {
      part[0] = m;
      part[1] = l;
    }
  }
}

// Pass 2: one warp per (batch, head).  Lanes take the splits' maxima and
// sums (32 splits at a time), the scales move to the dimension lanes by
// shuffle; every sum runs in a fixed order (deterministic).
constexpr int kMergeWarps = 4;

__global__ void __launch_bounds__(kMergeWarps * 32) sdpa_query_merge_kernel(const float* parts, long long rows,
                                                                             int splits, int hd,
                                                                             const cb_sdpa_args a) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * kMergeWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* base = parts + row * splits * (hd + 2);
  float m = -INFINITY;
  for (int s = lane; s < splits; s += 32) m = fmaxf(m, base[s * (hd + 2)]);
  m = warp_max(m);
  float l = 0.0f;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  for (int s0 = 0; s0 < splits; s0 += 32) {
    const int s = s0 + lane;
    const float scale = s < splits ? expf(base[s * (hd + 2)] - m) : 0.0f;
    const float ls = s < splits ? base[s * (hd + 2) + 1] * scale : 0.0f;
    l += warp_sum(ls);
    const int n = splits - s0 < 32 ? splits - s0 : 32;
    for (int j = 0; j < n; ++j) {
      const float sc = __shfl_sync(0xffffffffu, scale, j);
      const float* part = base + (s0 + j) * (hd + 2) + 2;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < hd) acc[i] = fmaf(part[d], sc, acc[i]);
      }
    }
  }
  float* out = a.out + out_index(a, row / a.heads, row % a.heads, 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < hd) out[d] = __fdiv_rn(acc[i], l);
  }
}

// ---------------------------------------------------------------------------
// Decode: grid (splits, kv_heads), 256 threads; the work of one block is
// attention_item (attn_core.cuh).
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(const cb_decode_attention_args a) {
  extern __shared__ float smem[];
  __shared__ int s_last;
  prefetch_share(a.prefetch_ptr, a.prefetch_bytes, static_cast<long long>(blockIdx.y) * gridDim.x + blockIdx.x,
                 static_cast<long long>(gridDim.x) * gridDim.y, threadIdx.x, kAttnThreads);
  pdl_wait();
  pdl_launch_dependents();
  attention_item<HD>(a, blockIdx.y, blockIdx.x, gridDim.x, smem, &s_last, threadIdx.x);
}

// ---- batched decode attention -------------------------------------------
// Sequence b's q | k | v row starts at qkv + b * qkv_stride; its caches,
// output, partials and counters are the b-th of `batch` equal slices;
// position, masks and RoPE row are shared (the sequences step together).
// One CTA per (range of 32-key chunks, KV head, sequence).  The chunks of a
// range are staged with cp.async into two alternating shared-memory buffers
// (the next chunk's copies are in flight while the current one is scored),
// each query head keeps an online softmax state (max, sum, p.v) across the
// chunks, and one partial per head is written per CTA; the last CTA of a
// (sequence, KV head) group merges the partials in range order.  Per chunk
// the arithmetic is the single-sequence decode attention's (RoPE of q and
// k at the bound position, write-mask blend of the cache rows, scores
// s / divisor + mask, exp against the running max).
// K/V element types of the batched kernel's shared-memory chunks: float32,
// or bfloat16 (a bfloat16 cache stays bfloat16 in shared memory: half the
// bytes; values convert to float32 where they are used).
template <typename KT>
struct KvTraits;
template <>
struct KvTraits<float> {
  static constexpr int kPad = 4;  // K row padding (elements): conflict-free 16-byte score loads
  static constexpr int kDtype = CB_F32;
};
template <>
struct KvTraits<uint16_t> {
  static constexpr int kPad = 8;  // keeps K rows 16-byte aligned for cp.async, loads conflict-free
  static constexpr int kDtype = CB_BF16;
};

// Four / two consecutive K/V values of a shared-memory row as float32.
__device__ __forceinline__ float4 smem_load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 smem_load4(const uint16_t* p) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                     __uint_as_float(w.y & 0xffff0000u));
}
__device__ __forceinline__ float2 smem_load2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 smem_load2(const uint16_t* p) {
  const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
// Stores four values already representable in the row's type.
__device__ __forceinline__ void smem_store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void smem_store4(uint16_t* p, float4 v) {
  *reinterpret_cast<uint2*>(p) = make_uint2((__float_as_uint(v.x) >> 16) | (__float_as_uint(v.y) & 0xffff0000u),
                                            (__float_as_uint(v.z) >> 16) | (__float_as_uint(v.w) & 0xffff0000u));
}

template <int HD, typename KT>
struct ChunkSmem {
  static constexpr int KS = HD + KvTraits<KT>::kPad;  // padded K rows (elements)
  static constexpr int kKBytes = kAttnSplit * KS * static_cast<int>(sizeof(KT));
  static constexpr int kVBytes = kAttnSplit * HD * static_cast<int>(sizeof(KT));
  // one staging buffer: K rows [32][KS], V rows [32][HD], write mask [32], mask [32]
  static constexpr int kBufBytes = kKBytes + kVBytes + 2 * kAttnSplit * 4;
  static_assert(kKBytes % 16 == 0 && kVBytes % 16 == 0, "16-byte aligned staging rows");
  float *q_rot, *k_new, *v_new, *cs, *sn;
  unsigned char* bufs;
  __device__ ChunkSmem(float* smem, int group) {
    q_rot = smem;                // [group][HD]
    k_new = q_rot + group * HD;  // [HD]
    v_new = k_new + HD;          // [HD]
    cs = v_new + HD;             // [HD / 2]
    sn = cs + HD / 2;            // [HD / 2]
    bufs = reinterpret_cast<unsigned char*>(sn + HD / 2);  // [2][kBufBytes]; 16-byte aligned (HD % 32 == 0)
  }
  __device__ KT* ks(int b) const { return reinterpret_cast<KT*>(bufs + b * kBufBytes); }
  __device__ KT* vs(int b) const { return reinterpret_cast<KT*>(bufs + b * kBufBytes + kKBytes); }
  __device__ float* wm(int b) const { return reinterpret_cast<float*>(bufs + b * kBufBytes + kKBytes + kVBytes); }
  __device__ float* maskv(int b) const { return wm(b) + kAttnSplit; }
};

inline long long chunk_smem_bytes(long long group, long long hd, int kv_dtype) {
  const long long es = kv_dtype == CB_BF16 ? 2 : 4, pad = kv_dtype == CB_BF16 ? 8 : 4;
  return ((group + 2) * hd + hd) * 4 + 2 * (kAttnSplit * (hd + pad) * es + kAttnSplit * hd * es + 2 * kAttnSplit * 4);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Issue the copies of chunk `chunk`'s K/V rows into buffer `buf` (one commit
// group per thread, possibly empty).
template <int HD, typename KT, int NT>
__device__ __forceinline__ void stage_chunk(const cb_decode_attention_args& a, const ChunkSmem<HD, KT>& s, int buf,
                                            int g, long long chunk, int tid) {
  constexpr int kUnits = HD * static_cast<int>(sizeof(KT)) / 16;  // 16-byte pieces per row
  constexpr int kEs = static_cast<int>(sizeof(KT));
  const long long lo = chunk * kAttnSplit;
  const int n = attn_rows(a, static_cast<int>(chunk));
  const long long first = (static_cast<long long>(g) * a.context + lo) * HD;
  const char* kc = static_cast<const char*>(kv_at(static_cast<const void*>(a.k_cache), first, KvTraits<KT>::kDtype));
  const char* vc = static_cast<const char*>(kv_at(static_cast<const void*>(a.v_cache), first, KvTraits<KT>::kDtype));
  char* kd = reinterpret_cast<char*>(s.ks(buf));
  char* vd = reinterpret_cast<char*>(s.vs(buf));
  for (int e = tid; e < n * kUnits; e += NT) {
    const int r = e / kUnits, u = e % kUnits;
    cp_async16(kd + r * ChunkSmem<HD, KT>::KS * kEs + u * 16, kc + r * HD * kEs + u * 16);
    cp_async16(vd + r * HD * kEs + u * 16, vc + r * HD * kEs + u * 16);
  }
  cp_async_commit();
}

// Write-mask and mask value of row `tid` of chunk `chunk` (threads tid < 32;
// the loads are consumed later, so they stay in flight meanwhile).
__device__ __forceinline__ void chunk_masks(const cb_decode_attention_args& a, long long chunk, int tid, float* wm,
                                            float* mk) {
  const long long r = chunk * kAttnSplit + tid;
  const bool in = tid < kAttnSplit && r < a.context;
  *wm = in ? load_as_f32(a.write_mask, r, a.write_mask_dtype) : 0.0f;
  *mk = in ? load_as_f32(a.mask, r, a.mask_dtype) : 0.0f;
}

// NT: threads per CTA (one warp per query head of the group, HPW heads per warp; 128 threads for groups
// of up to four heads, so more CTAs fit an SM)
template <int HD, int HPW, typename KT, int NT>  // HPW: query heads per warp (group <= NT / 32 * HPW); KT: K/V element type
__global__ void __launch_bounds__(NT, 1024 / NT) decode_attention_batched_kernel(const cb_decode_attention_args args,
                                                                                   long long qkv_stride,
                                                                                   int chunks_per_cta) {
  extern __shared__ float smem[];
  __shared__ int s_last;
  cb_decode_attention_args a = args;
  const long long b = blockIdx.z;
  const int g = static_cast<int>(blockIdx.y);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int warps = NT / 32;
  constexpr int half = HD / 2;
  constexpr int KS = ChunkSmem<HD, KT>::KS;
  constexpr int kDt = KvTraits<KT>::kDtype;
  constexpr int kPairs = (HD + 63) / 64;  // float2 output dims per lane
  const long long kv_rows = a.kv_heads * a.context * a.head_size;
  a.qkv += b * qkv_stride;
  a.k_cache = kv_at(a.k_cache, b * kv_rows, kDt);
  a.v_cache = kv_at(a.v_cache, b * kv_rows, kDt);
  a.out += b * a.heads * a.head_size;
  a.scratch += b * static_cast<long long>(gridDim.x) * a.heads * (a.head_size + 2);
  a.counters += b * a.kv_heads;
  const int group = static_cast<int>(a.heads / a.kv_heads);
  ChunkSmem<HD, KT> s(smem, group);
  const long long splits = (a.context + kAttnSplit - 1) / kAttnSplit;
  const long long c0 = static_cast<long long>(blockIdx.x) * chunks_per_cta;
  const long long c1 = c0 + chunks_per_cta < splits ? c0 + chunks_per_cta : splits;

  // the first chunk's copies and mask values overlap the RoPE row and q/k/v loads
  stage_chunk<HD, KT, NT>(a, s, 0, g, c0, tid);
  float wm_next, mk_next;
  chunk_masks(a, c0, tid, &wm_next, &mk_next);
  long long pos = load_index(a.position, 0, a.position_dtype);
  if (pos < 0 || pos >= a.n_positions) {
    if (tid == 0 && blockIdx.x == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_POSITION);
    pos = pos < 0 ? 0 : a.n_positions - 1;
  }
  for (int j = tid; j < half; j += NT) {
    s.cs[j] = a.cos_table[pos * half + j];
    s.sn[j] = a.sin_table[pos * half + j];
  }
  __syncthreads();
  for (int i = tid; i < group * half; i += NT) {
    const int h = i / half, j = i % half;
    const float* src = a.qkv + a.q_off + (static_cast<long long>(g) * group + h) * HD;
    const float lo = __ldcg(src + j), hi = __ldcg(src + j + half), c = s.cs[j], sv = s.sn[j];
    s.q_rot[h * HD + j] = fmaf(-hi, sv, __fmul_rn(lo, c));
    s.q_rot[h * HD + j + half] = fmaf(hi, c, __fmul_rn(lo, sv));
  }
  for (int j = tid; j < half; j += NT) {
    const float* src = a.qkv + a.k_off + static_cast<long long>(g) * HD;
    const float lo = __ldcg(src + j), hi = __ldcg(src + j + half), c = s.cs[j], sv = s.sn[j];
    s.k_new[j] = fmaf(-hi, sv, __fmul_rn(lo, c));
    s.k_new[j + half] = fmaf(hi, c, __fmul_rn(lo, sv));
  }
  for (int d = tid; d < HD; d += NT) s.v_new[d] = __ldcg(a.qkv + a.v_off + static_cast<long long>(g) * HD + d);
  if (tid < kAttnSplit) {
    s.wm(0)[tid] = wm_next;
    s.maskv(0)[tid] = mk_next;
  }

  float m_run[HPW], l_run[HPW];
  float2 acc[HPW][kPairs];
#pragma unroll
  for (int k = 0; k < HPW; ++k) {
    m_run[k] = -INFINITY;
    l_run[k] = 0.0f;
#pragma unroll
    for (int i = 0; i < kPairs; ++i) acc[k][i] = make_float2(0.0f, 0.0f);
  }

  for (long long c = c0; c < c1; ++c) {
    const int buf = static_cast<int>((c - c0) & 1);
    const bool more = c + 1 < c1;
    if (more) {
      stage_chunk<HD, KT, NT>(a, s, buf ^ 1, g, c + 1, tid);
      chunk_masks(a, c + 1, tid, &wm_next, &mk_next);  // stored after this chunk's scores
      cp_async_wait<1>();  // this thread's copies of chunk c have landed
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // every thread's copies of chunk c (and, first time round, q/k/v) are visible

    // rows with wm != 0 get the blend, in shared memory and in the cache
    const long long lo_pos = c * kAttnSplit;
    const int n = attn_rows(a, static_cast<int>(c));
    const long long first = (static_cast<long long>(g) * a.context + lo_pos) * HD;
    void* kc = kv_at(a.k_cache, first, kDt);
    void* vc = kv_at(a.v_cache, first, kDt);
    KT* ks = s.ks(buf);
    KT* vs = s.vs(buf);
    for (int e = tid; e < n * (HD / 4); e += NT) {
      const int r = e / (HD / 4), d4 = (e % (HD / 4)) * 4;
      const float wm = s.wm(buf)[r];
      if (wm == 0.0f) continue;
      const float keep = round_to(__fsub_rn(1.0f, wm), a.one_minus_dtype);
      float4 kv = smem_load4(ks + r * KS + d4);
      float4 vv = smem_load4(vs + r * HD + d4);
      float* kf = &kv.x;
      float* vf = &vv.x;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kf[i] = __fadd_rn(__fmul_rn(kf[i], keep), __fmul_rn(s.k_new[d4 + i], wm));
        vf[i] = __fadd_rn(__fmul_rn(vf[i], keep), __fmul_rn(s.v_new[d4 + i], wm));
      }
      kv = kv_store4(kc, e, kDt, kv);  // rounded for a bfloat16 cache, and attended as stored
      vv = kv_store4(vc, e, kDt, vv);
      smem_store4(ks + r * KS + d4, kv);
      smem_store4(vs + r * HD + d4, vv);
    }
    __syncthreads();

    // a warp's HPW query heads: scores with lane = position (each K row
    // loaded and converted once for all of them), then p @ v with lane = two
    // dims (each V pair loaded once), folded into every head's running state
    float x[HPW];
#pragma unroll
    for (int k = 0; k < HPW; ++k) x[k] = -INFINITY;
    if (lane < n) {
      float sacc[HPW][4];
#pragma unroll
      for (int k = 0; k < HPW; ++k) sacc[k][0] = sacc[k][1] = sacc[k][2] = sacc[k][3] = 0.0f;
      if constexpr (sizeof(KT) == 4) {
        const float4* kr = reinterpret_cast<const float4*>(ks + lane * KS);
#pragma unroll
        for (int d = 0; d < HD / 4; ++d) {
          const float4 ka = kr[d];
#pragma unroll
          for (int k = 0; k < HPW; ++k) {
            if (warp + k * warps >= group) continue;
            const float4 qa = reinterpret_cast<const float4*>(s.q_rot + (warp + k * warps) * HD)[d];
            sacc[k][0] = fmaf(qa.x, ka.x, sacc[k][0]);
            sacc[k][1] = fmaf(qa.y, ka.y, sacc[k][1]);
            sacc[k][2] = fmaf(qa.z, ka.z, sacc[k][2]);
            sacc[k][3] = fmaf(qa.w, ka.w, sacc[k][3]);
          }
        }
      } else {  // eight bfloat16 K values per 16-byte load, in the same accumulation order
        const uint4* kr = reinterpret_cast<const uint4*>(ks + lane * KS);
#pragma unroll
        for (int d = 0; d < HD / 8; ++d) {
          const uint4 w = kr[d];
          const float k0 = __uint_as_float(w.x << 16), k1 = __uint_as_float(w.x & 0xffff0000u);
          const float k2 = __uint_as_float(w.y << 16), k3 = __uint_as_float(w.y & 0xffff0000u);
          const float k4 = __uint_as_float(w.z << 16), k5 = __uint_as_float(w.z & 0xffff0000u);
          const float k6 = __uint_as_float(w.w << 16), k7 = __uint_as_float(w.w & 0xffff0000u);
#pragma unroll
          for (int k = 0; k < HPW; ++k) {
            if (warp + k * warps >= group) continue;
            const float4* q = reinterpret_cast<const float4*>(s.q_rot + (warp + k * warps) * HD);
            const float4 qa = q[2 * d], qb = q[2 * d + 1];
            sacc[k][0] = fmaf(qa.x, k0, sacc[k][0]);
            sacc[k][1] = fmaf(qa.y, k1, sacc[k][1]);
            sacc[k][2] = fmaf(qa.z, k2, sacc[k][2]);
            sacc[k][3] = fmaf(qa.w, k3, sacc[k][3]);
            sacc[k][0] = fmaf(qb.x, k4, sacc[k][0]);
            sacc[k][1] = fmaf(qb.y, k5, sacc[k][1]);
            sacc[k][2] = fmaf(qb.z, k6, sacc[k][2]);
            sacc[k][3] = fmaf(qb.w, k7, sacc[k][3]);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < HPW; ++k)
        x[k] = __fadd_rn(__fdiv_rn((sacc[k][0] + sacc[k][1]) + (sacc[k][2] + sacc[k][3]), a.divisor),
                         s.maskv(buf)[lane]);
    }
    float p[HPW], scale[HPW];
#pragma unroll
    for (int k = 0; k < HPW; ++k) {
      const float mn = fmaxf(m_run[k], warp_max(x[k]));
      scale[k] = expf(m_run[k] - mn);  // 0 on the first chunk (running max -inf)
      p[k] = lane < n ? expf(x[k] - mn) : 0.0f;
      l_run[k] = fmaf(l_run[k], scale[k], warp_sum(p[k]));
      m_run[k] = mn;
    }
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
      const int d = i * 64 + 2 * lane;
      const bool mine = d < HD;
      float2 a0[HPW], a1[HPW];
#pragma unroll
      for (int k = 0; k < HPW; ++k) a0[k] = a1[k] = make_float2(0.0f, 0.0f);
      for (int j = 0; j < n; j += 2) {  // every lane shuffles; rows j < n only are read
        float p0[HPW], p1[HPW];
#pragma unroll
        for (int k = 0; k < HPW; ++k) {
          p0[k] = __shfl_sync(0xffffffffu, p[k], j);
          p1[k] = __shfl_sync(0xffffffffu, p[k], j + 1);
        }
        if (mine) {
          const float2 v0 = smem_load2(vs + j * HD + d);
#pragma unroll
          for (int k = 0; k < HPW; ++k) {
            a0[k].x = fmaf(p0[k], v0.x, a0[k].x);
            a0[k].y = fmaf(p0[k], v0.y, a0[k].y);
          }
          if (j + 1 < n) {
            const float2 v1 = smem_load2(vs + (j + 1) * HD + d);
#pragma unroll
            for (int k = 0; k < HPW; ++k) {
              a1[k].x = fmaf(p1[k], v1.x, a1[k].x);
              a1[k].y = fmaf(p1[k], v1.y, a1[k].y);
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        acc[k][i].x = fmaf(acc[k][i].x, scale[k], a0[k].x + a1[k].x);
        acc[k][i].y = fmaf(acc[k][i].y, scale[k], a0[k].y + a1[k].y);
      }
    }
    if (more && tid < kAttnSplit) {
      s.wm(buf ^ 1)[tid] = wm_next;
      s.maskv(buf ^ 1)[tid] = mk_next;
    }
    __syncthreads();  // buffer `buf` is refilled by the copies issued for chunk c + 2
  }

  // this CTA's partial per head: (max, sum, unnormalised output)
#pragma unroll
  for (int k = 0; k < HPW; ++k) {
    const int h = warp + k * warps;
    if (h >= group) break;
    float* part = a.scratch + (static_cast<long long>(blockIdx.x) * a.heads + g * group + h) * (HD + 2);
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
      const int d = i * 64 + 2 * lane;
      if (d < HD) *reinterpret_cast<float2*>(part + 2 + d) = acc[k][i];
    }
    if (lane == 0) {
      part[0] = m_run[k];
      part[1] = l_run[k];
    }
  }

  // the last CTA of the group merges the partials in range order; the
  // barrier orders every thread's partial before thread 0's release, whose
  // acquire side (the last CTA's thread 0, then its barrier) makes them
  // visible there
  __syncthreads();
  const int parts = static_cast<int>(gridDim.x);
  if (tid == 0) s_last = ticket_acq_rel(a.counters + g) == static_cast<unsigned>(parts - 1);
  __syncthreads();
  if (!s_last) return;
  const long long stride = a.heads * (HD + 2);
  for (int h = warp; h < group; h += warps) {
    const long long head = static_cast<long long>(g) * group + h;
    const float* base = a.scratch + head * (HD + 2);
    float m = -INFINITY;
    for (int sp = lane; sp < parts; sp += 32) m = fmaxf(m, __ldcg(base + sp * stride));
    m = warp_max(m);
    float l = 0.0f, out[HD / 32 > 0 ? HD / 32 : 1];
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) out[i] = 0.0f;
    for (int s0 = 0; s0 < parts; s0 += 32) {
      const int sp = s0 + lane;
      const float sc_mine = sp < parts ? expf(__ldcg(base + sp * stride) - m) : 0.0f;
      l += warp_sum(sp < parts ? __ldcg(base + sp * stride + 1) * sc_mine : 0.0f);
      const int n = parts - s0 < 32 ? parts - s0 : 32;
      for (int j = 0; j < n; ++j) {
        const float sc = __shfl_sync(0xffffffffu, sc_mine, j);
        const float* part = base + (s0 + j) * stride + 2;
#pragma unroll
        for (int i = 0; i < HD / 32; ++i) out[i] = fmaf(__ldcg(part + lane + 32 * i), sc, out[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) a.out[head * HD + lane + 32 * i] = __fdiv_rn(out[i], l);
  }
  if (tid == 0) a.counters[g] = 0u;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

long long cb_decode_attention_batched_scratch(const cb_decode_attention_args* a, long long batch) {
  if (a == nullptr || batch <= 0) return 0;
  return batch * cb_decode_attention_scratch(a);
}

int cb_decode_attention_batched(const cb_decode_attention_args* a, long long batch, long long qkv_stride,
                                cb_stream_t stream) {
  CB_REQUIRE(a != nullptr && batch >= 1 && batch < 65536, "decode attention: batch %lld (1..65535)", batch);
  CB_REQUIRE(a->head_size == 32 || a->head_size == 64 || a->head_size == 128 || a->head_size == 256,
             "decode attention: head size %lld unsupported (32/64/128/256)", a->head_size);
  CB_REQUIRE(a->kv_heads > 0 && a->heads % a->kv_heads == 0, "decode attention: bad head grouping");
  CB_REQUIRE(a->context > 0, "decode attention: empty context");
  CB_REQUIRE(a->qkv != nullptr && a->mask != nullptr && a->write_mask != nullptr && a->position != nullptr &&
                 a->scratch != nullptr && a->counters != nullptr && a->out != nullptr,
             "decode attention: qkv, masks, position, scratch, counters and out are required");
  CB_REQUIRE(qkv_stride >= a->v_off + a->kv_heads * a->head_size, "decode attention: qkv rows overlap");
  CB_REQUIRE(a->split == 0 || a->split == kAttnSplit, "decode attention: split must be %d", kAttnSplit);
  const long long splits = (a->context + kAttnSplit - 1) / kAttnSplit;
  CB_REQUIRE(splits < (1LL << 31) && a->kv_heads < 65536, "decode attention: grid too large");
  const long long group = a->heads / a->kv_heads;
  CB_REQUIRE(group <= 32, "decode attention: at most 32 query heads per KV head (got %lld)", group);
  CB_REQUIRE(a->kv_dtype == CB_F32 || a->kv_dtype == CB_BF16, "decode attention: caches must be float32 or bfloat16");
  const size_t smem = static_cast<size_t>(chunk_smem_bytes(group, a->head_size, a->kv_dtype));
  CB_REQUIRE(smem <= 200 * 1024, "decode attention: too many query heads per KV head");
  const long long groups = batch * a->kv_heads;
  const bool narrow = group <= 8;  // 128-thread CTAs (two heads per warp past four), twice as many per SM
  const int threads = narrow ? 128 : 256;
  using BatchedKernel = void (*)(const cb_decode_attention_args, long long, int);
  BatchedKernel kernel = nullptr;
#define CB_BATCHED_PICK(HD, HPW)                                                                          \
  kernel = a->kv_dtype == CB_BF16 ? (narrow ? decode_attention_batched_kernel<HD, HPW, uint16_t, 128>       \
                                            : decode_attention_batched_kernel<HD, HPW, uint16_t, 256>)      \
                                  : (narrow ? decode_attention_batched_kernel<HD, HPW, float, 128>          \
                                            : decode_attention_batched_kernel<HD, HPW, float, 256>);
#define CB_BATCHED_HD(HD)            \
  case HD:                           \
    if (group <= 4)                  \
      CB_BATCHED_PICK(HD, 1)         \
    else if (group <= 16)            \
      CB_BATCHED_PICK(HD, 2)         \
    else                             \
      CB_BATCHED_PICK(HD, 4)         \
    break;
  switch (a->head_size) {
    CB_BATCHED_HD(32)
    CB_BATCHED_HD(64)
    CB_BATCHED_HD(128)
    CB_BATCHED_HD(256)
  }
#undef CB_BATCHED_HD
#undef CB_BATCHED_PICK
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  // Each CTA takes a range of consecutive chunks of its (sequence, KV head).
  // The range length minimises waves x (chunks per CTA + one chunk's worth of
  // per-CTA set-up and merge) over the CTAs resident at once -- shared
  // memory, not threads, bounds them at head size 128 -- so that no second
  // wave runs a few CTAs while the other SMs idle.
  static thread_local BatchedKernel cached_kernel = nullptr;
  static thread_local size_t cached_smem = 0;
  static thread_local int cached_resident = 0;
  if (e == cudaSuccess && (kernel != cached_kernel || smem != cached_smem)) {
    int resident = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kernel, threads, smem);
    cached_kernel = kernel;
    cached_smem = smem;
    cached_resident = resident > 0 ? resident : 1;
  }
  const long long capacity = static_cast<long long>(cached_resident) * sm_count();
  long long chunks = splits, best_cost = -1, best_waves = 0;
  for (long long c = 1; c <= splits; ++c) {
    const long long ctas_per_group = (splits + c - 1) / c;
    if (c > 1 && (splits + c - 2) / (c - 1) == ctas_per_group) continue;  // same CTAs, longer ranges
    const long long waves = (groups * ctas_per_group + capacity - 1) / capacity;
    const long long cost = waves * (c + 1);
    if (best_cost < 0 || cost < best_cost || (cost == best_cost && waves < best_waves)) {
      best_cost = cost;
      best_waves = waves;
      chunks = c;
    }
  }
  const long long ctas = (splits + chunks - 1) / chunks;
  const dim3 grid(static_cast<unsigned>(ctas), static_cast<unsigned>(a->kv_heads), static_cast<unsigned>(batch));
  const int per_cta = static_cast<int>(chunks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (e == cudaSuccess) kernel<<<grid, threads, smem, s>>>(*a, qkv_stride, per_cta);
  if (e != cudaSuccess) {
    set_error("cb_decode_attention_batched: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_decode_attention_batched");
}

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

long long cb_sdpa_query_scratch(const cb_sdpa_args* a) {
  if (a == nullptr || a->batch <= 0 || a->heads <= 0 || a->tk <= 0 || a->head_size <= 0) return 0;
  const long long splits = (a->tk + kQSplit - 1) / kQSplit;
  return a->batch * a->heads * splits * (a->head_size + 2) * static_cast<long long>(sizeof(float));
}

int cb_sdpa_query(const cb_sdpa_args* a, void* scratch, cb_stream_t stream) {
  CB_REQUIRE(a != nullptr && a->q != nullptr && a->k != nullptr && a->v != nullptr && a->out != nullptr,
             "sdpa_query: q, k, v and out are required");
  CB_REQUIRE(a->tq == 1, "sdpa_query: one query row per head (tq = %lld)", a->tq);
  CB_REQUIRE(a->head_size == 32 || a->head_size == 64 || a->head_size == 128 || a->head_size == 256,
             "sdpa_query: head size %lld unsupported (32/64/128/256)", a->head_size);
  CB_REQUIRE(a->kv_heads > 0 && a->heads % a->kv_heads == 0, "sdpa_query: heads must be a multiple of KV heads");
  CB_REQUIRE(a->k_dtype == CB_F32 && a->v_dtype == CB_F32, "sdpa_query: K/V must be float32");
  CB_REQUIRE(a->k_strides[3] == 1 && a->v_strides[3] == 1 && a->k_strides[2] % 4 == 0 && a->v_strides[2] % 4 == 0 &&
                 a->k_strides[1] % 4 == 0 && a->v_strides[1] % 4 == 0 && a->k_strides[0] % 4 == 0 &&
                 a->v_strides[0] % 4 == 0 && a->k_offset % 4 == 0 && a->v_offset % 4 == 0 &&
                 (reinterpret_cast<uintptr_t>(a->k) & 15) == 0 && (reinterpret_cast<uintptr_t>(a->v) & 15) == 0,
             "sdpa_query: K/V rows must be contiguous and 16-byte aligned");
  CB_REQUIRE(scratch != nullptr && (reinterpret_cast<uintptr_t>(scratch) & 15) == 0,
             "sdpa_query: scratch (cb_sdpa_query_scratch bytes, 16-byte aligned) is required");
  if (a->batch == 0 || a->heads == 0) return CB_OK;
  const long long splits = (a->tk + kQSplit - 1) / kQSplit;
  CB_REQUIRE(splits < (1LL << 31) && a->kv_heads < 65536 && a->batch < 65536, "sdpa_query: grid too large");
  const long long group = a->heads / a->kv_heads;
  const size_t smem = static_cast<size_t>(qsplit_smem_floats(group, a->head_size)) * sizeof(float);
  CB_REQUIRE(smem <= 200 * 1024, "sdpa_query: too many query heads per KV head");
  float* parts = static_cast<float*>(scratch);
  const dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(a->kv_heads), static_cast<unsigned>(a->batch));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define CB_QUERY_CASE(HD)                                                                                   \
  case HD:                                                                                                  \
    e = cudaFuncSetAttribute(sdpa_query_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,            \
                             static_cast<int>(smem));                                                       \
    if (e == cudaSuccess) sdpa_query_kernel<HD><<<grid, kThreads, smem, s>>>(*a, parts, static_cast<int>(splits)); \
    break;
  switch (a->head_size) {
    CB_QUERY_CASE(32)
    CB_QUERY_CASE(64)
    CB_QUERY_CASE(128)
    CB_QUERY_CASE(256)
  }
#undef CB_QUERY_CASE
  if (e != cudaSuccess) {
    set_error("cb_sdpa_query: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  const long long rows = a->batch * a->heads;
  sdpa_query_merge_kernel<<<static_cast<unsigned>((rows + kMergeWarps - 1) / kMergeWarps), kMergeWarps * 32, 0, s>>>(
      parts, rows, static_cast<int>(splits), static_cast<int>(a->head_size), *a);
  return check_launch("cb_sdpa_query");
}

long long cb_decode_attention_scratch(const cb_decode_attention_args* a) {
  const long long splits = (a->context + kAttnSplit - 1) / kAttnSplit;
  return splits * a->heads * (a->head_size + 2);
}

int cb_decode_attention(const cb_decode_attention_args* a, cb_stream_t stream) {
  CB_REQUIRE(a->head_size == 32 || a->head_size == 64 || a->head_size == 128 || a->head_size == 256,
             "decode attention: head size %lld unsupported (32/64/128/256)", a->head_size);
  CB_REQUIRE(a->kv_heads > 0 && a->heads % a->kv_heads == 0, "decode attention: bad head grouping");
  CB_REQUIRE(a->context > 0, "decode attention: empty context");
  CB_REQUIRE(a->mask != nullptr && a->write_mask != nullptr && a->position != nullptr,
             "decode attention: mask, write mask and position are required");
  CB_REQUIRE(a->kv_dtype == CB_F32 || a->kv_dtype == CB_BF16, "decode attention: caches must be float32 or bfloat16");
  CB_REQUIRE(a->split == 0 || a->split == kAttnSplit, "decode attention: split must be %d", kAttnSplit);
  const long long splits = (a->context + kAttnSplit - 1) / kAttnSplit;
  CB_REQUIRE(splits < 65536 && a->kv_heads < 65536, "decode attention: grid too large");
  const long long group = a->heads / a->kv_heads;
  const long long hd = a->head_size;
  const size_t smem = static_cast<size_t>(attn_smem_floats(group, hd)) * sizeof(float);
  CB_REQUIRE(smem <= 200 * 1024, "decode attention: too many query heads per KV head");
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(a->kv_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define CB_DECODE_CASE(HD)                                                                          \
  case HD:                                                                                          \
    cudaFuncSetAttribute(decode_attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                         static_cast<int>(smem));                                                   \
    e = launch(decode_attention_kernel<HD>, grid, dim3(kAttnThreads), smem, s, a->pdl != 0, *a);         \
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

// Single-token decode attention for one (context split, KV head) work item,
// shared by the standalone cb_decode_attention kernel and the decode-step
// megakernel.  256 threads (8 warps) execute it; `attn_sync` synchronises
// them (named barrier 1) so it also runs inside a block that has extra warps.
//
// The item has two halves:
//  * attention_stage_cache: the split's K/V cache rows, write-mask and mask
//    values into shared memory.  Nothing here depends on this step's q/k/v,
//    so the megakernel runs it before waiting for the QKV phase;
//  * attention_finish: rope the new q/k rows, apply the write-mask blend
//    cache*(1-wm) + new*wm (float32, as llama.py:511-512 computes it) to the
//    rows with wm != 0 and write them back (rounded to bfloat16 for a
//    bfloat16 cache), compute every (query head,
//    position) score in one pass (x = q.k / divisor + mask), and write the
//    split's partial softmax state.  With `merge`, the last item of each KV
//    group then merges the splits in split order (deterministic) and resets
//    the group counter; without it the caller merges (attention_merge_chunk).
#pragma once

#include "common.cuh"
#include "sync.cuh"

namespace cb {

constexpr int kAttnThreads = 256;
constexpr int kAttnSplit = 32;

__device__ __forceinline__ void attn_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnThreads) : "memory");
}

// Shared floats an item needs.
__host__ __device__ inline long long attn_smem_floats(long long group, long long hd) {
  return (group + 2) * hd + kAttnSplit * (hd + 4) + kAttnSplit * hd + 2 * kAttnSplit + hd;
}

template <int HD>
struct AttnSmem {
  static constexpr int KS = HD + 4;  // padded K rows: conflict-free float4 score loads
  float *q_rot, *k_new, *v_new, *ks, *vs, *wm, *maskv, *cs, *sn;
  __device__ AttnSmem(float* smem, int group) {
    q_rot = smem;                        // [group][HD]
    k_new = q_rot + group * HD;          // [HD]
    v_new = k_new + HD;                  // [HD]
    ks = v_new + HD;                     // [kAttnSplit][KS]
    vs = ks + kAttnSplit * KS;           // [kAttnSplit][HD]
    wm = vs + kAttnSplit * HD;           // [kAttnSplit]
    maskv = wm + kAttnSplit;             // [kAttnSplit]
    cs = maskv + kAttnSplit;             // [HD / 2]: the position's RoPE cosines
    sn = cs + HD / 2;                    // [HD / 2]: sines
  }
};

// KV cache element access for float32 or bfloat16 caches: `base` offset by
// `elems` elements, and groups of four consecutive values (16 or 8 bytes).
__device__ __forceinline__ const void* kv_at(const void* base, long long elems, int dtype) {
  return static_cast<const char*>(base) + elems * (dtype == CB_BF16 ? 2 : 4);
}
__device__ __forceinline__ void* kv_at(void* base, long long elems, int dtype) {
  return static_cast<char*>(base) + elems * (dtype == CB_BF16 ? 2 : 4);
}
__device__ __forceinline__ float4 kv_load4(const void* base, long long i4, int dtype) {
  if (dtype == CB_BF16) {
    const uint2 w = __ldcg(reinterpret_cast<const uint2*>(base) + i4);
    return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                       __uint_as_float(w.y & 0xffff0000u));
  }
  return __ldcg(reinterpret_cast<const float4*>(base) + i4);
}
// Stores four values (rounded to bfloat16 for a bfloat16 cache) and returns
// them as stored.
__device__ __forceinline__ float4 kv_store4(void* base, long long i4, int dtype, float4 v) {
  if (dtype == CB_BF16) {
    const uint32_t b0 = __bfloat16_as_ushort(__float2bfloat16_rn(v.x)), b1 = __bfloat16_as_ushort(__float2bfloat16_rn(v.y));
    const uint32_t b2 = __bfloat16_as_ushort(__float2bfloat16_rn(v.z)), b3 = __bfloat16_as_ushort(__float2bfloat16_rn(v.w));
    reinterpret_cast<uint2*>(base)[i4] = make_uint2(b0 | (b1 << 16), b2 | (b3 << 16));
    return make_float4(__uint_as_float(b0 << 16), __uint_as_float(b1 << 16), __uint_as_float(b2 << 16),
                       __uint_as_float(b3 << 16));
  }
  reinterpret_cast<float4*>(base)[i4] = v;
  return v;
}

__device__ __forceinline__ int attn_rows(const cb_decode_attention_args& a, int split) {
  const long long lo = static_cast<long long>(split) * kAttnSplit;
  return static_cast<int>(a.context - lo < kAttnSplit ? a.context - lo : kAttnSplit);
}

template <int HD>
__device__ void attention_stage_cache(const cb_decode_attention_args& a, int g, int split, float* smem,
                                      int tid) {
  const int group = static_cast<int>(a.heads / a.kv_heads);
  AttnSmem<HD> s(smem, group);
  constexpr int half = HD / 2;
  const long long lo_pos = static_cast<long long>(split) * kAttnSplit;
  const int n = attn_rows(a, split);
  const long long first = (static_cast<long long>(g) * a.context + lo_pos) * HD;
  const void* kc = kv_at(static_cast<const void*>(a.k_cache), first, a.kv_dtype);
  const void* vc = kv_at(static_cast<const void*>(a.v_cache), first, a.kv_dtype);
  for (int e = tid; e < n * (HD / 4); e += kAttnThreads) {
    const int r = e / (HD / 4), d4 = (e % (HD / 4)) * 4;
    const float4 kv = kv_load4(kc, e, a.kv_dtype);
    const float4 vv = kv_load4(vc, e, a.kv_dtype);
    *reinterpret_cast<float4*>(s.ks + r * AttnSmem<HD>::KS + d4) = kv;
    *reinterpret_cast<float4*>(s.vs + r * HD + d4) = vv;
  }
  // V rows past a short last split are zeros: p @ v runs a fixed number of
  // rows, and 0 * 0 adds nothing
  for (int e = n * HD + tid; e < kAttnSplit * HD; e += kAttnThreads) s.vs[e] = 0.0f;
  for (int r = tid; r < n; r += kAttnThreads) {
    s.wm[r] = load_as_f32(a.write_mask, lo_pos + r, a.write_mask_dtype);
    s.maskv[r] = load_as_f32(a.mask, lo_pos + r, a.mask_dtype);
  }
  // the position's RoPE row (the position is an input of the step, not of q/k/v)
  long long pos = load_index(a.position, 0, a.position_dtype);
  if (pos < 0 || pos >= a.n_positions) {
    if (tid == 0 && split == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_POSITION);
    pos = pos < 0 ? 0 : a.n_positions - 1;
  }
  for (int j = tid; j < half; j += kAttnThreads) {
    s.cs[j] = a.cos_table[pos * half + j];
    s.sn[j] = a.sin_table[pos * half + j];
  }
}

// Merged attention output for elements [e0, e0 + n) of one head (n <= 8,
// inside one head) from the split partials (scratch layout above).  Online
// over splits: the same value as the in-kernel merge up to the last bits.
// Loads go through L1 (the partials are written once per launch, before the
// caller's phase): a lane's eight values share sectors the L1 fetches once.
__device__ __forceinline__ void attention_merge_chunk(const float* parts, long long heads, int hd, int splits,
                                                      long long e0, int n, float* out) {
  const long long head = e0 / hd;
  const int d0 = static_cast<int>(e0 % hd);
  const long long stride = heads * (hd + 2);
  const float* base = parts + head * (hd + 2);
  float m = -INFINITY, lsum = 0.0f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll 4
  for (int sp = 0; sp < splits; ++sp) {
    const float* part = base + sp * stride;
    const float ms = __ldca(part), ls = __ldca(part + 1);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = i < n ? __ldca(part + 2 + d0 + i) : 0.0f;
    if (ms > m) {
      const float rescale = expf(m - ms);  // 0 on the first split (m = -inf)
      lsum *= rescale;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= rescale;
      m = ms;
    }
    const float scale = expf(ms - m);
    lsum = fmaf(ls, scale, lsum);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = fmaf(v[i], scale, acc[i]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < n) out[i] = __fdiv_rn(acc[i], lsum);
}

// Merged output for the two elements [e0, e0 + 2) of one head, for up to
// kMergeRegSplits splits: every split's max, sum and two values are loaded
// first (one round trip), then merged in split order -- max over the splits,
// then the rescaled sums -- as two passes over registers.
constexpr int kMergeRegSplits = 16;

__device__ __forceinline__ void attention_merge_pair_regs(const float* parts, long long heads, int hd, int splits,
                                                          long long e0, float* out) {
  const long long head = e0 / hd;
  const int d0 = static_cast<int>(e0 % hd);
  const long long stride = heads * (hd + 2);
  const float* base = parts + head * (hd + 2);
  float m[kMergeRegSplits], l[kMergeRegSplits], v0[kMergeRegSplits], v1[kMergeRegSplits];
#pragma unroll
  for (int sp = 0; sp < kMergeRegSplits; ++sp) {
    if (sp < splits) {
      const float* part = base + sp * stride;
      m[sp] = __ldcg(part);
      l[sp] = __ldcg(part + 1);
      const float2 v = __ldcg(reinterpret_cast<const float2*>(part + 2 + d0));
      v0[sp] = v.x;
      v1[sp] = v.y;
    }
  }
  float mmax = -INFINITY;
#pragma unroll
  for (int sp = 0; sp < kMergeRegSplits; ++sp)
    if (sp < splits) mmax = fmaxf(mmax, m[sp]);
  float lsum = 0.0f, a0 = 0.0f, a1 = 0.0f;
#pragma unroll
  for (int sp = 0; sp < kMergeRegSplits; ++sp) {
    if (sp < splits) {
      const float scale = expf(m[sp] - mmax);
      lsum = fmaf(l[sp], scale, lsum);
      a0 = fmaf(v0[sp], scale, a0);
      a1 = fmaf(v1[sp], scale, a1);
    }
  }
  out[0] = __fdiv_rn(a0, lsum);
  out[1] = __fdiv_rn(a1, lsum);
}

// Needs attention_stage_cache's shared memory (and an attn_sync after it).
// kRegMerge = false compiles only the warp-per-head merge (fewer registers:
// more blocks per SM for launches of many small items).
template <int HD, bool kRegMerge = true>
__device__ void attention_finish(const cb_decode_attention_args& a, int g, int split, int splits, float* smem,
                                 int* s_last, int tid, bool merge, unsigned long long* stamps = nullptr) {
  const int group = static_cast<int>(a.heads / a.kv_heads);
  constexpr int half = HD / 2;
  constexpr int KS = AttnSmem<HD>::KS;
  AttnSmem<HD> s(smem, group);
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int warps = kAttnThreads / 32;
  const float* cs = s.cs;
  const float* sn = s.sn;
  for (int i = tid; i < group * half; i += kAttnThreads) {
    const int h = i / half, j = i % half;
    const float* src = a.qkv + a.q_off + (static_cast<long long>(g) * group + h) * HD;
    const float lo = __ldcg(src + j), hi = __ldcg(src + j + half), c = cs[j], sv = sn[j];
    s.q_rot[h * HD + j] = fmaf(-hi, sv, __fmul_rn(lo, c));
    s.q_rot[h * HD + j + half] = fmaf(hi, c, __fmul_rn(lo, sv));
  }
  for (int j = tid; j < half; j += kAttnThreads) {
    const float* src = a.qkv + a.k_off + static_cast<long long>(g) * HD;
    const float lo = __ldcg(src + j), hi = __ldcg(src + j + half), c = cs[j], sv = sn[j];
    s.k_new[j] = fmaf(-hi, sv, __fmul_rn(lo, c));
    s.k_new[j + half] = fmaf(hi, c, __fmul_rn(lo, sv));
  }
  for (int d = tid; d < HD; d += kAttnThreads)
    s.v_new[d] = __ldcg(a.qkv + a.v_off + static_cast<long long>(g) * HD + d);
  attn_sync();
  if (stamps != nullptr && tid == 0) stamps[0] = global_ns();

  // rows with wm != 0 get the blend, in shared memory and in the cache
  const long long lo_pos = static_cast<long long>(split) * kAttnSplit;
  const int n = attn_rows(a, split);
  const long long first = (static_cast<long long>(g) * a.context + lo_pos) * HD;
  void* kc = kv_at(a.k_cache, first, a.kv_dtype);
  void* vc = kv_at(a.v_cache, first, a.kv_dtype);
  for (int e = tid; e < n * (HD / 4); e += kAttnThreads) {
    const int r = e / (HD / 4), d4 = (e % (HD / 4)) * 4;
    const float wm = s.wm[r];
    if (wm == 0.0f) continue;
    const float keep = round_to(__fsub_rn(1.0f, wm), a.one_minus_dtype);
    float4 kv = *reinterpret_cast<float4*>(s.ks + r * KS + d4);
    float4 vv = *reinterpret_cast<float4*>(s.vs + r * HD + d4);
    float* kf = &kv.x;
    float* vf = &vv.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      kf[i] = __fadd_rn(__fmul_rn(kf[i], keep), __fmul_rn(s.k_new[d4 + i], wm));
      vf[i] = __fadd_rn(__fmul_rn(vf[i], keep), __fmul_rn(s.v_new[d4 + i], wm));
    }
    kv = kv_store4(kc, e, a.kv_dtype, kv);  // attended as stored
    vv = kv_store4(vc, e, a.kv_dtype, vv);
    *reinterpret_cast<float4*>(s.ks + r * KS + d4) = kv;
    *reinterpret_cast<float4*>(s.vs + r * HD + d4) = vv;
  }
  attn_sync();
  if (stamps != nullptr && tid == 0) stamps[1] = global_ns();

  // One warp per query head (looping): scores with lane = position, then
  // p @ v with lane = two dims, the probabilities moving between them by
  // shuffle.  Partials (max, sum, unnormalised output) to scratch.
  for (int h = warp; h < group; h += warps) {
    float x = -INFINITY;
    if (lane < n) {
      const float4* q = reinterpret_cast<const float4*>(s.q_rot + h * HD);
      const float4* k = reinterpret_cast<const float4*>(s.ks + lane * KS);
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll
      for (int d = 0; d < HD / 4; ++d) {
        const float4 qa = q[d], ka = k[d];
        s0 = fmaf(qa.x, ka.x, s0);
        s1 = fmaf(qa.y, ka.y, s1);
        s2 = fmaf(qa.z, ka.z, s2);
        s3 = fmaf(qa.w, ka.w, s3);
      }
      x = __fadd_rn(__fdiv_rn((s0 + s1) + (s2 + s3), a.divisor), s.maskv[lane]);
    }
    const float m = warp_max(x);
    const float p = lane < n ? expf(x - m) : 0.0f;
    const float l = warp_sum(p);
    float* part = a.scratch + (static_cast<long long>(split) * a.heads + g * group + h) * (HD + 2);
#pragma unroll
    for (int d0 = 0; d0 < HD; d0 += 64) {
      const int d = d0 + 2 * lane;
      const bool mine = d < HD;
      float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
      // every row of the split's slot: p is 0 at lanes >= n and those V rows
      // are zeros, so the sums equal the sums over the n rows
#pragma unroll
      for (int j = 0; j < kAttnSplit; j += 2) {
        const float p0 = __shfl_sync(0xffffffffu, p, j);
        const float p1 = __shfl_sync(0xffffffffu, p, j + 1);
        if (mine) {
          const float2 v0 = *reinterpret_cast<const float2*>(s.vs + j * HD + d);
          const float2 v1 = *reinterpret_cast<const float2*>(s.vs + (j + 1) * HD + d);
          acc0.x = fmaf(p0, v0.x, acc0.x);
          acc0.y = fmaf(p0, v0.y, acc0.y);
          acc1.x = fmaf(p1, v1.x, acc1.x);
          acc1.y = fmaf(p1, v1.y, acc1.y);
        }
      }
      if (mine) *reinterpret_cast<float2*>(part + 2 + d) = make_float2(acc0.x + acc1.x, acc0.y + acc1.y);
    }
    if (lane == 0) {
      part[0] = m;
      part[1] = l;
    }
  }
  if (stamps != nullptr && tid == 0) stamps[2] = stamps[3] = global_ns();
  if (!merge) return;

  // merge the splits of this KV group in split order; the barrier orders every
  // thread's partial before thread 0's release, whose acquire side (the last
  // item's thread 0, then its barrier) makes all partials visible there
  attn_sync();
  if (tid == 0) {
    const unsigned ticket = ticket_acq_rel(a.counters + g);
    *s_last = ticket == static_cast<unsigned>(splits - 1);
  }
  attn_sync();
  if (!*s_last) return;
  if (kRegMerge && splits <= kMergeRegSplits) {
    for (int i = tid; i < group * half; i += kAttnThreads) {  // two dims of one head per thread
      const long long e0 = (static_cast<long long>(g) * group + i / half) * HD + (i % half) * 2;
      float merged[8];
      attention_merge_pair_regs(a.scratch, a.heads, HD, splits, e0, merged);
      a.out[e0] = merged[0];
      a.out[e0 + 1] = merged[1];
    }
  } else {
    // many splits: one warp per head; lanes take the splits' maxima and sums,
    // the scales move to the dimension lanes by shuffle, so every split's
    // values are loaded independently (sums in a fixed order: deterministic)
    const long long stride = a.heads * (HD + 2);
    for (int h = warp; h < group; h += warps) {
      const long long head = static_cast<long long>(g) * group + h;
      const float* base = a.scratch + head * (HD + 2);
      float m = -INFINITY;
      for (int sp = lane; sp < splits; sp += 32) m = fmaxf(m, __ldcg(base + sp * stride));
      m = warp_max(m);
      float l = 0.0f, acc[HD / 32];
#pragma unroll
      for (int i = 0; i < HD / 32; ++i) acc[i] = 0.0f;
      for (int s0 = 0; s0 < splits; s0 += 32) {
        const int sp = s0 + lane;
        const float scale = sp < splits ? expf(__ldcg(base + sp * stride) - m) : 0.0f;
        l += warp_sum(sp < splits ? __ldcg(base + sp * stride + 1) * scale : 0.0f);
        const int n = splits - s0 < 32 ? splits - s0 : 32;
#pragma unroll 4
        for (int j = 0; j < n; ++j) {
          const float sc = __shfl_sync(0xffffffffu, scale, j);
          const float* part = base + (s0 + j) * stride + 2;
#pragma unroll
          for (int i = 0; i < HD / 32; ++i) acc[i] = fmaf(__ldcg(part + lane + 32 * i), sc, acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < HD / 32; ++i) a.out[head * HD + lane + 32 * i] = __fdiv_rn(acc[i], l);
    }
  }
  if (tid == 0) a.counters[g] = 0u;
}

// The whole item: stage, then finish with the in-kernel merge.
template <int HD, bool kRegMerge = true>
__device__ void attention_item(const cb_decode_attention_args& a, int g, int split, int splits, float* smem,
                               int* s_last, int tid) {
  attention_stage_cache<HD>(a, g, split, smem, tid);
  attn_sync();
  attention_finish<HD, kRegMerge>(a, g, split, splits, smem, s_last, tid, true);
}

}  // namespace cb

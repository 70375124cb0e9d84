// Single-token decode attention for one (context split, KV head) work item,
// shared by the standalone cb_decode_attention kernel and the decode-step
// megakernel.  256 threads (8 warps) execute it; `bar` synchronises them
// (named barrier 1) so it also runs inside a block that has extra warps.
//
// The item ropes the new q/k rows, stages its split's K/V rows in shared
// memory -- applying the write-mask blend cache*(1-wm) + new*wm (float32, as
// llama.py:511-512 computes it) to the rows it owns and writing them back --
// computes every (query head, position) score in one pass
// (x = q.k / divisor + mask), and writes its partial softmax state.  The last
// item of each KV group merges the splits in split order (deterministic) and
// resets the group counter.
#pragma once

#include "common.cuh"

namespace cb {

constexpr int kAttnThreads = 256;
constexpr int kAttnSplit = 32;

__device__ __forceinline__ void attn_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnThreads) : "memory");
}

// Shared floats the item needs.
__host__ __device__ inline long long attn_smem_floats(long long group, long long hd) {
  return (group + 2) * hd + kAttnSplit * (hd + 1) + kAttnSplit * hd + group * kAttnSplit + 2 * group;
}

template <int HD>
__device__ void attention_item(const cb_decode_attention_args& a, int g, int split, int splits, float* smem,
                               int* s_last, int tid) {
  const int group = static_cast<int>(a.heads / a.kv_heads);
  constexpr int half = HD / 2;
  constexpr int KS = HD + 1;
  float* q_rot = smem;
  float* k_new = q_rot + group * HD;
  float* v_new = k_new + HD;
  float* ks = v_new + HD;
  float* vs = ks + kAttnSplit * KS;
  float* probs = vs + kAttnSplit * HD;
  float* stats = probs + group * kAttnSplit;
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int warps = kAttnThreads / 32;

  long long pos = load_index(a.position, 0, a.position_dtype);
  if (pos < 0 || pos >= a.n_positions) {
    if (tid == 0 && split == 0 && a.error_flag != nullptr) atomicExch(a.error_flag, CB_FLAG_POSITION);
    pos = pos < 0 ? 0 : a.n_positions - 1;
  }
  const float* cs = a.cos_table + pos * half;
  const float* sn = a.sin_table + pos * half;
  for (int i = tid; i < group * half; i += kAttnThreads) {
    const int h = i / half, j = i % half;
    const float* src = a.qkv + a.q_off + (static_cast<long long>(g) * group + h) * HD;
    const float lo = __ldcg(src + j), hi = __ldcg(src + j + half), c = cs[j], s = sn[j];
    q_rot[h * HD + j] = fmaf(-hi, s, __fmul_rn(lo, c));
    q_rot[h * HD + j + half] = fmaf(hi, c, __fmul_rn(lo, s));
  }
  for (int j = tid; j < half; j += kAttnThreads) {
    const float* src = a.qkv + a.k_off + static_cast<long long>(g) * HD;
    const float lo = __ldcg(src + j), hi = __ldcg(src + j + half), c = cs[j], s = sn[j];
    k_new[j] = fmaf(-hi, s, __fmul_rn(lo, c));
    k_new[j + half] = fmaf(hi, c, __fmul_rn(lo, s));
  }
  for (int d = tid; d < HD; d += kAttnThreads)
    v_new[d] = __ldcg(a.qkv + a.v_off + static_cast<long long>(g) * HD + d);
  attn_sync();

  // stage this split's K/V rows; rows with wm != 0 get the blend
  const long long lo_pos = static_cast<long long>(split) * kAttnSplit;
  const int n = static_cast<int>(a.context - lo_pos < kAttnSplit ? a.context - lo_pos : kAttnSplit);
  float* kc = a.k_cache + (static_cast<long long>(g) * a.context + lo_pos) * HD;
  float* vc = a.v_cache + (static_cast<long long>(g) * a.context + lo_pos) * HD;
  for (int e = tid; e < n * (HD / 4); e += kAttnThreads) {
    const int r = e / (HD / 4), d4 = (e % (HD / 4)) * 4;
    float4 kv = __ldcg(reinterpret_cast<const float4*>(kc) + e);
    float4 vv = __ldcg(reinterpret_cast<const float4*>(vc) + e);
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
    kd[0] = kv.x;
    kd[1] = kv.y;
    kd[2] = kv.z;
    kd[3] = kv.w;
    *reinterpret_cast<float4*>(vs + r * HD + d4) = vv;
  }
  attn_sync();

  // scores: warp = query head (looping), lane = position
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
    probs[h * kAttnSplit + lane] = p;
    if (lane == 0) {
      stats[2 * h] = m;
      stats[2 * h + 1] = l;
    }
  }
  attn_sync();

  // p @ v for every (head, dim) of the group; partials to scratch
  for (int i = tid; i < group * HD; i += kAttnThreads) {
    const int h = i / HD, d = i % HD;
    const float* p = probs + h * kAttnSplit;
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

  // merge the splits of this KV group in split order
  __threadfence();
  attn_sync();
  if (tid == 0) {
    const unsigned ticket = atomicAdd(a.counters + g, 1u);
    *s_last = ticket == static_cast<unsigned>(splits - 1);
  }
  attn_sync();
  if (!*s_last) return;
  __threadfence();
  for (int i = tid; i < group * HD; i += kAttnThreads) {
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

}  // namespace cb

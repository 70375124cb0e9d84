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

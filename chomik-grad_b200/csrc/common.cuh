// Shared device helpers for libchomik_b200 (sm_100a only).
//
// Numerics: the library reproduces chomik-grad's NumPy/ml_dtypes semantics.
// Every value lives in float32 registers; a node whose runtime dtype is
// bfloat16 or float16 is rounded to that dtype (round-to-nearest-even) after
// each operation, exactly as ml_dtypes/NumPy store each op's result.  The
// library is built without fast-math so division and sqrt are IEEE-rounded.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "chomik_b200.h"

namespace cb {

// ---- error plumbing ------------------------------------------------------
void set_error(const char* fmt, ...);
int check_launch(const char* what);

#define CB_REQUIRE(cond, ...)            \
  do {                                    \
    if (!(cond)) {                        \
      ::cb::set_error(__VA_ARGS__);       \
      return CB_ERR_INVALID;              \
    }                                     \
  } while (0)

// ---- dtype conversion ----------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == CB_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == CB_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float load_as_f32(const void* base, long long i, int dtype) {
  switch (dtype) {
    case CB_F32: return static_cast<const float*>(base)[i];
    case CB_BF16: return bf16_bits_to_f32(static_cast<const uint16_t*>(base)[i]);
    case CB_F16: return __half2float(static_cast<const __half*>(base)[i]);
    case CB_I32: return static_cast<float>(static_cast<const int32_t*>(base)[i]);
    case CB_I64: return static_cast<float>(static_cast<const long long*>(base)[i]);
    default: return 0.0f;
  }
}

// load_as_f32 through L2 only (ld.global.cg): for values other blocks of the
// same launch wrote, which this SM's L1 may hold stale copies of.
__device__ __forceinline__ float load_cg_f32(const void* base, long long i, int dtype) {
  switch (dtype) {
    case CB_F32: return __ldcg(static_cast<const float*>(base) + i);
    case CB_BF16: return bf16_bits_to_f32(__ldcg(static_cast<const unsigned short*>(base) + i));
    case CB_F16: return __half2float(__ushort_as_half(__ldcg(static_cast<const unsigned short*>(base) + i)));
    case CB_I32: return static_cast<float>(__ldcg(static_cast<const int*>(base) + i));
    case CB_I64: return static_cast<float>(__ldcg(static_cast<const long long*>(base) + i));
    default: return 0.0f;
  }
}

__device__ __forceinline__ void store_from_f32(void* base, long long i, int dtype, float v) {
  switch (dtype) {
    case CB_F32: static_cast<float*>(base)[i] = v; break;
    case CB_BF16: static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v); break;
    case CB_F16: static_cast<__half*>(base)[i] = __float2half_rn(v); break;
    default: break;
  }
}

__device__ __forceinline__ long long load_index(const void* base, long long i, int dtype) {
  return dtype == CB_I64 ? static_cast<const long long*>(base)[i]
                         : static_cast<long long>(static_cast<const int32_t*>(base)[i]);
}

// Eight packed bf16 (one 16-byte load) -> eight floats.
__device__ __forceinline__ void unpack_bf16x8(const uint4& w, float* f) {
  f[0] = __uint_as_float(w.x << 16); f[1] = __uint_as_float(w.x & 0xffff0000u);
  f[2] = __uint_as_float(w.y << 16); f[3] = __uint_as_float(w.y & 0xffff0000u);
  f[4] = __uint_as_float(w.z << 16); f[5] = __uint_as_float(w.z & 0xffff0000u);
  f[6] = __uint_as_float(w.w << 16); f[7] = __uint_as_float(w.w & 0xffff0000u);
}

// ---- warp reductions -----------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// np.argmax order: NaN beats everything (first NaN wins), then larger value,
// ties go to the lower index.
__device__ __forceinline__ bool argmax_better(float av, long long ai, float bv, long long bi) {
  const bool an = av != av, bn = bv != bv;
  if (an || bn) {
    if (an && bn) return ai < bi;
    return an;
  }
  if (av != bv) return av > bv;
  return ai < bi;
}

// ---- programmatic dependent launch (PDL) ---------------------------------
// Kernels launched with the programmatic-serialization attribute may start
// before their predecessor finishes; they must wait before touching its
// outputs.  Both instructions are no-ops for ordinary launches.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Fire-and-forget prefetch of [p, p + bytes) into L2 (bytes: multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's 1/ncta share of up to three byte ranges, prefetched into L2 in
// 64 KiB pieces by threads t = 0..nt-1 of the caller.  Ranges must be 16-byte
// aligned; used to stream the NEXT kernel's weights while this one runs.
__device__ __forceinline__ void prefetch_share(const void* const* ptrs, const long long* bytes,
                                               long long cta, long long ncta, int t, int nt) {
  long long total = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i) total += ptrs[i] != nullptr ? bytes[i] : 0;
  if (total <= 0) return;
  const long long per = ((total + ncta - 1) / ncta + 15) & ~15LL;
  long long lo = cta * per, hi = lo + per < total ? lo + per : total;
  constexpr long long kPiece = 64 * 1024;
  long long seg_start = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (ptrs[i] == nullptr) continue;
    const long long seg_end = seg_start + bytes[i];
    const long long a = lo > seg_start ? lo : seg_start;
    const long long b = hi < seg_end ? hi : seg_end;
    for (long long p = a + t * kPiece; p < b; p += static_cast<long long>(nt) * kPiece) {
      const long long n = b - p < kPiece ? b - p : kPiece;
      const long long n16 = n & ~15LL;
      if (n16 > 0)
        prefetch_l2(static_cast<const char*>(ptrs[i]) + (p - seg_start), static_cast<uint32_t>(n16));
    }
    seg_start = seg_end;
  }
}

// Launch helper: optional PDL attribute on the given stream.
template <typename Kernel, typename... Args>
inline cudaError_t launch(Kernel kernel, dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int sm_count();

}  // namespace cb

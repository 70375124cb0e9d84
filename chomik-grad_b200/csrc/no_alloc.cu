// Decode attention that allocates nothing: cb_decode_attention_noalloc.
//
// Who needs it.  cb_decode_attention wants a caller-owned scratch buffer
// (split partials) and a zeroed counter array.  Some callers cannot provide
// them:
//  * a host that binds this library through an FFI and only owns the arrays
//    of the graph it runs -- the compiled-program contract hands a backend
//    the bound inputs and outputs and nothing else, so a one-call-per-op
//    binding has no place to keep per-op scratch;
//  * a serving process that gives the whole device to a fixed arena at
//    start-up (weights, then a KV cache sized to the remaining HBM), where a
//    later cudaMalloc fails or needs a second allocator;
//  * a latency-bound decode loop, where cudaFree (and often cudaMalloc)
//    synchronises the device.
// For them the scratch lives in this file's fixed device arrays instead.
//
// Set-up.  The first call on a device (with that device current) looks up
// the arrays' addresses with cudaGetSymbolAddress and clears the counters
// with a synchronous cudaMemset + cudaDeviceSynchronize.  Make that first
// call before any stream capture on the device.  Later calls only launch.
//
// Limits.  splits * heads * (head_size + 2) floats of partials (splits =
// ceil(context / 32)) must fit kScratchFloats (1 Mi floats, 4 MiB), and kv_heads must not
// exceed kMaxKvHeads; larger requests are rejected before any launch.
//
// Sharing.  One scratch area per device serves every call: calls that
// overlap on the GPU (unordered streams, concurrent graph replays) race on
// it and give wrong results.  Calls ordered on one stream are safe; each
// call leaves the counters at zero for the next.
#include <mutex>

#include "attn_core.cuh"

namespace cb {
namespace {

constexpr long long kScratchFloats = 1LL << 20;  // 1 Mi floats (4 MiB) of split partials
constexpr int kMaxKvHeads = 256;
constexpr int kMaxDevices = 64;

// Zero at module load; cleared again at set-up.
static __device__ __align__(256) float g_scratch[kScratchFloats];
static __device__ __align__(256) unsigned int g_counters[kMaxKvHeads];

struct DeviceScratch {
  float* scratch = nullptr;
  unsigned int* counters = nullptr;
  bool ready = false;
};
std::mutex g_setup_mutex;
DeviceScratch g_devices[kMaxDevices];

// Once per device, with the device current: symbol addresses + zeroed counters.
int device_scratch(DeviceScratch* out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    set_error("decode attention (no-alloc): cudaGetDevice: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  CB_REQUIRE(device >= 0 && device < kMaxDevices, "decode attention (no-alloc): device %d beyond %d", device,
             kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceScratch& d = g_devices[device];
  if (!d.ready) {
    void* scratch = nullptr;
    void* counters = nullptr;
    e = cudaGetSymbolAddress(&scratch, g_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&counters, g_counters);
    if (e == cudaSuccess) e = cudaMemset(counters, 0, sizeof(g_counters));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      set_error("decode attention (no-alloc): scratch set-up on device %d: %s", device, cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
    d.scratch = static_cast<float*>(scratch);
    d.counters = static_cast<unsigned int*>(counters);
    d.ready = true;
  }
  *out = d;
  return CB_OK;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) decode_attention_noalloc_kernel(const cb_decode_attention_args a) {
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

int cb_decode_attention_noalloc(const cb_decode_attention_args* args, cb_stream_t stream) {
  CB_REQUIRE(args != nullptr, "decode attention (no-alloc): null args");
  const cb_decode_attention_args& a = *args;
  CB_REQUIRE(a.head_size == 32 || a.head_size == 64 || a.head_size == 128 || a.head_size == 256,
             "decode attention (no-alloc): head size %lld unsupported (32/64/128/256)", a.head_size);
  CB_REQUIRE(a.heads > 0 && a.kv_heads > 0 && a.heads % a.kv_heads == 0,
             "decode attention (no-alloc): bad head grouping");
  CB_REQUIRE(a.context > 0, "decode attention (no-alloc): empty context");
  CB_REQUIRE(a.kv_dtype == CB_F32 || a.kv_dtype == CB_BF16,
             "decode attention (no-alloc): caches must be float32 or bfloat16");
  CB_REQUIRE(a.mask != nullptr && a.write_mask != nullptr && a.position != nullptr,
             "decode attention (no-alloc): mask, write mask and position are required");
  CB_REQUIRE(a.split == 0 || a.split == kAttnSplit, "decode attention (no-alloc): split must be %d", kAttnSplit);
  const long long splits = (a.context + kAttnSplit - 1) / kAttnSplit;
  CB_REQUIRE(a.kv_heads <= kMaxKvHeads, "decode attention (no-alloc): %lld KV heads exceed the limit of %d",
             a.kv_heads, kMaxKvHeads);
  CB_REQUIRE(splits <= kScratchFloats / (a.heads * (a.head_size + 2)),
             "decode attention (no-alloc): context %lld x %lld heads x head size %lld needs %lld scratch floats, "
             "limit %lld",
             a.context, a.heads, a.head_size, splits * a.heads * (a.head_size + 2), kScratchFloats);
  const long long group = a.heads / a.kv_heads;
  const size_t smem = static_cast<size_t>(attn_smem_floats(group, a.head_size)) * sizeof(float);
  CB_REQUIRE(smem <= 200 * 1024, "decode attention (no-alloc): too many query heads per KV head");

  DeviceScratch d;
  const int status = device_scratch(&d);
  if (status != CB_OK) return status;
  cb_decode_attention_args k = a;
  k.scratch = d.scratch;
  k.counters = d.counters;

  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(a.kv_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define CB_NOALLOC_CASE(HD)                                                                                \
  case HD:                                                                                                 \
    e = cudaFuncSetAttribute(decode_attention_noalloc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             static_cast<int>(smem));                                                      \
    if (e == cudaSuccess) e = launch(decode_attention_noalloc_kernel<HD>, grid, dim3(kAttnThreads), smem, s, \
                                     a.pdl != 0, k);                                                       \
    break;
  switch (a.head_size) {
    CB_NOALLOC_CASE(32)
    CB_NOALLOC_CASE(64)
    CB_NOALLOC_CASE(128)
    CB_NOALLOC_CASE(256)
  }
#undef CB_NOALLOC_CASE
  if (e != cudaSuccess) {
    set_error("cb_decode_attention_noalloc: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return check_launch("cb_decode_attention_noalloc");
}

}  // extern "C"

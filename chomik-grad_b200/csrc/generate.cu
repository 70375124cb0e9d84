// On-device greedy decode driver: advances the per-step inputs of a decode
// program (token ids, position, attention mask, cache write mask) from the
// previous step's argmax, so K decode steps can be replayed back to back
// without a host round trip per token.  It writes exactly what the host loop
// of generate_tinyllama.py:772-786 builds for the next step.
#include "common.cuh"

namespace cb {
namespace {

// One block; thread b < rows advances sequence b (all sequences share the
// position and masks, written by thread 0).
__global__ void decode_advance_kernel(const long long* argmax, long long rows, void* ids, int ids_dtype,
                                      void* position, int position_dtype, void* mask, int mask_dtype,
                                      void* write_mask, int write_mask_dtype, long long context,
                                      long long* token_log, long long step, int* error_flag) {
  const long long pos = load_index(position, 0, position_dtype);
  const long long next = pos + 1;
  const bool past = next >= context || pos < 0;
  __syncthreads();  // every thread has read the position before thread 0 moves it
  for (long long b = threadIdx.x; b < rows; b += blockDim.x) {
    const long long token = argmax[b];
    if (token_log != nullptr) token_log[step * rows + b] = token;
    if (past) continue;
    if (ids_dtype == CB_I64) static_cast<long long*>(ids)[b] = token;
    else static_cast<int32_t*>(ids)[b] = static_cast<int32_t>(token);
  }
  if (threadIdx.x != 0) return;
  if (past) {
    if (error_flag != nullptr) atomicExch(error_flag, CB_FLAG_CONTEXT);
    return;
  }
  if (position_dtype == CB_I64) static_cast<long long*>(position)[0] = next;
  else static_cast<int32_t*>(position)[0] = static_cast<int32_t>(next);
  store_from_f32(mask, next, mask_dtype, 0.0f);
  store_from_f32(write_mask, pos, write_mask_dtype, 0.0f);
  store_from_f32(write_mask, next, write_mask_dtype, 1.0f);
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_decode_advance(const long long* argmax, void* ids, int ids_dtype, void* position,
                                 int position_dtype, void* mask, int mask_dtype, void* write_mask,
                                 int write_mask_dtype, long long context, long long* token_log,
                                 long long step, int* error_flag, cb_stream_t stream) {
  CB_REQUIRE(ids_dtype == CB_I32 || ids_dtype == CB_I64, "decode advance: ids must be int32/int64");
  CB_REQUIRE(position_dtype == CB_I32 || position_dtype == CB_I64, "decode advance: bad position dtype");
  decode_advance_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      argmax, 1, ids, ids_dtype, position, position_dtype, mask, mask_dtype, write_mask, write_mask_dtype,
      context, token_log, step, error_flag);
  return check_launch("cb_decode_advance");
}

extern "C" int cb_decode_advance_rows(const long long* argmax, long long rows, void* ids, int ids_dtype,
                                      void* position, int position_dtype, void* mask, int mask_dtype,
                                      void* write_mask, int write_mask_dtype, long long context,
                                      long long* token_log, long long step, int* error_flag, cb_stream_t stream) {
  CB_REQUIRE(rows >= 1, "decode advance: rows must be positive");
  CB_REQUIRE(ids_dtype == CB_I32 || ids_dtype == CB_I64, "decode advance: ids must be int32/int64");
  CB_REQUIRE(position_dtype == CB_I32 || position_dtype == CB_I64, "decode advance: bad position dtype");
  decode_advance_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      argmax, rows, ids, ids_dtype, position, position_dtype, mask, mask_dtype, write_mask, write_mask_dtype,
      context, token_log, step, error_flag);
  return check_launch("cb_decode_advance_rows");
}

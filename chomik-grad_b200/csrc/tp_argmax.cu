// Greedy argmax over a vocabulary-sharded lm_head (tensor parallel).
//
// Each rank holds vocab / ranks consecutive rows of the lm_head, so its
// logits are columns [col_offset, col_offset + width) of every row.  Instead
// of gathering the whole (rows, vocab) logits, every rank reduces its columns
// to one 16-byte record per row -- (value, global index) of its winner -- the
// group all-gathers those records (NCCL, on the caller's stream), and every
// rank picks the same winner from them.  The order is np.argmax's over the
// whole row (chomikgrad/lazy.py:128-134): a NaN first, then the larger
// value, then the lower index.  A rank's record is the first maximum of its
// own columns, and the columns of the ranks are disjoint, so the pick over
// the records equals the argmax over the gathered row.
#include "common.cuh"

namespace cb {
namespace {

constexpr int kArgmaxThreads = 512;

struct alignas(16) ArgmaxRecord {
  float value;
  int valid;
  long long index;  // global column
};
static_assert(sizeof(ArgmaxRecord) == 16, "records travel as four float32 words");

__global__ void __launch_bounds__(kArgmaxThreads) argmax_partial_kernel(const void* x, int dtype, long long width,
                                                                        long long col_offset, ArgmaxRecord* out) {
  __shared__ float best_v[kArgmaxThreads / 32];
  __shared__ long long best_i[kArgmaxThreads / 32];
  const long long row = blockIdx.x;
  float bv = 0.0f;
  long long bi = -1;
  for (long long j = threadIdx.x; j < width; j += blockDim.x) {
    const float v = load_as_f32(x, row * width + j, dtype);
    if (bi < 0 || argmax_better(v, j, bv, bi)) {
      bv = v;
      bi = j;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, off);
    const long long oi = __shfl_down_sync(0xffffffffu, bi, off);
    if (oi >= 0 && (bi < 0 || argmax_better(ov, oi, bv, bi))) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    best_v[warp] = bv;
    best_i[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bv = 0.0f;
    bi = -1;
    for (int w = 0; w < kArgmaxThreads / 32; ++w) {
      if (best_i[w] >= 0 && (bi < 0 || argmax_better(best_v[w], best_i[w], bv, bi))) {
        bv = best_v[w];
        bi = best_i[w];
      }
    }
    ArgmaxRecord r;
    r.value = bv;
    r.valid = 1;
    r.index = col_offset + bi;
    out[row] = r;
  }
}

// records: [ranks][rows], rank after rank (the all-gather's layout).
__global__ void argmax_pick_kernel(const ArgmaxRecord* records, int ranks, long long rows, long long* out) {
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float bv = 0.0f;
  long long bi = -1;
  for (int r = 0; r < ranks; ++r) {
    const ArgmaxRecord c = records[static_cast<long long>(r) * rows + row];
    if (c.valid && (bi < 0 || argmax_better(c.value, c.index, bv, bi))) {
      bv = c.value;
      bi = c.index;
    }
  }
  out[row] = bi < 0 ? 0 : bi;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cb_argmax_rows_partial(const void* x, int dtype, long long rows, long long width, long long col_offset,
                           void* records, cb_stream_t stream) {
  CB_REQUIRE(width > 0, "attempt to get argmax of an empty sequence");
  CB_REQUIRE(col_offset >= 0, "argmax partial: negative column offset");
  CB_REQUIRE(dtype == CB_F32 || dtype == CB_BF16 || dtype == CB_F16, "argmax partial: float logits only");
  if (rows == 0) return CB_OK;
  CB_REQUIRE(rows < (1LL << 31), "argmax partial: too many rows");
  CB_REQUIRE(x != nullptr && records != nullptr, "argmax partial: null pointer");
  CB_REQUIRE((reinterpret_cast<uintptr_t>(records) & 15) == 0, "argmax partial: records must be 16-byte aligned");
  argmax_partial_kernel<<<static_cast<unsigned>(rows), kArgmaxThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, dtype, width, col_offset, static_cast<ArgmaxRecord*>(records));
  return check_launch("cb_argmax_rows_partial");
}

int cb_argmax_pick(const void* records, int ranks, long long rows, long long* out_index, cb_stream_t stream) {
  CB_REQUIRE(ranks >= 1, "argmax pick: %d ranks", ranks);
  if (rows == 0) return CB_OK;
  CB_REQUIRE(rows < (1LL << 31), "argmax pick: too many rows");
  CB_REQUIRE(records != nullptr && out_index != nullptr, "argmax pick: null pointer");
  CB_REQUIRE((reinterpret_cast<uintptr_t>(records) & 15) == 0, "argmax pick: records must be 16-byte aligned");
  argmax_pick_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const ArgmaxRecord*>(records), ranks, rows, out_index);
  return check_launch("cb_argmax_pick");
}

int cb_argmax_rows_sharded(void* comm, int ranks, const void* x, int dtype, long long rows, long long width,
                           long long col_offset, void* scratch, long long* out_index, cb_stream_t stream) {
  CB_REQUIRE(width > 0, "attempt to get argmax of an empty sequence");
  CB_REQUIRE(ranks >= 1, "sharded argmax: %d ranks", ranks);
  CB_REQUIRE(col_offset >= 0, "sharded argmax: negative column offset");
  CB_REQUIRE(dtype == CB_F32 || dtype == CB_BF16 || dtype == CB_F16, "sharded argmax: float logits only");
  if (rows == 0) return CB_OK;
  CB_REQUIRE(rows < (1LL << 31), "sharded argmax: too many rows");
  CB_REQUIRE(x != nullptr && scratch != nullptr && out_index != nullptr, "sharded argmax: null pointer");
  CB_REQUIRE((reinterpret_cast<uintptr_t>(scratch) & 15) == 0, "sharded argmax: scratch must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ArgmaxRecord* local = static_cast<ArgmaxRecord*>(scratch);
  ArgmaxRecord* gathered = local + rows;
  int r = cb_argmax_rows_partial(x, dtype, rows, width, col_offset, local, stream);
  if (r != CB_OK) return r;
  if (ranks == 1) {
    if (cudaMemcpyAsync(gathered, local, static_cast<size_t>(rows) * sizeof(ArgmaxRecord), cudaMemcpyDeviceToDevice,
                        s) != cudaSuccess)
      return check_launch("cb_argmax_rows_sharded (copy)");
  } else {
    CB_REQUIRE(comm != nullptr, "sharded argmax: %d ranks need a communicator", ranks);
    r = cb_all_gather(comm, local, gathered, rows * static_cast<long long>(sizeof(ArgmaxRecord) / 4), CB_F32,
                      stream);
  }
  if (r != CB_OK) return r;
  return cb_argmax_pick(gathered, ranks, rows, out_index, stream);
}

}  // extern "C"

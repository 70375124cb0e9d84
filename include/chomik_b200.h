/*
 * chomik_b200.h -- C ABI of libchomik_b200.so, the sm_100a kernel library
 * behind chomik-grad's `cuda-b200` compiler plugin.
 *
 * Everything here takes raw device pointers, element counts/strides, a dtype
 * code and a cudaStream_t (passed as void*), and returns an int status:
 * CB_OK (0) or an error code whose text is available from cb_last_error().
 * No function allocates device memory; callers own every buffer.
 *
 * Each entry point replaces the reference behaviour cited beside it (paths
 * are inside the chomik-grad project).  The reference runs these operations
 * through its NumPy `cpu` compiler (chomikgrad/lazy.py:609-636) or CuPy
 * (chomikgrad/cuda_backend.py:619-701); the Python plugin in
 * cuda_b200/program.py binds these symbols with ctypes.
 */
#ifndef CHOMIK_B200_H
#define CHOMIK_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes: float32, bfloat16, float16, int32, int64 */
enum { CB_F32 = 0, CB_BF16 = 1, CB_F16 = 2, CB_I32 = 3, CB_I64 = 4 };

/* status codes */
enum { CB_OK = 0, CB_ERR_INVALID = 1, CB_ERR_CUDA = 2 };

/* values kernels store in an `error_flag` (0 = no error): an index outside
 * its table, a RoPE position outside the table, a decode step past the
 * context, bounded waits that gave up (a consumer waiting for data, a
 * producer waiting for a free slot, the end-of-kernel drain of copies), and a
 * sampled row whose probabilities are NaN */
enum {
  CB_FLAG_INDEX = 1,
  CB_FLAG_POSITION = 2,
  CB_FLAG_CONTEXT = 3,
  CB_FLAG_WAIT_DATA = 4,
  CB_FLAG_WAIT_SLOT = 5,
  CB_FLAG_WAIT_DRAIN = 6,
  CB_FLAG_WAIT_PHASE = 7, /* cb_decode_step: a block waiting for the previous phase */
  CB_FLAG_NAN = 8,        /* cb_sample_rows: NaN probabilities */
  CB_FLAG_WAIT_PEER = 9   /* cb_peer_all_reduce: a rank of the group did not arrive in time */
};

#define CB_MAX_DIMS 8
#define CB_EW_MAX_INPUTS 8
#define CB_EW_MAX_INSTR 40
#define CB_MM_MAX_BATCH 6

typedef void* cb_stream_t; /* cudaStream_t */

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

/* ---- library / runtime --------------------------------------------------*/
CB_API int cb_abi_version(void);
/* Text of the last error raised on the calling thread ("" if none). */
CB_API const char* cb_last_error(void);
/* Number of streaming multiprocessors of the current device. */
CB_API int cb_sm_count(int* count);

/* Stream-capture helpers for CUDA-graph replay of a compiled program.
 * Replaces the per-node Python dispatch of build_python_program's generated
 * `run` (chomikgrad/lazy.py:389-499; CUDAProgram.run cuda_backend.py:55-69). */
CB_API int cb_stream_create(cb_stream_t* stream);
CB_API int cb_stream_destroy(cb_stream_t stream);
CB_API int cb_capture_begin(cb_stream_t stream);
CB_API int cb_capture_end(cb_stream_t stream, void** graph_exec);
CB_API int cb_graph_launch(void* graph_exec, cb_stream_t stream);
CB_API int cb_graph_destroy(void* graph_exec);

/* ---- ELEMENTWISE ---------------------------------------------------------
 * Fused elementwise expression over a broadcast output shape.
 * Replaces NumpyCompiler._BINARY/_UNARY (chomikgrad/lazy.py:554-568) and the
 * CuPy fused elementwise kernel (chomikgrad/cuda_backend.py:703-748).
 * Register r < n_inputs is input r (converted to float32); register
 * n_inputs + i is the result of instruction i, rounded to round[i]'s dtype
 * (CB_F32 = no rounding).  The output is the last instruction's register
 * (or input 0 when n_instr == 0), stored contiguously as out_dtype. */
enum {
  CB_OP_ADD = 0, CB_OP_SUB = 1, CB_OP_MUL = 2, CB_OP_DIV = 3, CB_OP_EQUAL = 4,
  CB_OP_NEG = 5, CB_OP_EXP = 6, CB_OP_LOG = 7, CB_OP_SQRT = 8, CB_OP_RELU = 9,
  CB_OP_STEP = 10
};
typedef struct {
  int ndim;
  int n_inputs;
  int n_instr;
  int out_dtype;
  long long shape[CB_MAX_DIMS];
  const void* inputs[CB_EW_MAX_INPUTS];
  int in_dtype[CB_EW_MAX_INPUTS];
  long long in_strides[CB_EW_MAX_INPUTS][CB_MAX_DIMS]; /* elements; 0 = broadcast */
  long long in_offset[CB_EW_MAX_INPUTS];
  int op[CB_EW_MAX_INSTR];
  int lhs[CB_EW_MAX_INSTR];
  int rhs[CB_EW_MAX_INSTR];
  int round[CB_EW_MAX_INSTR];
  void* out;
} cb_elementwise_args;
CB_API int cb_elementwise(const cb_elementwise_args* args, cb_stream_t stream);

/* ---- REDUCE --------------------------------------------------------------
 * sum / max over `red` dims for every element of the `keep` dims.
 * Replaces np.sum / np.max(axis, keepdims) (chomikgrad/lazy.py:618-622).
 * sequential != 0 accumulates in index order rounding to acc_dtype after each
 * add -- NumPy's loop for bfloat16/float16 data; otherwise a tree order. */
enum { CB_REDUCE_SUM = 0, CB_REDUCE_MAX = 1 };
typedef struct {
  const void* in;
  int in_dtype;
  void* out; /* contiguous over keep dims */
  int out_dtype;
  int kind;
  int sequential;
  int acc_dtype;
  int n_keep;
  int n_red;
  long long in_offset;
  long long keep_shape[CB_MAX_DIMS];
  long long keep_strides[CB_MAX_DIMS];
  long long red_shape[CB_MAX_DIMS];
  long long red_strides[CB_MAX_DIMS];
} cb_reduce_args;
CB_API int cb_reduce(const cb_reduce_args* args, cb_stream_t stream);

/* ---- RESHAPE / PERMUTE materialisation -----------------------------------
 * out (contiguous) <- strided view of `in`; elem_bytes in {1,2,4,8}.
 * Replaces the copies np.reshape/np.transpose make for non-viewable layouts
 * (chomikgrad/lazy.py:624-628). */
CB_API int cb_copy_strided(const void* in, long long in_offset, void* out, int elem_bytes, int ndim,
                    const long long* shape, const long long* in_strides, cb_stream_t stream);

/* ---- MATMUL by a placement matrix ------------------------------------------
 * out (rows x n, contiguous) where out[r, j] = in[r, cols[j]], or 0 where
 * cols[j] < 0; `in` is a strided view whose last dimension (the contracted
 * one) has length shape[ndim-1] and whose leading dimensions give the rows.
 * This is `x @ P` for a constant 0/1 matrix P with one 1 per row and at most
 * one per column: the KV-cache placement of the prefill
 * (chomikgrad/llama.py:243-247, 411-418).  Each output is one input times 1
 * plus zeros, so the copy is the product exactly; values convert from
 * in_dtype to out_dtype. */
CB_API int cb_place_columns(const void* in, int in_dtype, int ndim, const long long* shape,
                            const long long* in_strides, const int* cols, long long n, void* out, int out_dtype,
                            cb_stream_t stream);

/* ---- KV-cache write mask, in place -----------------------------------------
 * cache (batch, heads, ctx, head_size) float32 contiguous becomes
 * cache * (1 - wm) + row * wm for the decode write mask wm (ctx values) and
 * the new rows `row` (batch, heads, 1, head_size; element strides
 * row_strides[4]): the blend of chomikgrad/llama.py:511-512.  1 - wm is
 * rounded to one_minus_dtype (the dtype the graph computes it in); products
 * and sum are float32.  Only rows with wm != 0 are rewritten: at wm == 0 the
 * blend is cache * 1 + row * 0, the cache itself for finite rows. */
CB_API int cb_kv_write(float* cache, long long batch, long long heads, long long ctx, long long head_size,
                       const void* row, int row_dtype, const long long* row_strides, const void* write_mask,
                       int write_mask_dtype, int one_minus_dtype, cb_stream_t stream);

/* ---- GATHER --------------------------------------------------------------
 * out[i, :] = table[idx[i], :] (rows of row_bytes bytes); negative indices
 * wrap once, out-of-range indices set *error_flag = 1 and write zeros.
 * Replaces np.take(table, idx, axis=0) (chomikgrad/lazy.py:633-634) and
 * cp.take (chomikgrad/cuda_backend.py:699-700). */
CB_API int cb_gather(const void* table, long long rows, long long row_bytes, const void* idx,
              int idx_dtype, long long n, void* out, int* error_flag, cb_stream_t stream);

/* ---- MATMUL --------------------------------------------------------------
 * Batched, broadcast C = A @ B with float32 accumulation; C contiguous
 * (batch..., m, n).  bf16 @ bf16 returns float32 like ml_dtypes.
 * Replaces np.matmul (chomikgrad/lazy.py:630-631) and cp.matmul/cuBLAS
 * (chomikgrad/cuda_backend.py:678-698). */
typedef struct {
  const void* a;
  int a_dtype;
  const void* b;
  int b_dtype;
  void* c;
  int c_dtype;
  long long m, n, k;
  long long a_offset, b_offset;
  long long a_rs, a_cs, b_rs, b_cs; /* element strides of the matrix dims */
  int batch_ndim;
  long long batch_shape[CB_MM_MAX_BATCH];
  long long a_bstride[CB_MM_MAX_BATCH];
  long long b_bstride[CB_MM_MAX_BATCH];
} cb_matmul_args;
CB_API int cb_matmul(const cb_matmul_args* args, cb_stream_t stream);

/* ---- rms_norm lowering ---------------------------------------------------
 * out = x / sqrt(sum(x*x)/divisor + eps) * w per row, each op rounded to the
 * dtype the reference graph gives it (dt_*), with a sequential sum when the
 * square is bf16/f16.  divisor and eps are the values of the graph's constant
 * leaves.  Replaces LlamaForCausalLM._rms_norm's portable chain
 * (chomikgrad/llama.py:279-287; MLX lowering mlx_backend.py:410-414).
 * With d_table != NULL the per-row sqrt term is read from d_table[d_index[r]]
 * (see cb_rmsnorm_row_table). */
typedef struct {
  const void* x;
  int x_dtype;
  long long rows, width, x_row_stride, x_offset;
  const void* x_index; /* optional: row r reads x row x_index[r] */
  int x_index_dtype;
  const void* w;
  int w_dtype;
  void* out;
  int out_dtype;
  float divisor, eps;
  int dt_sq, dt_sum, dt_mean, dt_t, dt_d, dt_y;
  const float* d_table;
} cb_rmsnorm_args;
CB_API int cb_rmsnorm(const cb_rmsnorm_args* args, cb_stream_t stream);
/* d_out[r] = rounded sqrt(mean(x_r^2) + eps) for each row of a constant
 * table, so that rms_norm(gather(table, ids)) costs a lookup at decode time. */
CB_API int cb_rmsnorm_row_table(const cb_rmsnorm_args* args, float* d_out, cb_stream_t stream);

/* ---- rope lowering -------------------------------------------------------
 * Rotate-half RoPE of x (B, H, T, hd) with cos/sin rows already rounded to the
 * rotation matrix dtype: out_j = x_j c_j - x_{j+h} s_j, out_{j+h} =
 * x_j s_j + x_{j+h} c_j.  Table layout [n_offsets][T][hd/2]; the offset is
 * read from a device scalar (NULL = 0).  Replaces the dense rotation matmul of
 * LlamaForCausalLM._apply_rope/_apply_rotation (chomikgrad/llama.py:293-323)
 * and its table _rope_rotations (:127-152). */
typedef struct {
  const void* x;
  int x_dtype;
  long long x_offset;
  long long x_strides[4];
  void* out; /* contiguous (B, H, T, hd) */
  int out_dtype;
  long long batch, heads, tokens, head_size;
  const float* cos_table;
  const float* sin_table;
  long long n_offsets;
  const void* offset;
  int offset_dtype;
  int* error_flag;
} cb_rope_args;
CB_API int cb_rope(const cb_rope_args* args, cb_stream_t stream);

/* ---- sdpa lowering -------------------------------------------------------
 * softmax((q @ k^T) / divisor + mask) @ v with grouped KV heads, float32
 * accumulation, online softmax.  q (B,H,Tq,D), k/v (B,Hkv,Tk,D), mask
 * broadcast to (B,H,Tq,Tk) via strides (mask == NULL: none); out contiguous
 * (B,H,Tq,D) float32.  Replaces the portable attention of
 * chomikgrad/llama.py:355-364 / :514-525 (repeat_kv :325-330, softmax
 * chomikgrad/tensor.py:325-334; MLX lowering mlx_backend.py:423-428). */
typedef struct {
  const void* q;
  int q_dtype;
  long long q_offset, q_strides[4];
  const void* k;
  int k_dtype;
  long long k_offset, k_strides[4];
  const void* v;
  int v_dtype;
  long long v_offset, v_strides[4];
  const void* mask;
  int mask_dtype;
  long long mask_offset, mask_strides[4];
  float* out;
  long long batch, heads, kv_heads, tq, tk, head_size;
  float divisor;
  /* element strides of out over (B, H, Tq, D); all 0 = contiguous.  D's
   * stride must be 1 (e.g. token-major (B, Tq, H, D) rows: {Tq*H*D, D, H*D, 1}) */
  long long out_strides[4];
} cb_sdpa_args;
CB_API int cb_sdpa(const cb_sdpa_args* args, cb_stream_t stream);

/* Single-query form of cb_sdpa (tq == 1): the attention of a batched decode
 * step, where each sequence's new query attends over its own cache
 * (chomikgrad/llama.py:514-525 -- scores, softmax, p @ v -- once per
 * sequence).  K/V float32 with contiguous, 16-byte aligned rows; q and mask
 * any dtype and strides.  Split over keys (32 per block) with a second pass
 * that merges the splits of each (batch, head) in split order
 * (deterministic).  `scratch`: cb_sdpa_query_scratch bytes, 16-byte aligned. */
CB_API long long cb_sdpa_query_scratch(const cb_sdpa_args* args);
CB_API int cb_sdpa_query(const cb_sdpa_args* args, void* scratch, cb_stream_t stream);

/* Tensor-core (tcgen05) form of cb_sdpa for prefill and verify blocks: the
 * same softmax(q k^T / divisor + mask) v (chomikgrad/llama.py:332-369,
 * tensor.py:325-334) with q, k, v split into bf16 hi/lo planes (three MMA
 * products per product of the reference, float32 accumulation and softmax).
 * head_size 64 or 128; out (batch, heads, tq, head_size) contiguous and
 * 16-byte aligned.  `causal` flags: CB_CAUSAL_SKIP asserts mask <= -5000 at
 * every key j > i + (tk - tq), whose key tiles are then skipped (their terms
 * are exact zeros of the float32 softmax); CB_CAUSAL_ZERO_BELOW (with SKIP)
 * asserts the mask is exactly 0 at every other key, so it is read only on
 * diagonal tiles.  `scratch`: cb_sdpa_tc_scratch bytes, 16-byte aligned.  A
 * bounded wait that gives up sets *error_flag (CB_FLAG_WAIT_*). */
enum { CB_CAUSAL_SKIP = 1, CB_CAUSAL_ZERO_BELOW = 2 };
CB_API long long cb_sdpa_tc_scratch(const cb_sdpa_args* args);
CB_API int cb_sdpa_tc(const cb_sdpa_args* args, int causal, void* scratch, int* error_flag, cb_stream_t stream);

/* ---- decode hot path -----------------------------------------------------*/

/* Streaming GEMV y = x W^T for one token, W in HF (out, in) row-major layout,
 * with an optional fused rms_norm prologue and a fused epilogue.  Up to three
 * weight matrices are processed as one logical matrix (rows concatenated),
 * e.g. q/k/v or gate/up.  Replaces the decode MATMULs of
 * LlamaForCausalLM._linear (chomikgrad/llama.py:275-277) plus the fused
 * chains that follow them: residual add (:529-535), SwiGLU silu(gate)*up
 * (:289-291, :371-380), and greedy argmax of the logits (DeviceAdapter.argmax,
 * chomikgrad/lazy.py:128-129; cuda_backend.py:37-38).
 * Scratch (argmax epilogue): scratch_val/scratch_idx hold one entry per CTA
 * and *counter must be 0 before the first launch (the kernel leaves it 0). */
enum { CB_NORM_NONE = 0, CB_NORM_RMS = 1, CB_NORM_RMS_TABLE = 2 };
enum { CB_EPI_STORE = 0, CB_EPI_RESIDUAL = 1, CB_EPI_SILU_MUL = 2, CB_EPI_ARGMAX = 3 };
typedef struct {
  const void* w[3];
  long long w_rows[3];
  int n_w;
  int w_dtype;
  long long k;
  const void* x;
  int x_dtype;
  const void* x_index; /* optional: x row = x + x_index[0] * k */
  int x_index_dtype;
  long long index_rows; /* rows of the tables x_index/residual_index select from */
  int* error_flag;      /* set to 1 (and row 0 used) when an index is out of range */
  int norm;
  const void* norm_w;
  int norm_w_dtype;
  float divisor, eps;
  int dt_sq, dt_sum, dt_mean, dt_t, dt_d, dt_y;
  int dt_norm_out;         /* dtype of the rms_norm output row */
  const float* norm_table; /* CB_NORM_RMS_TABLE: d per x_index row */
  int epilogue;
  const void* residual;
  int residual_dtype;
  const void* residual_index; /* optional: residual row = residual + idx * n_out */
  int residual_index_dtype;
  float* out;
  float* scratch_val;
  long long* scratch_idx;
  unsigned int* counter;
  long long* argmax_out;
  /* L2 prefetch of the NEXT kernel's weights, shared across this grid's
   * CTAs (16-byte aligned ranges; NULL = none). */
  const void* prefetch_ptr[3];
  long long prefetch_bytes[3];
  int grid; /* 0 = library default */
  int pdl;  /* launch with programmatic dependent launch */
} cb_gemv_args;
CB_API int cb_gemv(const cb_gemv_args* args, cb_stream_t stream);
/* CTAs cb_gemv launches for these args (size of the argmax scratch). */
CB_API int cb_gemv_grid(const cb_gemv_args* args, int* grid);

/* Single-token GQA attention over the bound KV cache, fused with RoPE of the
 * new q/k rows and the in-place cache update.  Replaces, per decode layer,
 * _apply_rotation for q and k (chomikgrad/llama.py:509-510), the write-mask
 * blend cache*(1-wm) + key*wm (:511-512), repeat_kv + masked softmax
 * attention (:514-525).  Rows r with wm[r] != 0 are rewritten with the
 * blend's float32 arithmetic; every other row is left untouched.
 * Split-K over the context; partials in `scratch` (splits * heads * (hd + 2)
 * floats) are combined by the last CTA of each KV group, which resets
 * counters[g] to 0 (counters must be 0 before the first launch). */
typedef struct {
  const float* qkv; /* raw q | k | v projections, float32 */
  long long q_off, k_off, v_off;
  long long heads, kv_heads, head_size, context;
  const void* position;
  int position_dtype;
  const float* cos_table; /* [n_positions][hd/2] */
  const float* sin_table;
  long long n_positions;
  void* k_cache; /* (kv_heads, context, hd) of kv_dtype, updated in place */
  void* v_cache;
  const void* write_mask; /* context values */
  int write_mask_dtype;
  int one_minus_dtype; /* dtype of (1 - write_mask) in the graph */
  const void* mask; /* additive attention mask, context values */
  int mask_dtype;
  float divisor;
  float* out; /* heads * hd float32 */
  float* scratch;
  unsigned int* counters; /* kv_heads */
  int* error_flag;
  const void* prefetch_ptr[3]; /* next kernel's weights, see cb_gemv_args */
  long long prefetch_bytes[3];
  int split; /* positions per CTA (0 = default) */
  int pdl;
  /* CB_F32 (0) or CB_BF16: the caches' element type.  A bfloat16 cache is
   * read as float32 values; the rows the write mask rewrites are blended in
   * float32 and stored rounded to bfloat16 (and attended as stored). */
  int kv_dtype;
} cb_decode_attention_args;
CB_API int cb_decode_attention(const cb_decode_attention_args* args, cb_stream_t stream);
/* Scratch floats cb_decode_attention needs for these args. */
CB_API long long cb_decode_attention_scratch(const cb_decode_attention_args* args);
/* cb_decode_attention over `batch` sequences stepping together (the same
 * position, masks and RoPE row): sequence b's q | k | v projections start at
 * qkv + b * qkv_stride, its caches are the b-th (kv_heads, context, hd)
 * slice of k_cache / v_cache, its output the b-th heads * hd slice of out;
 * scratch holds cb_decode_attention_batched_scratch floats and counters
 * batch * kv_heads zeros.  Replaces, for a batched decode step, the same
 * chain as cb_decode_attention for every sequence. */
CB_API long long cb_decode_attention_batched_scratch(const cb_decode_attention_args* args, long long batch);
CB_API int cb_decode_attention_batched(const cb_decode_attention_args* args, long long batch, long long qkv_stride,
                                       cb_stream_t stream);

/* cb_decode_attention for callers that cannot allocate device memory (an FFI
 * binding that owns only the graph's bound arrays, a process whose arena
 * already holds all of HBM, a decode loop that cannot afford the device
 * synchronisation cudaFree brings).  This entry point has no counterpart in
 * the reference.  `scratch` and `counters` in args are ignored: the library
 * uses its own fixed device arrays (1 Mi floats = 4 MiB of partials, 256
 * counters).
 * The first call on a device, with that device current, sets them up (symbol
 * lookup, counters cleared, device synchronised); make it before any stream
 * capture.  Larger requests (splits * heads * (head_size + 2) > 1 Mi floats,
 * kv_heads > 256) return CB_ERR_INVALID before any launch.  All calls on a
 * device share the arrays: calls that overlap on the GPU race. */
CB_API int cb_decode_attention_noalloc(const cb_decode_attention_args* args, cb_stream_t stream);

/* ---- tensor-core GEMM (tcgen05 + TMEM + TMA) -------------------------------
 * C = A x B^T for the prefill and batched-decode Linear layers: the MATMUL of
 * `inputs @ weight.T` (chomikgrad/llama.py:275-277, lazy.py:629-630) with the
 * weight in its (out, in) = (N, K) row-major layout.  B is bf16; A is bf16 or
 * float32.  The reference multiplies float32 activations by bf16 weights in
 * float32; here a float32 A is split into two bf16 planes hi = bf16(a),
 * lo = bf16(a - hi), whose products with bf16 weights are exact in float32,
 * and both are accumulated in float32 in TMEM (residual about 2^-16 of |a|).
 * Requirements: k % 8 == 0, n % 4 == 0, b 16-byte aligned with ldb % 8 ==
 * 0, c 16-byte aligned with ldc % 4 == 0.  `a_split` is scratch of
 * cb_gemm_tc_scratch bytes (the bf16 planes A is converted into; none for a
 * bf16 A with 16-byte aligned rows). */
typedef struct {
  const void* a; /* m x k, row stride lda (elements) */
  int a_dtype;   /* CB_BF16 or CB_F32 */
  long long lda;
  const void* b; /* n x k bf16, row stride ldb */
  long long ldb;
  float* c;      /* m x n float32, row stride ldc */
  long long ldc;
  long long m, n, k;
  void* a_split; /* scratch: the bf16 plane(s) of A */
  int* error_flag;
} cb_gemm_args;
CB_API long long cb_gemm_tc_scratch(const cb_gemm_args* args);
CB_API int cb_gemm_tc(const cb_gemm_args* args, cb_stream_t stream);

/* cb_gemm_tc with up to three weights sharing A and a fused epilogue -- the
 * prefill Linears of one layer (chomikgrad/llama.py:275-277) and the
 * elementwise work that follows them:
 *  CB_GEMM_STORE     c[i] = A B[i]^T for i < n_w (q/k/v: one launch, one
 *                    plane split of A);
 *  CB_GEMM_RESIDUAL  c[0] = residual + A B[0]^T, the add in float32 (the
 *                    residual adds after the O and down projections,
 *                    llama.py:529-535);
 *  CB_GEMM_SWIGLU    c[0] = silu(A B[0]^T) * (A B[1]^T), silu(g) =
 *                    g / (1 + exp(-g)), every step float32 (llama.py:289-291,
 *                    371-380); gate and up are never stored.
 * Operands as cb_gemm_tc; n[i] % 4 == 0, rows 16-byte aligned. */
enum { CB_GEMM_STORE = 0, CB_GEMM_RESIDUAL = 1, CB_GEMM_SWIGLU = 2 };
typedef struct {
  const void* a; /* m x k, row stride lda (elements), shared by every weight */
  int a_dtype;   /* CB_BF16 or CB_F32 */
  long long lda;
  long long m, k;
  int n_w;
  const void* b[3]; /* n[i] x k bf16, row stride ldb[i] */
  long long ldb[3];
  long long n[3];
  float* c[3];      /* m x n[i] float32, row stride ldc[i] (SwiGLU, residual: c[0]) */
  long long ldc[3];
  int epilogue;     /* CB_GEMM_* */
  const float* residual; /* m x n[0], row stride ldr (CB_GEMM_RESIDUAL) */
  long long ldr;
  void* a_split; /* scratch: the bf16 plane(s) of A */
  int* error_flag;
  /* A prologue (CB_ROWS_X_PLAIN or CB_ROWS_X_RMS): with RMS, A is
   * rms_norm(a) * norm_w, computed while A is split into planes, with the
   * rounding dtypes of cb_rmsnorm_args, rounded to dt_out (llama.py:279-287) */
  int x_mode;
  const void* norm_w;
  int norm_w_dtype;
  float divisor, eps;
  int dt_sq, dt_sum, dt_mean, dt_t, dt_d, dt_y, dt_out;
} cb_gemm_multi_args;
CB_API long long cb_gemm_tc_multi_scratch(const cb_gemm_multi_args* args);
CB_API int cb_gemm_tc_multi(const cb_gemm_multi_args* args, cb_stream_t stream);

/* ---- few-row tensor-core GEMM (batched decode) -----------------------------
 * out_i (rows x w_rows[i], float32, row stride ldo[i]) = x . W_i^T for up to
 * three bf16 weights W_i (w_rows[i] x k, row-major, 16-byte aligned) sharing
 * x (rows x k, float32 or bf16, row stride ldx): the q/k/v or gate/up
 * Linears of a decode step over a batch of 1..256 sequences
 * (chomikgrad/llama.py:275-277, 387-392, 371-380).  float32 x is split into
 * bf16 hi/lo planes (products exact, residual about 2^-16 of |x|); the
 * weight rows are the MMA's 128-row side.  The (128-row tile, 64-wide K
 * chunk) sequence is cut into `splits` equal contiguous ranges, one per
 * persistent CTA (splits = 0: one per SM); a tile cut between CTAs is
 * reduced in part order by its last part (deterministic).
 * `scratch`: cb_gemm_rows_scratch bytes, 16-byte aligned; `counters`:
 * cb_gemm_rows_counters unsigned ints, zero before the first call (calls
 * leave them zero).  k % 8 == 0. */
typedef struct {
  const void* x;
  int x_dtype;
  long long ldx;
  long long rows;
  long long k;
  int n_w;
  const void* w[3];
  long long w_rows[3];
  float* out[3];
  long long ldo[3];
  int splits;
  void* scratch;
  unsigned* counters;
  int* error_flag;
  /* x prologue, applied while x is split into planes (CB_ROWS_X_*):
   *  PLAIN   x as given;
   *  RMS     rms_norm(x) * norm_w with the rounding dtypes of
   *          cb_rmsnorm_args (llama.py:279-287), rounded to dt_out;
   *  SWIGLU  silu(x) * x2 = x / (1 + exp(-x)) * x2 in float32
   *          (llama.py:289-291, 371-380), x2 rows of stride ldx2. */
  int x_mode;
  const void* norm_w;
  int norm_w_dtype;
  float divisor, eps;
  int dt_sq, dt_sum, dt_mean, dt_t, dt_d, dt_y, dt_out;
  const void* x2;
  int x2_dtype;
  long long ldx2;
  /* epilogue (n_w == 1): out[0] = residual + x . W^T, the add in float32
   * (llama.py:529-535); NULL: store */
  const float* residual;
  long long ldr;
  /* 1: programmatic dependent launch -- the first stages of weight chunks
   * stream while the previous kernel finishes (x, residual and outputs wait
   * for it) */
  int pdl;
} cb_gemm_rows_args;
enum { CB_ROWS_X_PLAIN = 0, CB_ROWS_X_RMS = 1, CB_ROWS_X_SWIGLU = 2 };
CB_API long long cb_gemm_rows_scratch(const cb_gemm_rows_args* args);
CB_API long long cb_gemm_rows_counters(const cb_gemm_rows_args* args);
CB_API int cb_gemm_rows(const cb_gemm_rows_args* args, cb_stream_t stream);

/* ---- training ----------------------------------------------------------------
 * The reference's fused lowerings of compiled training steps (lowering hints
 * of chomikgrad/tensor.py:316-450; CuPy kernels cuda_backend.py:85-322) over
 * the last axis of contiguous (rows, width) float32 matrices, one warp per
 * row:
 *   cb_softmax_rows            y = exp(x - max) / sum   (log_form: (x - max) - log(sum))
 *   cb_softmax_backward_rows   dx = y * (g - sum(g * y)) (log_form: g - exp(y) * sum(g))
 *   cb_layer_norm_rows         y = (x - mean) / sqrt(mean((x - mean)^2) + eps) * w + b
 *   cb_layer_norm_backward_rows  any of dx (rows x width), dw, db (width;
 *                              column sums over the rows, in row order);
 *                              row_stats: rows * 2 floats of scratch, needed
 *                              for dw
 * cb_sgd_update: out[i] = param[i] - lr * grad[i] (the product rounded to
 * float32 first) for up to CB_SGD_GROUP float32 tensors in one launch; out
 * may alias param (in place).  Replaces the grouped SGD of
 * Compiler.update_native_parameters (cuda_backend.py:471-617). */
#define CB_SGD_GROUP 16
typedef struct {
  int n;
  float lr;
  const float* param[CB_SGD_GROUP];
  const float* grad[CB_SGD_GROUP];
  float* out[CB_SGD_GROUP];
  long long count[CB_SGD_GROUP];
} cb_sgd_group;
CB_API int cb_softmax_rows(const float* x, long long rows, long long width, int log_form, float* out,
                           cb_stream_t stream);
CB_API int cb_softmax_backward_rows(const float* grad, const float* y, long long rows, long long width,
                                    int log_form, float* out, cb_stream_t stream);
CB_API int cb_layer_norm_rows(const float* x, const float* w, const float* b, long long rows, long long width,
                              float eps, float* out, cb_stream_t stream);
CB_API int cb_layer_norm_backward_rows(const float* grad, const float* x, const float* w, long long rows,
                                       long long width, float eps, float* dx, float* dw, float* db,
                                       float* row_stats, cb_stream_t stream);
CB_API int cb_sgd_update(const cb_sgd_group* group, cb_stream_t stream);

/* ---- tensor-parallel collectives ------------------------------------------
 * The reference is single-GPU; these serve the tensor-parallel lowering of
 * its graphs (all_reduce after the row-sharded O and down projections).  A
 * sum all-reduce over NCCL, loaded at run time (cb_comm_load: a libnccl.so.2
 * path, or NULL for the one the process already has).  cb_comm_unique_id
 * writes NCCL's 128-byte id on one rank; every rank passes it to
 * cb_comm_init.  cb_all_reduce(src -> dst, count elements, CB_F32 or CB_BF16)
 * is issued on `stream`, so a CUDA graph captured on that stream holds it.
 * cb_all_gather writes the ranks' `count`-element src buffers into dst one
 * after the other in rank order (dst holds nranks * count elements): the
 * vocabulary-sharded lm_head's logits, gathered before the argmax. */
CB_API int cb_comm_load(const char* path);
CB_API int cb_comm_unique_id(void* out, int bytes);
CB_API int cb_comm_init(const void* id, int bytes, int nranks, int rank, void** comm);
CB_API int cb_comm_destroy(void* comm);
CB_API int cb_all_reduce(void* comm, const void* src, void* dst, long long count, int dtype, cb_stream_t stream);
CB_API int cb_all_gather(void* comm, const void* src, void* dst, long long count, int dtype, cb_stream_t stream);

/* One-shot all-reduce over NVLink peer memory, for the small per-layer sums
 * of the tensor-parallel decode (batch x hidden float32 after the O and
 * down projections; the graph's all_reduce, then hidden + sum).  Each rank
 * creates its exchange region (the one allocation of this library:
 * cudaMalloc of 2 * ranks * max_count floats plus flags) and gets its 64-byte
 * CUDA IPC handle; the ranks exchange handles (host side) and each maps the
 * others' regions with cb_peer_connect (handles[ranks][64], rank order).
 * cb_peer_all_reduce: every rank stores its `count` float32 partials into
 * every region over NVLink, raises its flags, waits (bounded, 10 s or
 * cb_peer_set_wait) for every rank's flags, and writes
 * out[i] = (residual[i] +) sum over ranks in rank order -- the same value on
 * every rank.  Every rank must make the same calls in the same order.  A rank
 * that does not arrive makes the others store CB_FLAG_WAIT_PEER in
 * *error_flag (results invalid).  Plain loads / stores only (no TMA, no
 * multicast). */
CB_API int cb_peer_create(int ranks, int rank, long long max_count, void** group, void* handle_out,
                          int handle_bytes);
CB_API int cb_peer_connect(void* group, const void* handles, int handle_bytes);
CB_API int cb_peer_set_wait(void* group, long long wait_ns);
CB_API int cb_peer_max_count(void* group, long long* count);
CB_API int cb_peer_all_reduce(void* group, const float* src, void* out, int out_dtype, const void* residual,
                              int residual_dtype, long long count, int* error_flag, cb_stream_t stream);
CB_API int cb_peer_destroy(void* group);

/* Greedy argmax of every row over a vocabulary-sharded lm_head, without
 * gathering the logits.  Replaces DeviceAdapter.argmax_last_axis
 * (chomikgrad/lazy.py:132-134) for a rank whose logits `x` (rows x width) are
 * columns [col_offset, col_offset + width) of the whole rows: each rank
 * reduces its columns to a 16-byte (value, global index) record per row, the
 * records are all-gathered over `comm` (NCCL, on `stream`; comm may be NULL
 * when ranks == 1) and every rank writes the same winner to out_index[rows]:
 * np.argmax of the whole row (a NaN first, then the larger value, then the
 * lower index).  scratch: (ranks + 1) * rows * 16 bytes, 16-byte aligned. */
CB_API int cb_argmax_rows_sharded(void* comm, int ranks, const void* x, int dtype, long long rows, long long width,
                                  long long col_offset, void* scratch, long long* out_index, cb_stream_t stream);
/* Its two halves: cb_argmax_rows_partial writes each row's record
 * {float value; int valid; long long global index} to records[rows];
 * cb_argmax_pick reduces records[ranks][rows] (rank after rank) to
 * out_index[rows]. */
CB_API int cb_argmax_rows_partial(const void* x, int dtype, long long rows, long long width, long long col_offset,
                                  void* records, cb_stream_t stream);
CB_API int cb_argmax_pick(const void* records, int ranks, long long rows, long long* out_index, cb_stream_t stream);

/* ---- whole decode step in one launch --------------------------------------
 * The fused decode step of LlamaDecoderStep (chomikgrad/llama.py:469-543)
 * -- per layer the norm->QKV GEMV, RoPE + cache blend + attention, O GEMV +
 * residual, norm->gate/up GEMV, SwiGLU->down GEMV + residual, then the final
 * norm->lm_head GEMV + greedy argmax -- as phases of ONE persistent,
 * cooperative launch (one block per SM) instead of one launch per kernel.
 * Each block streams its rows of every phase through a shared-memory ring
 * (bulk copies, continuing across phase boundaries, with L2 prefetch of the
 * next phase), and waits (bounded) for the previous phase on a grid-wide
 * counter before it stages x.  Results equal cb_gemv / cb_decode_attention
 * run one after another with the same arguments. */
enum { CB_PHASE_GEMV = 0, CB_PHASE_ATTENTION = 1 };
/* x of a GEMV phase: as given, or the SwiGLU of a [gate | up] vector of
 * 2*k float32 values: x[i] = silu(v[i]) * v[k + i] (llama.py:289-291,371-380) */
enum { CB_X_PLAIN = 0, CB_X_SILU_MUL = 1 };
typedef struct {
  int kind;   /* CB_PHASE_* */
  int x_mode; /* CB_X_*, GEMV phases */
  cb_gemv_args gemv;           /* grid, pdl and prefetch fields are ignored */
  cb_decode_attention_args attention; /* split 0 or 32; pdl, prefetch ignored */
} cb_step_phase;
/* Launch shape of a prepared step (filled by cb_decode_step_prepare). */
typedef struct {
  int grid;      /* blocks per step: one per SM */
  int n_phases;
  int w_dtype;   /* weight dtype of every GEMV phase */
  int head_size; /* of the attention phases (0: none) */
  long long slot_bytes, x_bytes, norm_bytes, smem; /* shared-memory layout */
  /* L2 lookahead: bytes of its rows of the next GEMV phase each block asks L2
   * to prefetch when it starts streaming a phase (prepare sets the default) */
  long long prefetch_bytes;
  /* ring copies each producer lane keeps in flight (1 or 2; prepare sets 2):
   * fewer queue less data ahead of the consumers' latency-critical loads */
  int lane_inflight;
  /* 1: from the start of a phase's wait until its x is staged, issue no new
   * ring copies, so the latency-critical loads of that window do not queue
   * behind bulk data; 0 (prepare's default): keep streaming */
  int quiet_window;
  /* tests only (0 = off): 1 + the index of a block that withholds its
   * arrival after the first phase, so every block's wait for that phase
   * runs out (after about 1 s) and the step stops with CB_FLAG_WAIT_PHASE;
   * the caller then zeroes the counters, as after any wait that gave up */
  int test_withhold;
  /* optional (NULL = off): grid * n_phases * 12 nanosecond stamps
   * (%globaltimer) per block and phase, for tuning the schedule: wait begins,
   * wait ends, x staged, phase done, producer issued the phase's last stage,
   * thread 0's x loads returned, norm sum done, the last warp's x loads
   * returned, thread 0 normalised x, the last warp finished staging, 2 spare */
  unsigned long long* timeline;
} cb_decode_step_config;
/* Device bytes of the schedule table cb_decode_step_prepare writes. */
CB_API long long cb_decode_step_table_bytes(int n_phases);
/* prepare flags: merge an attention phase's splits while the next phase (the
 * O projection reading its output) stages x, instead of in the attention
 * phase itself (the output is then never written) */
enum { CB_STEP_MERGE_IN_STAGE = 1 };
/* Check the phases and write their schedule to `table` (device memory of
 * cb_decode_step_table_bytes bytes; synchronous, so not during stream
 * capture).  The table holds the phases' pointers: prepare again when any
 * changes.  An argmax phase's scratch must hold config->grid entries.
 * SwiGLU (CB_EPI_SILU_MUL) phases: each block streams the same rows of gate
 * and up, at most 128 rows per block. */
CB_API int cb_decode_step_prepare(const cb_step_phase* phases, int n_phases, void* table,
                                  long long table_bytes, int flags, cb_decode_step_config* config);
/* Run the prepared step.  `counters`: n_phases unsigned ints, zero before
 * the first launch; a step that completes leaves them zero (after a wait
 * gave up -- *error_flag >= CB_FLAG_WAIT_DATA -- the caller zeroes them and
 * the attention/argmax counters of the phases).  Launches of one table must
 * not overlap on the GPU. */
CB_API int cb_decode_step(const void* table, const cb_decode_step_config* config, unsigned int* counters,
                          int* error_flag, cb_stream_t stream);

/* On-device greedy step driver for back-to-back decode replays: from the
 * previous step's argmax it writes the next step's token id, position + 1,
 * attention mask row (position+1 -> 0) and write mask (one-hot at the new
 * position), exactly what the host loop of
 * examples/generate_tinyllama.py:772-786 builds each step; token_log[step]
 * records the token.  Sets *error_flag = 3 instead of writing past the
 * context. */
CB_API int cb_decode_advance(const long long* argmax, void* ids, int ids_dtype, void* position,
                      int position_dtype, void* mask, int mask_dtype, void* write_mask,
                      int write_mask_dtype, long long context, long long* token_log, long long step,
                      int* error_flag, cb_stream_t stream);

/* The same for `rows` sequences decoded together (one batched program):
 * ids[b] = argmax[b], token_log[step * rows + b]; position and masks are
 * shared. */
CB_API int cb_decode_advance_rows(const long long* argmax, long long rows, void* ids, int ids_dtype,
                                  void* position, int position_dtype, void* mask, int mask_dtype,
                                  void* write_mask, int write_mask_dtype, long long context,
                                  long long* token_log, long long step, int* error_flag, cb_stream_t stream);

/* Row-wise argmax with np.argmax semantics (first max, NaN wins).
 * Replaces DeviceAdapter.argmax / argmax_last_axis (chomikgrad/lazy.py:128-134,
 * cuda_backend.py:37-41). */
CB_API int cb_argmax_rows(const void* x, int dtype, long long rows, long long width,
                   long long* out_index, cb_stream_t stream);

/* Temperature / top-k sampling of each row of a logit matrix, on the device.
 * Replaces the host sampler sample_token (examples/generate_tinyllama.py
 * :124-143) that sample_native_token (:146-157) calls for temperature != 0:
 * v = logits / temperature in float64, top-k filter, p = softmax(v),
 * token = the first index whose cumulative p exceeds u * sum(p), where u is
 * the caller's draw -- NumPy's Generator.choice(V, p=p) takes exactly one
 * u = rng.random() and returns that index.  Ties at the k-th largest value
 * keep the lowest indices.  A row with a NaN logit, or whose largest
 * logit / temperature is not finite, gets token -1 and CB_FLAG_NAN (NumPy's
 * choice raises ValueError on NaN probabilities). */
typedef struct {
  const void* logits;
  int logits_dtype;            /* CB_F32 / CB_BF16 / CB_F16 */
  long long rows, width, ld;   /* ld: elements between consecutive rows (>= width) */
  double temperature;          /* > 0 (temperature 0 is cb_argmax_rows) */
  long long top_k;             /* <= 0 or >= width: no top-k filter */
  const double* uniforms;      /* device: one draw in [0, 1) per row */
  long long* out;              /* device: one token id per row */
  int* error_flag;             /* optional: CB_FLAG_NAN */
} cb_sample_args;
CB_API int cb_sample_rows(const cb_sample_args* a, cb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CHOMIK_B200_H */

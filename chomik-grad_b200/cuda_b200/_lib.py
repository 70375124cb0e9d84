"""ctypes binding of ``libchomik_b200.so`` (declared in include/chomik_b200.h).

The structures below mirror the C header field for field.  Loading fails
loudly when the library is missing: the plugin has no CPU fallback.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_longlong, c_uint, c_void_p
from pathlib import Path
from typing import Optional

import numpy as np

LIBRARY_PATH = Path(__file__).resolve().parent / "libchomik_b200.so"

F32, BF16, F16, I32, I64 = 0, 1, 2, 3, 4
CAUSAL_SKIP, CAUSAL_ZERO_BELOW = 1, 2  # cb_sdpa_tc causal flags
MAX_DIMS = 8
EW_MAX_INPUTS = 8
EW_MAX_INSTR = 40
MM_MAX_BATCH = 6

OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "equal": 4, "neg": 5, "exp": 6,
       "log": 7, "sqrt": 8, "relu": 9, "step": 10}
BINARY = {"add", "sub", "mul", "div", "equal"}
REDUCE_SUM, REDUCE_MAX = 0, 1
NORM_NONE, NORM_RMS, NORM_RMS_TABLE = 0, 1, 2
EPI_STORE, EPI_RESIDUAL, EPI_SILU_MUL, EPI_ARGMAX = 0, 1, 2, 3
PHASE_GEMV, PHASE_ATTENTION = 0, 1
X_PLAIN, X_SILU_MUL = 0, 1
STEP_MERGE_IN_STAGE = 1

LL8 = c_longlong * MAX_DIMS


class ElementwiseArgs(ctypes.Structure):
    _fields_ = [
        ("ndim", c_int), ("n_inputs", c_int), ("n_instr", c_int), ("out_dtype", c_int),
        ("shape", LL8),
        ("inputs", c_void_p * EW_MAX_INPUTS),
        ("in_dtype", c_int * EW_MAX_INPUTS),
        ("in_strides", LL8 * EW_MAX_INPUTS),
        ("in_offset", c_longlong * EW_MAX_INPUTS),
        ("op", c_int * EW_MAX_INSTR), ("lhs", c_int * EW_MAX_INSTR),
        ("rhs", c_int * EW_MAX_INSTR), ("round", c_int * EW_MAX_INSTR),
        ("out", c_void_p),
    ]


class ReduceArgs(ctypes.Structure):
    _fields_ = [
        ("in_", c_void_p), ("in_dtype", c_int), ("out", c_void_p), ("out_dtype", c_int),
        ("kind", c_int), ("sequential", c_int), ("acc_dtype", c_int),
        ("n_keep", c_int), ("n_red", c_int), ("in_offset", c_longlong),
        ("keep_shape", LL8), ("keep_strides", LL8), ("red_shape", LL8), ("red_strides", LL8),
    ]


class MatmulArgs(ctypes.Structure):
    _fields_ = [
        ("a", c_void_p), ("a_dtype", c_int), ("b", c_void_p), ("b_dtype", c_int),
        ("c", c_void_p), ("c_dtype", c_int),
        ("m", c_longlong), ("n", c_longlong), ("k", c_longlong),
        ("a_offset", c_longlong), ("b_offset", c_longlong),
        ("a_rs", c_longlong), ("a_cs", c_longlong), ("b_rs", c_longlong), ("b_cs", c_longlong),
        ("batch_ndim", c_int),
        ("batch_shape", c_longlong * MM_MAX_BATCH),
        ("a_bstride", c_longlong * MM_MAX_BATCH),
        ("b_bstride", c_longlong * MM_MAX_BATCH),
    ]


class RmsNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_int),
        ("rows", c_longlong), ("width", c_longlong), ("x_row_stride", c_longlong),
        ("x_offset", c_longlong),
        ("x_index", c_void_p), ("x_index_dtype", c_int),
        ("w", c_void_p), ("w_dtype", c_int),
        ("out", c_void_p), ("out_dtype", c_int),
        ("divisor", c_float), ("eps", c_float),
        ("dt_sq", c_int), ("dt_sum", c_int), ("dt_mean", c_int), ("dt_t", c_int),
        ("dt_d", c_int), ("dt_y", c_int),
        ("d_table", c_void_p),
    ]


class RopeArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_int), ("x_offset", c_longlong),
        ("x_strides", c_longlong * 4),
        ("out", c_void_p), ("out_dtype", c_int),
        ("batch", c_longlong), ("heads", c_longlong), ("tokens", c_longlong),
        ("head_size", c_longlong),
        ("cos_table", c_void_p), ("sin_table", c_void_p),
        ("n_offsets", c_longlong), ("offset", c_void_p), ("offset_dtype", c_int),
        ("error_flag", c_void_p),
    ]


class SdpaArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_dtype", c_int), ("q_offset", c_longlong), ("q_strides", c_longlong * 4),
        ("k", c_void_p), ("k_dtype", c_int), ("k_offset", c_longlong), ("k_strides", c_longlong * 4),
        ("v", c_void_p), ("v_dtype", c_int), ("v_offset", c_longlong), ("v_strides", c_longlong * 4),
        ("mask", c_void_p), ("mask_dtype", c_int), ("mask_offset", c_longlong),
        ("mask_strides", c_longlong * 4),
        ("out", c_void_p),
        ("batch", c_longlong), ("heads", c_longlong), ("kv_heads", c_longlong),
        ("tq", c_longlong), ("tk", c_longlong), ("head_size", c_longlong),
        ("divisor", c_float), ("out_strides", c_longlong * 4),
    ]


class SampleArgs(ctypes.Structure):
    _fields_ = [
        ("logits", c_void_p), ("logits_dtype", c_int),
        ("rows", c_longlong), ("width", c_longlong), ("ld", c_longlong),
        ("temperature", ctypes.c_double), ("top_k", c_longlong),
        ("uniforms", c_void_p), ("out", c_void_p), ("error_flag", c_void_p),
    ]


class GemvArgs(ctypes.Structure):
    _fields_ = [
        ("w", c_void_p * 3), ("w_rows", c_longlong * 3), ("n_w", c_int), ("w_dtype", c_int),
        ("k", c_longlong),
        ("x", c_void_p), ("x_dtype", c_int), ("x_index", c_void_p), ("x_index_dtype", c_int),
        ("index_rows", c_longlong), ("error_flag", c_void_p),
        ("norm", c_int), ("norm_w", c_void_p), ("norm_w_dtype", c_int),
        ("divisor", c_float), ("eps", c_float),
        ("dt_sq", c_int), ("dt_sum", c_int), ("dt_mean", c_int), ("dt_t", c_int),
        ("dt_d", c_int), ("dt_y", c_int), ("dt_norm_out", c_int),
        ("norm_table", c_void_p),
        ("epilogue", c_int),
        ("residual", c_void_p), ("residual_dtype", c_int),
        ("residual_index", c_void_p), ("residual_index_dtype", c_int),
        ("out", c_void_p),
        ("scratch_val", c_void_p), ("scratch_idx", c_void_p), ("counter", c_void_p),
        ("argmax_out", c_void_p),
        ("prefetch_ptr", c_void_p * 3), ("prefetch_bytes", c_longlong * 3),
        ("grid", c_int), ("pdl", c_int),
    ]


class DecodeAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", c_void_p), ("q_off", c_longlong), ("k_off", c_longlong), ("v_off", c_longlong),
        ("heads", c_longlong), ("kv_heads", c_longlong), ("head_size", c_longlong),
        ("context", c_longlong),
        ("position", c_void_p), ("position_dtype", c_int),
        ("cos_table", c_void_p), ("sin_table", c_void_p), ("n_positions", c_longlong),
        ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("write_mask", c_void_p), ("write_mask_dtype", c_int), ("one_minus_dtype", c_int),
        ("mask", c_void_p), ("mask_dtype", c_int),
        ("divisor", c_float),
        ("out", c_void_p), ("scratch", c_void_p), ("counters", c_void_p), ("error_flag", c_void_p),
        ("prefetch_ptr", c_void_p * 3), ("prefetch_bytes", c_longlong * 3),
        ("split", c_int), ("pdl", c_int), ("kv_dtype", c_int),
    ]


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("a", c_void_p), ("a_dtype", c_int), ("lda", c_longlong),
        ("b", c_void_p), ("ldb", c_longlong),
        ("c", c_void_p), ("ldc", c_longlong),
        ("m", c_longlong), ("n", c_longlong), ("k", c_longlong),
        ("a_split", c_void_p), ("error_flag", c_void_p),
    ]


GEMM_STORE, GEMM_RESIDUAL, GEMM_SWIGLU = 0, 1, 2  # cb_gemm_tc_multi epilogues


class GemmMultiArgs(ctypes.Structure):
    _fields_ = [
        ("a", c_void_p), ("a_dtype", c_int), ("lda", c_longlong),
        ("m", c_longlong), ("k", c_longlong), ("n_w", c_int),
        ("b", c_void_p * 3), ("ldb", c_longlong * 3), ("n", c_longlong * 3),
        ("c", c_void_p * 3), ("ldc", c_longlong * 3),
        ("epilogue", c_int), ("residual", c_void_p), ("ldr", c_longlong),
        ("a_split", c_void_p), ("error_flag", c_void_p),
        ("x_mode", c_int), ("norm_w", c_void_p), ("norm_w_dtype", c_int),
        ("divisor", c_float), ("eps", c_float),
        ("dt_sq", c_int), ("dt_sum", c_int), ("dt_mean", c_int), ("dt_t", c_int), ("dt_d", c_int),
        ("dt_y", c_int), ("dt_out", c_int),
    ]


class GemmRowsArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_int), ("ldx", c_longlong), ("rows", c_longlong), ("k", c_longlong),
        ("n_w", c_int), ("w", c_void_p * 3), ("w_rows", c_longlong * 3),
        ("out", c_void_p * 3), ("ldo", c_longlong * 3), ("splits", c_int),
        ("scratch", c_void_p), ("counters", c_void_p), ("error_flag", c_void_p),
        ("x_mode", c_int), ("norm_w", c_void_p), ("norm_w_dtype", c_int),
        ("divisor", c_float), ("eps", c_float),
        ("dt_sq", c_int), ("dt_sum", c_int), ("dt_mean", c_int), ("dt_t", c_int), ("dt_d", c_int),
        ("dt_y", c_int), ("dt_out", c_int),
        ("x2", c_void_p), ("x2_dtype", c_int), ("ldx2", c_longlong),
        ("residual", c_void_p), ("ldr", c_longlong), ("pdl", c_int),
    ]


ROWS_X_PLAIN, ROWS_X_RMS, ROWS_X_SWIGLU = 0, 1, 2  # cb_gemm_rows x prologues
STEP_X_VECTORS = 3 * 256  # x vectors (8 bf16-weight or 4 float32-weight columns) a cb_decode_step phase stages
STEP_ROWS_PER_BLOCK = 128  # SwiGLU gate/up pairs one cb_decode_step block owns in a phase


class StepPhase(ctypes.Structure):
    _fields_ = [("kind", c_int), ("x_mode", c_int), ("gemv", GemvArgs), ("attention", DecodeAttentionArgs)]


SGD_GROUP = 16


class SgdGroup(ctypes.Structure):
    _fields_ = [("n", c_int), ("lr", c_float), ("param", c_void_p * SGD_GROUP), ("grad", c_void_p * SGD_GROUP),
                ("out", c_void_p * SGD_GROUP), ("count", c_longlong * SGD_GROUP)]


class DecodeStepConfig(ctypes.Structure):
    _fields_ = [("grid", c_int), ("n_phases", c_int), ("w_dtype", c_int), ("head_size", c_int),
                ("slot_bytes", c_longlong), ("x_bytes", c_longlong), ("norm_bytes", c_longlong),
                ("smem", c_longlong),
                ("prefetch_bytes", c_longlong), ("lane_inflight", c_int), ("quiet_window", c_int),
                ("test_withhold", c_int),
                ("timeline", c_void_p)]


class KernelError(RuntimeError):
    """A libchomik_b200 entry point returned a non-zero status."""


_LIB: Optional[ctypes.CDLL] = None

_SIGNATURES = {
    "cb_abi_version": ([], c_int),
    "cb_last_error": ([], c_char_p),
    "cb_sm_count": ([POINTER(c_int)], c_int),
    "cb_stream_create": ([POINTER(c_void_p)], c_int),
    "cb_stream_destroy": ([c_void_p], c_int),
    "cb_capture_begin": ([c_void_p], c_int),
    "cb_capture_end": ([c_void_p, POINTER(c_void_p)], c_int),
    "cb_graph_launch": ([c_void_p, c_void_p], c_int),
    "cb_graph_destroy": ([c_void_p], c_int),
    "cb_elementwise": ([POINTER(ElementwiseArgs), c_void_p], c_int),
    "cb_reduce": ([POINTER(ReduceArgs), c_void_p], c_int),
    "cb_copy_strided": ([c_void_p, c_longlong, c_void_p, c_int, c_int, POINTER(c_longlong),
                         POINTER(c_longlong), c_void_p], c_int),
    "cb_gather": ([c_void_p, c_longlong, c_longlong, c_void_p, c_int, c_longlong, c_void_p,
                   c_void_p, c_void_p], c_int),
    "cb_matmul": ([POINTER(MatmulArgs), c_void_p], c_int),
    "cb_rmsnorm": ([POINTER(RmsNormArgs), c_void_p], c_int),
    "cb_rmsnorm_row_table": ([POINTER(RmsNormArgs), c_void_p, c_void_p], c_int),
    "cb_rope": ([POINTER(RopeArgs), c_void_p], c_int),
    "cb_sdpa": ([POINTER(SdpaArgs), c_void_p], c_int),
    "cb_comm_load": ([c_char_p], c_int),
    "cb_comm_unique_id": ([c_void_p, c_int], c_int),
    "cb_comm_init": ([c_void_p, c_int, c_int, c_int, POINTER(c_void_p)], c_int),
    "cb_comm_destroy": ([c_void_p], c_int),
    "cb_all_reduce": ([c_void_p, c_void_p, c_void_p, c_longlong, c_int, c_void_p], c_int),
    "cb_all_gather": ([c_void_p, c_void_p, c_void_p, c_longlong, c_int, c_void_p], c_int),
    "cb_sdpa_query_scratch": ([POINTER(SdpaArgs)], c_longlong),
    "cb_sdpa_query": ([POINTER(SdpaArgs), c_void_p, c_void_p], c_int),
    "cb_gemv": ([POINTER(GemvArgs), c_void_p], c_int),
    "cb_gemv_grid": ([POINTER(GemvArgs), POINTER(c_int)], c_int),
    "cb_decode_attention": ([POINTER(DecodeAttentionArgs), c_void_p], c_int),
    "cb_decode_attention_scratch": ([POINTER(DecodeAttentionArgs)], c_longlong),
    "cb_decode_attention_batched_scratch": ([POINTER(DecodeAttentionArgs), c_longlong], c_longlong),
    "cb_decode_attention_batched": ([POINTER(DecodeAttentionArgs), c_longlong, c_longlong, c_void_p], c_int),
    "cb_decode_attention_noalloc": ([POINTER(DecodeAttentionArgs), c_void_p], c_int),
    "cb_place_columns": ([c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_longlong, c_void_p, c_int,
                          c_void_p], c_int),
    "cb_sdpa_tc_scratch": ([POINTER(SdpaArgs)], c_longlong),
    "cb_sdpa_tc": ([POINTER(SdpaArgs), c_int, c_void_p, c_void_p, c_void_p], c_int),
    "cb_kv_write": ([c_void_p, c_longlong, c_longlong, c_longlong, c_longlong, c_void_p, c_int,
                     POINTER(c_longlong), c_void_p, c_int, c_int, c_void_p], c_int),
    "cb_gemm_rows_scratch": ([POINTER(GemmRowsArgs)], c_longlong),
    "cb_gemm_rows_counters": ([POINTER(GemmRowsArgs)], c_longlong),
    "cb_gemm_rows": ([POINTER(GemmRowsArgs), c_void_p], c_int),
    "cb_gemm_tc_scratch": ([POINTER(GemmArgs)], c_longlong),
    "cb_gemm_tc": ([POINTER(GemmArgs), c_void_p], c_int),
    "cb_gemm_tc_multi_scratch": ([POINTER(GemmMultiArgs)], c_longlong),
    "cb_gemm_tc_multi": ([POINTER(GemmMultiArgs), c_void_p], c_int),
    "cb_decode_step_table_bytes": ([c_int], c_longlong),
    "cb_decode_step_prepare": ([POINTER(StepPhase), c_int, c_void_p, c_longlong, c_int,
                                POINTER(DecodeStepConfig)], c_int),
    "cb_decode_step": ([c_void_p, POINTER(DecodeStepConfig), c_void_p, c_void_p, c_void_p], c_int),
    "cb_argmax_rows": ([c_void_p, c_int, c_longlong, c_longlong, c_void_p, c_void_p], c_int),
    "cb_argmax_rows_sharded": ([c_void_p, c_int, c_void_p, c_int, c_longlong, c_longlong, c_longlong, c_void_p,
                                c_void_p, c_void_p], c_int),
    "cb_argmax_rows_partial": ([c_void_p, c_int, c_longlong, c_longlong, c_longlong, c_void_p, c_void_p], c_int),
    "cb_argmax_pick": ([c_void_p, c_int, c_longlong, c_void_p, c_void_p], c_int),
    "cb_peer_create": ([c_int, c_int, c_longlong, c_void_p, c_void_p, c_int], c_int),
    "cb_peer_connect": ([c_void_p, c_void_p, c_int], c_int),
    "cb_peer_set_wait": ([c_void_p, c_longlong], c_int),
    "cb_peer_max_count": ([c_void_p, c_void_p], c_int),
    "cb_peer_all_reduce": ([c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_longlong, c_void_p, c_void_p],
                           c_int),
    "cb_peer_destroy": ([c_void_p], c_int),
    "cb_softmax_rows": ([c_void_p, c_longlong, c_longlong, c_int, c_void_p, c_void_p], c_int),
    "cb_softmax_backward_rows": ([c_void_p, c_void_p, c_longlong, c_longlong, c_int, c_void_p, c_void_p], c_int),
    "cb_layer_norm_rows": ([c_void_p, c_void_p, c_void_p, c_longlong, c_longlong, c_float, c_void_p, c_void_p],
                           c_int),
    "cb_layer_norm_backward_rows": ([c_void_p, c_void_p, c_void_p, c_longlong, c_longlong, c_float, c_void_p,
                                     c_void_p, c_void_p, c_void_p, c_void_p], c_int),
    "cb_sgd_update": ([c_void_p, c_void_p], c_int),
    "cb_sample_rows": ([c_void_p, c_void_p], c_int),
    "cb_decode_advance": ([c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p,
                           c_int, c_longlong, c_void_p, c_longlong, c_void_p, c_void_p], c_int),
    "cb_decode_advance_rows": ([c_void_p, c_longlong, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                c_void_p, c_int, c_longlong, c_void_p, c_longlong, c_void_p, c_void_p], c_int),
}

EXPORTED = tuple(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load (once) and type the library; raises if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIBRARY_PATH.exists():
        raise ImportError(
            f"{LIBRARY_PATH.name} is not built; run `python -m cuda_b200._build` "
            "(the cuda-b200 plugin has no CPU fallback)")
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    for name, (args, result) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = result
    _LIB = lib
    return lib


FLAG_INDEX, FLAG_POSITION, FLAG_CONTEXT = 1, 2, 3
FLAG_WAIT_DATA, FLAG_WAIT_SLOT, FLAG_WAIT_DRAIN, FLAG_WAIT_PHASE = 4, 5, 6, 7
FLAG_NAN = 8
FLAG_WAIT_PEER = 9


def flag_error(value: int) -> Exception:
    """The exception for a kernel error-flag value (CB_FLAG_* in the header)."""
    if value == FLAG_INDEX:
        return IndexError("gather index is outside the first dimension")
    if value == FLAG_POSITION:
        return IndexError("RoPE position is outside the precomputed table")
    if value == FLAG_CONTEXT:
        return IndexError("decode step would write past the KV-cache context")
    if value == FLAG_NAN:  # what NumPy's Generator.choice raises for the reference's sampler
        return ValueError("probabilities contain NaN")
    waits = {FLAG_WAIT_DATA: "a consumer waiting for weight data",
             FLAG_WAIT_SLOT: "a producer waiting for a free ring slot",
             FLAG_WAIT_DRAIN: "the end-of-kernel drain of bulk copies",
             FLAG_WAIT_PHASE: "a block waiting for the previous phase of the decode step",
             FLAG_WAIT_PEER: "the peer all-reduce waiting for another rank of the group"}
    if value in waits:
        return KernelError(f"kernel timed out in {waits[value]} (results are invalid)")
    return KernelError(f"kernel error flag {value}")


def check(status: int, what: str = "") -> None:
    if status != 0:
        message = load().cb_last_error().decode(errors="replace")
        raise KernelError(f"{what or 'libchomik_b200'}: {message}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def dtype_code(dtype: np.dtype) -> int:
    dtype = np.dtype(dtype)
    if dtype == np.float32:
        return F32
    if dtype.name == "bfloat16":
        return BF16
    if dtype == np.float16:
        return F16
    if dtype == np.int32:
        return I32
    if dtype == np.int64:
        return I64
    raise TypeError(f"cuda-b200 does not support dtype {dtype}")


def ll_array(values, size: int = MAX_DIMS):
    arr = (c_longlong * size)()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr

"""cb_decode_attention_batched against a float64 restatement, through the C ABI.

The batched decode attention ropes q and k at the shared position, blends
the new k / v rows into every sequence's caches where the write mask is
non-zero, and attends over the context (llama.py:509-525 per sequence).  A
CTA walks a range of 32-key chunks with an online softmax and the last CTA
of each (sequence, KV head) merges the ranges, so the cases cover one and
many chunks per CTA, one range per group (nothing to merge), ragged last
chunks, and 1, 2 and 4 query heads per warp.  Bars: attention output within
2e-5 of float64 (float32 arithmetic over up to 1280 keys), updated caches
within 1e-6 (the roped row differs from a float64 rotation by rounding).
With bfloat16 caches the kernel reads bfloat16 K/V and stores the rows it
writes rounded to bfloat16; the float64 restatement attends over the same
rounded rows, and the written rows agree within one bfloat16 rounding.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from plan_interpreter import _blend, _rotate, _softmax_attention

pytestmark = pytest.mark.gpu

CASES = [
    # batch, heads, kv_heads, head_size, context, position
    (32, 32, 4, 64, 768, 700),    # TinyLlama bs32: 4 ranges of 6 chunks per group
    (48, 16, 4, 128, 200, 150),   # ranges of 3, 3 and 1 (8-row) chunks
    (64, 32, 8, 128, 1280, 1000), # one range per group: the whole context, no merge
    (3, 8, 1, 32, 100, 37),       # one chunk per CTA, ragged last chunk
    (8, 32, 2, 64, 500, 499),     # 16 query heads per KV head: two per warp
    (4, 32, 1, 64, 96, 0),        # 32 query heads per KV head: four per warp
]


def _tables(hd, n_positions):
    inv = 1.0 / (10000.0 ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    angles = np.outer(np.arange(n_positions, dtype=np.float64), inv)
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


@pytest.mark.parametrize("kv_dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("batch,heads,kv,hd,ctx,pos", CASES)
def test_batched_decode_attention_matches_float64(batch, heads, kv, hd, ctx, pos, kv_dtype):
    import ml_dtypes
    import torch

    from cuda_b200 import _lib
    from cuda_b200.graphs import decode_masks

    bf = kv_dtype == "bfloat16"
    store = np.dtype(ml_dtypes.bfloat16) if bf else np.dtype(np.float32)
    rng = np.random.default_rng(batch * 1000 + ctx)
    row = (heads + 2 * kv) * hd
    qkv = rng.normal(0, 1, (batch, row)).astype(np.float32)
    k_cache = rng.normal(0, 1, (batch, kv, ctx, hd)).astype(store).astype(np.float32)
    v_cache = rng.normal(0, 1, (batch, kv, ctx, hd)).astype(store).astype(np.float32)
    mask, write = decode_masks(pos, ctx, np.float32)
    n_positions = ctx + 8
    cos, sin = _tables(hd, n_positions)

    dev = {name: torch.from_numpy(np.ascontiguousarray(v)).cuda()
           for name, v in (("qkv", qkv), ("k", k_cache), ("v", v_cache), ("mask", mask.reshape(-1)),
                           ("write", write.reshape(-1)), ("cos", cos), ("sin", sin))}
    if bf:
        dev["k"], dev["v"] = dev["k"].to(torch.bfloat16), dev["v"].to(torch.bfloat16)
    position = torch.tensor([pos], dtype=torch.int64).cuda()
    out = torch.full((batch, heads * hd), float("nan")).cuda()
    splits = -(-ctx // 32)
    scratch = torch.empty(batch * splits * heads * (hd + 2)).cuda()
    counters = torch.zeros(batch * kv, dtype=torch.int32).cuda()
    flag = torch.zeros(1, dtype=torch.int32).cuda()
    a = _lib.DecodeAttentionArgs()
    a.qkv = dev["qkv"].data_ptr()
    a.q_off, a.k_off, a.v_off = 0, heads * hd, (heads + kv) * hd
    a.heads, a.kv_heads, a.head_size, a.context = heads, kv, hd, ctx
    a.position, a.position_dtype = position.data_ptr(), _lib.I64
    a.cos_table, a.sin_table, a.n_positions = dev["cos"].data_ptr(), dev["sin"].data_ptr(), n_positions
    a.k_cache, a.v_cache = dev["k"].data_ptr(), dev["v"].data_ptr()
    a.write_mask, a.write_mask_dtype, a.one_minus_dtype = dev["write"].data_ptr(), _lib.F32, _lib.F32
    a.mask, a.mask_dtype = dev["mask"].data_ptr(), _lib.F32
    a.divisor = float(np.sqrt(hd))
    a.out, a.scratch, a.counters, a.error_flag = out.data_ptr(), scratch.data_ptr(), counters.data_ptr(), flag.data_ptr()
    a.split, a.pdl = 32, 0
    a.kv_dtype = _lib.BF16 if bf else _lib.F32
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the second call checks that the counters were reset (caches: second blend is idempotent)
        _lib.call("cb_decode_attention_batched", ctypes.byref(a), batch, row, stream)
        torch.cuda.synchronize()
    assert int(flag.item()) == 0
    assert not counters.any()

    want_out = np.zeros((batch, heads * hd))
    for b in range(batch):
        q = _rotate(qkv[b, : heads * hd].reshape(1, heads, 1, hd), cos[pos][None], sin[pos][None])
        k = _rotate(qkv[b, heads * hd: (heads + kv) * hd].reshape(1, kv, 1, hd), cos[pos][None], sin[pos][None])
        v = qkv[b, (heads + kv) * hd:].reshape(1, kv, 1, hd)
        kc = _blend(k_cache[b: b + 1], k, write.reshape(-1), np.float32).astype(store).astype(np.float32)
        vc = _blend(v_cache[b: b + 1], v, write.reshape(-1), np.float32).astype(store).astype(np.float32)
        k_cache[b], v_cache[b] = kc[0], vc[0]
        want_out[b] = _softmax_attention(q, kc, vc, mask.reshape(1, 1, 1, -1).astype(np.float64),
                                         float(np.sqrt(hd))).reshape(-1)
    # bf16: a written row may round the other way than the restatement's (one bf16 ulp, 2^-8 relative)
    np.testing.assert_allclose(out.cpu().numpy(), want_out, rtol=0, atol=2e-3 if bf else 2e-5)
    tol = dict(rtol=2 ** -7, atol=1e-4) if bf else dict(rtol=0, atol=1e-6)
    np.testing.assert_allclose(dev["k"].float().cpu().numpy(), k_cache, **tol)
    np.testing.assert_allclose(dev["v"].float().cpu().numpy(), v_cache, **tol)

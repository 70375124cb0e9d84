"""cb_decode_attention_noalloc against cb_decode_attention, through the C ABI.

The no-alloc entry point serves callers that cannot allocate device memory:
it keeps its split partials and per-KV-head counters in fixed device arrays
inside the library.  Two calls in a row (different positions, the second on
the caches the first updated) must match the allocating entry point.  The
counters are not readable from outside the library; that each call leaves
them at zero is shown by its effect: two more calls with four KV heads (the
first uses counters 0-3, the second reuses them, including the two that no
earlier call touched) also match the allocating entry point, which only holds
if every counter was back at zero.  This file is named to run last, so it is
exercised both alone and after every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HEADS, KV_HEADS, HEAD_SIZE, CONTEXT, N_POSITIONS = 8, 2, 64, 80, 128


def _inputs(torch, seed, heads=HEADS, kv_heads=KV_HEADS):
    gen = torch.Generator().manual_seed(seed)
    qkv = torch.randn((heads + 2 * kv_heads) * HEAD_SIZE, generator=gen)
    k_cache = torch.randn(kv_heads, CONTEXT, HEAD_SIZE, generator=gen)
    v_cache = torch.randn(kv_heads, CONTEXT, HEAD_SIZE, generator=gen)
    return qkv, k_cache, v_cache


def _tables(torch):
    inv = 1.0 / (10000.0 ** (np.arange(0, HEAD_SIZE, 2, dtype=np.float64) / HEAD_SIZE))
    angles = np.outer(np.arange(N_POSITIONS, dtype=np.float64), inv)
    return (torch.from_numpy(np.cos(angles).astype(np.float32)).cuda(),
            torch.from_numpy(np.sin(angles).astype(np.float32)).cuda())


class _Case:
    """Device buffers of one decode-attention call at `position`."""

    def __init__(self, torch, tables, qkv, k_cache, v_cache, position, share_caches=None,
                 heads=HEADS, kv_heads=KV_HEADS):
        from cuda_b200 import _lib
        from cuda_b200.graphs import decode_masks

        mask, write = decode_masks(position, CONTEXT, np.float32)
        self.qkv = qkv.cuda()
        if share_caches is not None:  # update another case's caches in place
            self.k_cache, self.v_cache = share_caches.k_cache, share_caches.v_cache
        else:
            self.k_cache = k_cache.clone().cuda()
            self.v_cache = v_cache.clone().cuda()
        self.position = torch.tensor([position], dtype=torch.int64).cuda()
        self.mask = torch.from_numpy(mask.reshape(-1).copy()).cuda()
        self.write = torch.from_numpy(write.reshape(-1).copy()).cuda()
        self.out = torch.full((heads * HEAD_SIZE,), float("nan")).cuda()
        self.flag = torch.zeros(1, dtype=torch.int32).cuda()
        a = _lib.DecodeAttentionArgs()
        a.qkv = self.qkv.data_ptr()
        a.q_off, a.k_off, a.v_off = 0, heads * HEAD_SIZE, (heads + kv_heads) * HEAD_SIZE
        a.heads, a.kv_heads, a.head_size, a.context = heads, kv_heads, HEAD_SIZE, CONTEXT
        a.position, a.position_dtype = self.position.data_ptr(), _lib.I64
        a.cos_table, a.sin_table = tables[0].data_ptr(), tables[1].data_ptr()
        a.n_positions = N_POSITIONS
        a.k_cache, a.v_cache = self.k_cache.data_ptr(), self.v_cache.data_ptr()
        a.write_mask, a.write_mask_dtype = self.write.data_ptr(), _lib.F32
        a.one_minus_dtype = _lib.F32
        a.mask, a.mask_dtype = self.mask.data_ptr(), _lib.F32
        a.divisor = float(np.sqrt(HEAD_SIZE))
        a.out = self.out.data_ptr()
        a.error_flag = self.flag.data_ptr()
        a.split, a.pdl = 32, 0
        self.args = a

    def results(self):
        return [t.cpu().numpy() for t in (self.out, self.k_cache, self.v_cache, self.flag)]


def _allocating(torch, case):
    """The existing entry point, with caller-allocated scratch and counters."""
    from cuda_b200 import _lib

    floats = _lib.load().cb_decode_attention_scratch(ctypes.byref(case.args))
    scratch = torch.empty(floats, dtype=torch.float32, device="cuda")
    counters = torch.zeros(case.args.kv_heads, dtype=torch.int32, device="cuda")
    case.args.scratch, case.args.counters = scratch.data_ptr(), counters.data_ptr()
    _lib.call("cb_decode_attention", ctypes.byref(case.args), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert not counters.any().item()
    return case.results()


def _no_alloc(torch, case):
    from cuda_b200 import _lib

    case.args.scratch = case.args.counters = None
    _lib.call("cb_decode_attention_noalloc", ctypes.byref(case.args), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return case.results()


def test_no_alloc_decode_attention_matches_two_calls_in_a_row():
    torch = pytest.importorskip("torch")
    tables = _tables(torch)
    qkv1, k_cache, v_cache = _inputs(torch, 1)
    qkv2, _, _ = _inputs(torch, 2)
    # call 1 at position 37 (second split); call 2 at 70 (third, ragged split)
    # on the caches call 1 left behind
    expect1 = _allocating(torch, _Case(torch, tables, qkv1, k_cache, v_cache, 37))
    expect2 = _allocating(torch, _Case(torch, tables, qkv2, torch.from_numpy(expect1[1]),
                                       torch.from_numpy(expect1[2]), 70))
    first = _Case(torch, tables, qkv1, k_cache, v_cache, 37)
    second = _Case(torch, tables, qkv2, None, None, 70, share_caches=first)
    torch.cuda.synchronize()
    got1 = _no_alloc(torch, first)
    free_before = torch.cuda.mem_get_info()[0]
    got2 = _no_alloc(torch, second)
    assert torch.cuda.mem_get_info()[0] == free_before
    for got, expect in ((got1, expect1), (got2, expect2)):
        assert np.isfinite(got[0]).all()
        for g, e in zip(got[:3], expect[:3]):
            np.testing.assert_allclose(g, e, rtol=1e-4, atol=1e-6)
        assert got[3][0] == 0 and expect[3][0] == 0
    # the caches changed only in the written row
    assert not np.array_equal(got1[1][:, 37], k_cache.numpy()[:, 37])
    np.testing.assert_array_equal(np.delete(got1[1], 37, axis=1), np.delete(k_cache.numpy(), 37, axis=1))

    # two more calls in order with four KV heads: counters 2 and 3 are used for the first time by
    # the third call and again by the fourth, so the fourth matches only if the third reset them
    wide = dict(heads=16, kv_heads=4)
    qkv3, k3, v3 = _inputs(torch, 3, **wide)
    qkv4, _, _ = _inputs(torch, 4, **wide)
    expect3 = _allocating(torch, _Case(torch, tables, qkv3, k3, v3, 50, **wide))
    expect4 = _allocating(torch, _Case(torch, tables, qkv4, torch.from_numpy(expect3[1]),
                                       torch.from_numpy(expect3[2]), 51, **wide))
    third = _Case(torch, tables, qkv3, k3, v3, 50, **wide)
    fourth = _Case(torch, tables, qkv4, None, None, 51, share_caches=third, **wide)
    got3 = _no_alloc(torch, third)
    got4 = _no_alloc(torch, fourth)
    for got, expect in ((got3, expect3), (got4, expect4)):
        assert np.isfinite(got[0]).all()
        for g, e in zip(got[:3], expect[:3]):
            np.testing.assert_allclose(g, e, rtol=1e-4, atol=1e-6)
        assert got[3][0] == 0


def test_no_alloc_decode_attention_rejects_requests_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    heads, kv_heads, hd, context = 32, 8, 128, 8192  # 256 splits * 32 * 130 = 1,064,960 > 1 Mi floats
    qkv = torch.zeros((heads + 2 * kv_heads) * hd, device="cuda")
    k_cache = torch.zeros(kv_heads, context, hd, device="cuda")
    v_cache = torch.zeros_like(k_cache)
    mask = torch.zeros(context, device="cuda")
    write = torch.zeros(context, device="cuda")
    position = torch.zeros(1, dtype=torch.int64, device="cuda")
    tables = torch.zeros(2, 16, hd // 2, device="cuda")
    out = torch.zeros(heads * hd, device="cuda")
    a = _lib.DecodeAttentionArgs()
    a.qkv, a.q_off, a.k_off, a.v_off = qkv.data_ptr(), 0, heads * hd, (heads + kv_heads) * hd
    a.heads, a.kv_heads, a.head_size, a.context = heads, kv_heads, hd, context
    a.position, a.position_dtype = position.data_ptr(), _lib.I64
    a.cos_table, a.sin_table, a.n_positions = tables[0].data_ptr(), tables[1].data_ptr(), 16
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.write_mask, a.write_mask_dtype, a.one_minus_dtype = write.data_ptr(), _lib.F32, _lib.F32
    a.mask, a.mask_dtype, a.divisor = mask.data_ptr(), _lib.F32, float(np.sqrt(hd))
    a.out = out.data_ptr()
    with pytest.raises(_lib.KernelError, match="scratch floats"):
        _lib.call("cb_decode_attention_noalloc", ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert not out.any().item()

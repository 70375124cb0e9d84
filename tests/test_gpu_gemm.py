"""cb_gemm_tc (tcgen05 / TMEM / TMA) against a float64 torch reference.

C = A @ B^T with B a bf16 (n, k) weight.  bf16 A: products are exact and the
float32 accumulation is the only rounding.  float32 A: split into bf16 hi +
lo planes, leaving a residual of about 2^-16 of each |a|.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [  # m, n, k: tile tails in m, both tile widths in n, deep and shallow k
    (128, 256, 64),
    (100, 128, 128),
    (300, 512, 2048),
    (257, 384, 5632),
    (2048, 2560, 2048),
    (16, 64, 256),      # tiny: one partial tile in every dimension
    (77, 688, 688),     # k and n tails (688 = 10.75 x 64)
    (130, 260, 200),    # k % 64 = 8, n % 128 = 4
]


def _run(torch, a, b, out=None):
    from cuda_b200 import _lib

    m, k = a.shape
    n = b.shape[0]
    c = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") if out is None else out
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = _lib.GemmArgs()
    g.a, g.lda = a.data_ptr(), a.stride(0)
    g.a_dtype = _lib.F32 if a.dtype == torch.float32 else _lib.BF16
    g.b, g.ldb = b.data_ptr(), b.stride(0)
    g.c, g.ldc = c.data_ptr(), c.stride(0)
    g.m, g.n, g.k = m, n, k
    scratch = _lib.load().cb_gemm_tc_scratch(ctypes.byref(g))
    buf = torch.empty(max(scratch, 16), dtype=torch.uint8, device="cuda")
    g.a_split = buf.data_ptr()
    g.error_flag = flag.data_ptr()
    _lib.call("cb_gemm_tc", ctypes.byref(g), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    return c


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("a_dtype", ["bf16", "f32"])
def test_gemm_tc_matches_float64(m, n, k, a_dtype):
    torch = pytest.importorskip("torch")
    gen = torch.Generator().manual_seed(m * 7 + n * 3 + k)
    a = torch.randn(m, k, generator=gen)
    b = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
    if a_dtype == "bf16":
        a = a.to(torch.bfloat16)
    got = _run(torch, a.cuda(), b.cuda()).cpu().double()
    ref = a.double() @ b.double().T
    scale = (a.double().abs() @ b.double().abs().T)  # bound of each dot product's terms
    err = (got - ref).abs()
    # float32 accumulation over k terms; plus the hi/lo residual for float32 A
    bound = scale * (k * 2.0 ** -23 + (2.0 ** -15 if a_dtype == "f32" else 0.0)) + 1e-6
    assert torch.isfinite(got).all()
    assert bool((err <= bound).all()), float((err / bound).max())


def test_gemm_tc_strided_a_and_c():
    torch = pytest.importorskip("torch")
    gen = torch.Generator().manual_seed(5)
    m, n, k = 200, 256, 256
    a_full = torch.randn(m, k + 64, generator=gen).cuda()
    a = a_full[:, 32:32 + k]  # row stride k + 64, not 16-byte aligned start for bf16 TMA
    b = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    c_full = torch.zeros(m, n + 128, device="cuda")
    c = c_full[:, :n]
    _run(torch, a, b, out=c)
    ref = a.double().cpu() @ b.double().cpu().T
    np.testing.assert_allclose(c.cpu().double().numpy(), ref.numpy(), rtol=1e-4, atol=1e-4)
    assert not c_full[:, n:].any()  # nothing written beyond n


def test_gemm_tc_rejects_unsupported_shapes():
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    a = torch.zeros(64, 90, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(128, 90, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.KernelError, match="multiple of 8"):
        _run(torch, a, b)
    b = torch.zeros(126, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.KernelError, match="multiple of 4"):
        _run(torch, a[:, :80].contiguous(), b[:, :80].contiguous())


ROWS_CASES = [  # rows, weight row counts, k, splits (0 = chosen)
    (1, (2048,), 2048, 0),
    (5, (2048, 256, 256), 2048, 0),
    (32, (5632, 5632), 2048, 0),
    (32, (2048,), 5632, 0),
    (32, (300,), 200, 1),
    (100, (640, 64), 1024, 3),
    (256, (384,), 512, 0),
]


@pytest.mark.parametrize("rows,ns,k,splits", ROWS_CASES)
@pytest.mark.parametrize("x_dtype", ["f32", "bf16"])
def test_gemm_rows_matches_float64(rows, ns, k, splits, x_dtype):
    """cb_gemm_rows (swap-AB, split K, last-CTA reduction) against float64, twice in a row."""
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    gen = torch.Generator().manual_seed(rows * 13 + k + len(ns))
    x = torch.randn(rows, k, generator=gen)
    if x_dtype == "bf16":
        x = x.to(torch.bfloat16)
    ws = [(torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16) for n in ns]
    xd, wd = x.cuda(), [w.cuda() for w in ws]
    outs = [torch.full((rows, n + 8), float("nan"), device="cuda") for n in ns]  # row stride n + 8
    a = _lib.GemmRowsArgs()
    a.x, a.x_dtype, a.ldx = xd.data_ptr(), _lib.F32 if x_dtype == "f32" else _lib.BF16, k
    a.rows, a.k, a.n_w, a.splits = rows, k, len(ns), splits
    for i, (w, o) in enumerate(zip(wd, outs)):
        a.w[i], a.w_rows[i], a.out[i], a.ldo[i] = w.data_ptr(), w.shape[0], o.data_ptr(), o.stride(0)
    lib = _lib.load()
    scratch = torch.empty(lib.cb_gemm_rows_scratch(ctypes.byref(a)), dtype=torch.uint8, device="cuda")
    counters = torch.zeros(lib.cb_gemm_rows_counters(ctypes.byref(a)), dtype=torch.int32, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    a.scratch, a.counters, a.error_flag = scratch.data_ptr(), counters.data_ptr(), flag.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the counters must be re-armed by the first call
        for o in outs:
            o[:, : o.shape[1] - 8].fill_(float("nan"))
        _lib.call("cb_gemm_rows", ctypes.byref(a), stream)
        torch.cuda.synchronize()
        assert int(flag.item()) == 0 and not counters.any()
        for w, o in zip(ws, outs):
            n = w.shape[0]
            got = o[:, :n].cpu().double()
            ref = x.double() @ w.double().T
            scale = x.double().abs() @ w.double().abs().T
            bound = scale * (k * 2.0 ** -23 + (2.0 ** -15 if x_dtype == "f32" else 0.0)) + 1e-6
            assert torch.isfinite(got).all()
            assert bool(((got - ref).abs() <= bound).all()), float(((got - ref).abs() / bound).max())
            assert torch.isnan(o[:, n:]).all()  # nothing written past n


def _multi(torch, a, ws, epilogue, residual=None):
    """cb_gemm_tc_multi: returns the output tensors (row stride n + 8: nothing may land past n)."""
    from cuda_b200 import _lib

    m, k = a.shape
    g = _lib.GemmMultiArgs()
    g.a, g.lda, g.m, g.k = a.data_ptr(), a.stride(0), m, k
    g.a_dtype = _lib.F32 if a.dtype == torch.float32 else _lib.BF16
    g.n_w, g.epilogue = len(ws), epilogue
    outs = []
    for i, w in enumerate(ws):
        g.b[i], g.ldb[i], g.n[i] = w.data_ptr(), w.stride(0), w.shape[0]
    for i in range(1 if epilogue != _lib.GEMM_STORE else len(ws)):
        c = torch.full((m, ws[i].shape[0] + 8), float("nan"), device="cuda")
        g.c[i], g.ldc[i] = c.data_ptr(), c.stride(0)
        outs.append(c)
    if residual is not None:
        g.residual, g.ldr = residual.data_ptr(), residual.stride(0)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    scratch = torch.empty(max(_lib.load().cb_gemm_tc_multi_scratch(ctypes.byref(g)), 16), dtype=torch.uint8,
                          device="cuda")
    g.a_split, g.error_flag = scratch.data_ptr(), flag.data_ptr()
    for _ in range(2):  # twice: a second launch over the same buffers gives the same result
        _lib.call("cb_gemm_tc_multi", ctypes.byref(g), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    for o, w in zip(outs, ws):
        assert torch.isnan(o[:, w.shape[0]:]).all()
    return [o[:, : w.shape[0]].cpu().double() for o, w in zip(outs, ws)]


def _bound(a, w, k, a_dtype):
    scale = a.double().abs() @ w.double().abs().T
    return scale * (k * 2.0 ** -23 + (2.0 ** -15 if a_dtype == "f32" else 0.0)) + 1e-6


@pytest.mark.parametrize("m,ns,k", [(300, (2048, 256, 256), 2048), (130, (260, 128), 200), (64, (688,), 688)])
@pytest.mark.parametrize("a_dtype", ["bf16", "f32"])
def test_gemm_multi_grouped_matches_float64(m, ns, k, a_dtype):
    """q/k/v-style: several weights share A, one launch."""
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    gen = torch.Generator().manual_seed(m + k + len(ns))
    a = torch.randn(m, k, generator=gen)
    if a_dtype == "bf16":
        a = a.to(torch.bfloat16)
    ws = [(torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16) for n in ns]
    got = _multi(torch, a.cuda(), [w.cuda() for w in ws], _lib.GEMM_STORE)
    for g, w in zip(got, ws):
        ref = a.double() @ w.double().T
        assert bool(((g - ref).abs() <= _bound(a, w, k, a_dtype)).all())


@pytest.mark.parametrize("m,n,k", [(300, 512, 2048), (2048, 2048, 5632), (77, 260, 200)])
def test_gemm_multi_residual_matches_float64(m, n, k):
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    gen = torch.Generator().manual_seed(m * 3 + n)
    a = torch.randn(m, k, generator=gen)
    w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
    r = torch.randn(m, n, generator=gen)
    (got,) = _multi(torch, a.cuda(), [w.cuda()], _lib.GEMM_RESIDUAL, residual=r.cuda())
    ref = r.double() + a.double() @ w.double().T
    bound = _bound(a, w, k, "f32") + r.double().abs() * 2.0 ** -23
    assert bool(((got - ref).abs() <= bound).all())


@pytest.mark.parametrize("m,n,k", [(300, 5632, 2048), (2048, 5632, 2048), (100, 688, 256)])
@pytest.mark.parametrize("a_dtype", ["bf16", "f32"])
def test_gemm_multi_swiglu_matches_float64(m, n, k, a_dtype):
    """silu(A Wg^T) * (A Wu^T) in one launch, against float64."""
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    gen = torch.Generator().manual_seed(n + k + m)
    a = torch.randn(m, k, generator=gen)
    if a_dtype == "bf16":
        a = a.to(torch.bfloat16)
    wg = (torch.randn(n, k, generator=gen) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(n, k, generator=gen) * 0.05).to(torch.bfloat16)
    (got,) = _multi(torch, a.cuda(), [wg.cuda(), wu.cuda()], _lib.GEMM_SWIGLU)
    g = a.double() @ wg.double().T
    u = a.double() @ wu.double().T
    ref = g / (1 + torch.exp(-g)) * u
    bg, bu = _bound(a, wg, k, a_dtype), _bound(a, wu, k, a_dtype)
    silu = (g / (1 + torch.exp(-g))).abs()
    bound = 1.2 * bg * (u.abs() + bu) + (silu + 1.2 * bg) * bu + 4 * 2.0 ** -23 * ref.abs() + 1e-6
    assert torch.isfinite(got).all()
    assert bool(((got - ref).abs() <= bound).all()), float(((got - ref).abs() / bound).max())

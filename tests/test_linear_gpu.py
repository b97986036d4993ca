"""Parity of the CUDA linear (split-int8 tcgen05 GEMM) with the oracle.

Mirrors the reference's matrix-product tests (src/kernels/mod.rs:962-1128): shapes with ragged
edges, every epilogue, accumulate, and the config-1 shape. Three bars:
  * the quantized activations and the two int32 sums are bit-exact against the oracle;
  * the scaled output equals the oracle's step-for-step restatement of the CUDA epilogue bit for
    bit (act none/relu) or within 1e-5 relative (SiLU, which the epilogue computes with the
    approximate exponential and reciprocal and a contracted scale-and-bias step);
  * against the reference's own f32 path (int8 weights widened, f32 activations), each output
    matrix is within 1e-3 max-relative: max|got - ref| / max|ref| <= 1e-3.
"""

import numpy as np
import pytest

from telmo_b200 import synthetic

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (1, 7, 5), (5, 13, 17), (6, 64, 16), (7, 33, 31), (13, 100, 50),
          (64, 128, 96), (129, 300, 257), (200, 1024, 384), (300, 2049, 130)]


def _case(m, k, n, seed):
    g = synthetic.rng(seed)
    a = g.standard_normal((m, k), dtype=np.float32)
    values, scales, _, _ = synthetic.int8_matrix(g, n, k)
    bias = (g.standard_normal(n) * 0.02).astype(np.float32)
    c0 = g.standard_normal((m, n), dtype=np.float32)
    return a, values, scales, bias, c0


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _upload(ctx, values, scales, n, k):
    from telmo_b200 import PackedWeights, Precision
    return PackedWeights(n, k, Precision.INT8, values, scales).upload(ctx)


def max_rel(got, ref):
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_quantized_activations_are_bit_exact(ctx, oracle_lib, m, k, n):
    import torch
    from telmo_b200 import Kernels
    a, *_ = _case(m, k, n, 1)
    ldq = (k + 15) // 16 * 16
    hi = torch.zeros((m, ldq), dtype=torch.int8, device="cuda")
    lo = torch.zeros_like(hi)
    s = torch.zeros(m, dtype=torch.float32, device="cuda")
    Kernels(ctx).quantize_x2(_dev(a), k, m, k, hi, lo, ldq, s)
    ctx.check()
    whi, wlo, ws = oracle_lib.quantize_x2(a)
    assert np.array_equal(hi.cpu().numpy()[:, :k], whi)
    assert np.array_equal(lo.cpu().numpy()[:, :k], wlo)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    assert not hi.cpu().numpy()[:, k:].any()


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_int32_sums_are_bit_exact(ctx, oracle_lib, m, k, n):
    import torch
    from telmo_b200 import DType, Kernels
    a, values, scales, bias, _ = _case(m, k, n, 2)
    w = _upload(ctx, values, scales, n, k)
    out = torch.zeros((2, m, n), dtype=torch.int32, device="cuda")
    Kernels(ctx).matmul(_dev(a), k, m, w, out, n, out_dtype=DType.I32_PAIR)
    ctx.check()
    hi, lo, _ = oracle_lib.quantize_x2(a)
    want_hi, want_lo = oracle_lib.gemm_i8_x2_acc(hi, lo, values, n, k)
    got = out.cpu().numpy()
    assert np.array_equal(got[0], want_hi)
    assert np.array_equal(got[1], want_lo)


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("act,accumulate,with_bias,scale", [
    (0, False, False, 1.0), (1, False, True, 0.5), (2, True, True, 0.5), (0, True, False, 0.5)])
def test_linear_matches_the_oracle(ctx, oracle_lib, m, k, n, act, accumulate, with_bias, scale):
    from telmo_b200 import Act, Epilogue, Kernels
    a, values, scales, bias, c0 = _case(m, k, n, 3)
    w = _upload(ctx, values, scales, n, k)
    b = bias if with_bias else None
    c = _dev(c0)
    Kernels(ctx).linear(_dev(a), m, w, c, Epilogue(bias=None if b is None else _dev(b),
                                                   act=Act(act), scale=scale,
                                                   accumulate=accumulate))
    ctx.check()
    got = c.cpu().numpy()
    exact = oracle_lib.linear_x2(a, values, scales, n, k, b, act, scale, c0, accumulate)
    if act == 2:
        assert np.allclose(got, exact, rtol=1e-5, atol=1e-6)
    else:
        assert np.array_equal(got.view(np.uint32), exact.view(np.uint32))
    ref = oracle_lib.linear_int8(a, values, scales, n, k, b, act, scale, c0, accumulate)
    assert max_rel(got, ref) <= 1e-3


def test_config1_full_size(ctx, oracle_lib):
    """Config 1 (benches/matmul.rs shape): A [1500, 1024] f32, W int8 [4096, 1024], bias."""
    import torch
    from telmo_b200 import DType, Epilogue, Kernels
    a, (values, scales, n, k), bias = synthetic.config1()
    m = a.shape[0]
    w = _upload(ctx, values, scales, n, k)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    kern = Kernels(ctx)
    kern.linear(_dev(a), m, w, c, Epilogue(bias=_dev(bias)))
    sums = torch.zeros((2, m, n), dtype=torch.int32, device="cuda")
    kern.matmul(_dev(a), k, m, w, sums, n, out_dtype=DType.I32_PAIR)
    ctx.check()
    got = c.cpu().numpy()
    ref = oracle_lib.linear_int8(a, values, scales, n, k, bias, threads=8)
    assert max_rel(got, ref) <= 1e-3
    # int32 sums bit-exact on a sample of rows (the full oracle triple loop takes minutes).
    rows = np.array([0, 1, 127, 128, 500, 1023, 1499])
    hi, lo, s = oracle_lib.quantize_x2(a[rows])
    want_hi, want_lo = oracle_lib.gemm_i8_x2_acc(hi, lo, values, n, k)
    got_sums = sums.cpu().numpy()
    assert np.array_equal(got_sums[0][rows], want_hi)
    assert np.array_equal(got_sums[1][rows], want_lo)


def test_bf16_output(ctx, oracle_lib):
    import torch
    from telmo_b200 import Epilogue, Kernels
    m, k, n = 77, 256, 200
    a, values, scales, bias, _ = _case(m, k, n, 4)
    w = _upload(ctx, values, scales, n, k)
    c = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    Kernels(ctx).linear(_dev(a), m, w, c, Epilogue(bias=_dev(bias)))
    ctx.check()
    exact = oracle_lib.linear_x2(a, values, scales, n, k, bias)
    want = torch.from_numpy(exact).to(torch.bfloat16).float().numpy()
    assert np.array_equal(c.float().cpu().numpy(), want)


# ---- Q8_0 weights (src/quant.rs:8-13): one scale per 32 inputs of each output ---------------------

Q8_SHAPES = [(1, 32, 1), (5, 64, 17), (7, 96, 31), (129, 320, 257), (200, 1024, 384),
             (300, 2048, 130), (64, 4096, 96)]


def _q8_case(m, k, n, seed):
    # Rows and blocks of very different magnitudes, so the blocks' scales matter.
    g = synthetic.rng(seed)
    a = g.standard_normal((m, k), dtype=np.float32)
    w = g.standard_normal((n, k)) * np.exp(g.standard_normal((n, 1)))
    w = (w * np.repeat(np.exp(g.standard_normal((n, k // 32))), 32, axis=1) / np.sqrt(k)).astype(np.float32)
    values, scales = synthetic.q8_0_panels(w)
    bias = (g.standard_normal(n) * 0.02).astype(np.float32)
    c0 = g.standard_normal((m, n), dtype=np.float32)
    return a, values, scales, bias, c0


def _upload_q8(ctx, values, scales, n, k):
    from telmo_b200 import PackedWeights, Precision
    return PackedWeights(n, k, Precision.Q8_0, values, scales).upload(ctx)


@pytest.mark.parametrize("m,k,n", Q8_SHAPES)
@pytest.mark.parametrize("act,accumulate,with_bias,scale", [
    (0, False, False, 1.0), (1, False, True, 0.5), (2, True, True, 0.5), (0, True, False, 0.5)])
def test_q8_0_linear_matches_the_oracle(ctx, oracle_lib, m, k, n, act, accumulate, with_bias, scale):
    # Bit-exact against the restated GPU arithmetic (two-level weights, split activations), and
    # within the north star's 1e-3 max-relative of the reference's exact Q8_0 product.
    from telmo_b200 import Act, Epilogue, Kernels
    a, values, scales, bias, c0 = _q8_case(m, k, n, 5)
    w = _upload_q8(ctx, values, scales, n, k)
    b = bias if with_bias else None
    c = _dev(c0)
    Kernels(ctx).linear(_dev(a), m, w, c, Epilogue(bias=None if b is None else _dev(b),
                                                   act=Act(act), scale=scale,
                                                   accumulate=accumulate))
    ctx.check()
    got = c.cpu().numpy()
    exact = oracle_lib.linear_x2_q8_0(a, values, scales, n, k, b, act, scale, c0, accumulate)
    if act == 2:
        assert np.allclose(got, exact, rtol=1e-5, atol=1e-6)
    else:
        assert np.array_equal(got.view(np.uint32), exact.view(np.uint32))
    ref = oracle_lib.linear_q8_0(a, values, scales, n, k, b, act, scale, c0, accumulate)
    assert max_rel(got, ref) <= 1e-3


def test_q8_0_config1_shape(ctx, oracle_lib):
    """Config 1's shape with Q8_0 weights: the reference's product within 2e-4 max-relative and
    the i32 sums (hi . W_hi, lo . W_hi + hi . W_lo) bit-exact on sampled rows."""
    import torch
    from telmo_b200 import DType, Epilogue, Kernels
    a, (v8, s8, n, k), bias = synthetic.config1()
    m = a.shape[0]
    w = synthetic.rows_from_panels(v8, n, k).astype(np.float32) * s8[:n, None]
    values, scales = synthetic.q8_0_panels(w)
    dw = _upload_q8(ctx, values, scales, n, k)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    kern = Kernels(ctx)
    kern.linear(_dev(a), m, dw, c, Epilogue(bias=_dev(bias)))
    sums = torch.zeros((2, m, n), dtype=torch.int32, device="cuda")
    kern.matmul(_dev(a), k, m, dw, sums, n, out_dtype=DType.I32_PAIR)
    ctx.check()
    ref = oracle_lib.linear_q8_0(a, values, scales, n, k, bias, threads=8)
    assert max_rel(c.cpu().numpy(), ref) <= 2e-4
    rows = np.array([0, 1, 127, 128, 777, 1499])
    hi, lo, _ = oracle_lib.quantize_x2(a[rows])
    w_hi, w_lo, _ = oracle_lib.q8_0_two_level(values, scales, n, k)
    want_hi, want_lo = oracle_lib.gemm_i8_x2w_acc(hi, lo, w_hi, w_lo, n, k)
    got_sums = sums.cpu().numpy()
    assert np.array_equal(got_sums[0][rows], want_hi)
    assert np.array_equal(got_sums[1][rows], want_lo)


def test_q8_0_inputs_must_be_whole_blocks(ctx):
    import ctypes
    from telmo_b200 import _lib
    values = np.zeros(16 * 48, np.int8)
    scales = np.zeros(16 * 2, np.float32)
    h = ctypes.c_void_p()
    rc = _lib.load().telmo_weights_upload(ctx.handle, _lib.precision_code("q8_0"), 16, 48,
                                          values.ctypes.data, scales.ctypes.data, ctypes.byref(h))
    assert rc == _lib.TELMO_ERR_ARGUMENT
    rc = _lib.load().telmo_weights_upload(ctx.handle, _lib.precision_code("f16"), 16, 48,
                                          values.ctypes.data, scales.ctypes.data, ctypes.byref(h))
    assert rc == _lib.TELMO_ERR_UNSUPPORTED


def test_bad_arguments_are_errors_not_crashes(ctx):
    import torch
    from telmo_b200 import Epilogue, Kernels, TelmoError
    a, values, scales, bias, _ = _case(4, 32, 16, 5)
    w = _upload(ctx, values, scales, 16, 32)
    c = torch.zeros((4, 16), dtype=torch.float32, device="cuda")
    kern = Kernels(ctx)
    with pytest.raises(TelmoError):
        kern.matmul(_dev(a), 31, 4, w, c, 16)           # lda below k
    with pytest.raises(TelmoError):
        kern.matmul(_dev(a), 32, 4, w, c, 15)           # ldc below n
    with pytest.raises(TelmoError):
        kern.linear(None, 4, w, c)                       # null input
    kern.linear(_dev(a), 0, w, c, Epilogue.PLAIN)        # m = 0 is a no-op
    ctx.check()


def test_quantize_x2_refuses_unaligned_levels(ctx):
    # The quantizer stores the levels four bytes at a time and the product reads them through
    # 16-byte aligned tensor maps: an offset hi or lo pointer is an argument error, found on the
    # host before anything is launched, and the context stays usable.
    import torch
    from telmo_b200 import _lib
    m, k, ldq = 8, 64, 64
    a = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    buf = torch.zeros(2 * m * ldq + 64, dtype=torch.int8, device="cuda")
    s = torch.zeros(m, dtype=torch.float32, device="cuda")
    L = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    hi, lo = buf.data_ptr(), buf.data_ptr() + m * ldq
    for bad_hi, bad_lo in [(hi + 4, lo), (hi, lo + 8), (hi + 1, lo + 1)]:
        rc = L.telmo_quantize_x2(ctx.handle, a.data_ptr(), k, m, k, bad_hi, bad_lo, ldq, s.data_ptr(), stream)
        assert rc == _lib.TELMO_ERR_ARGUMENT
        assert b"aligned" in L.telmo_last_error(ctx.handle)
    assert L.telmo_quantize_x2(ctx.handle, a.data_ptr(), k, m, k, hi, lo, ldq, s.data_ptr(), stream) == 0
    ctx.check()

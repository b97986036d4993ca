"""telmo_linear_noalloc: the matrix product for callers that cannot let a library allocate device
memory (a service that gives all device memory to its own pool or fixed budget up front, or a
latency-critical stream that cannot take the device-wide synchronisation cudaMalloc and cudaFree
imply). Its quantization scratch is a fixed array compiled into the library.

Called through the C ABI, it must give exactly what telmo_linear gives, on calls in a row (each
smaller than config 1's first, so stale scratch from an earlier call would show), for Int8 and
Q8_0 weights and f32 and bf16 outputs, and must refuse a product too large for the fixed
scratch. This file is collected last.
"""

import ctypes

import numpy as np
import pytest

from telmo_b200 import _lib, synthetic

pytestmark = pytest.mark.gpu


def _noalloc(ctx, a, m, w, c, bias=None, act=0, scale=1.0, accumulate=0, dtype=0):
    import torch
    return _lib.load().telmo_linear_noalloc(
        ctx.handle, a.data_ptr(), w.k, m, w.handle, None if bias is None else bias.data_ptr(), act,
        scale, accumulate, c.data_ptr(), dtype, w.n, torch.cuda.current_stream().cuda_stream)


def _linear(ctx, a, m, w, c, bias=None, act=0, scale=1.0, accumulate=0, dtype=0):
    import torch
    return _lib.load().telmo_linear(
        ctx.handle, a.data_ptr(), w.k, m, w.handle, None if bias is None else bias.data_ptr(), act,
        scale, accumulate, c.data_ptr(), dtype, w.n, torch.cuda.current_stream().cuda_stream)


def _case(ctx, m, k, n, seed, precision="int8"):
    import torch
    from telmo_b200 import PackedWeights, Precision
    g = synthetic.rng(seed)
    a = torch.from_numpy(g.standard_normal((m, k), dtype=np.float32)).cuda()
    entry = synthetic.int8_matrix(g, n, k)
    if precision == "q8_0":  # the same rows re-quantized per block of 32 inputs
        values, scales = synthetic.as_q8_0(entry)[:2]
        prec = Precision.Q8_0
    else:
        values, scales = entry[:2]
        prec = Precision.INT8
    bias = torch.from_numpy((g.standard_normal(n) * 0.02).astype(np.float32)).cuda()
    w = PackedWeights(n, k, prec, values, scales).upload(ctx)
    return a, w, bias


# (m, k, n, act, accumulate, output dtype, weight precision, seed): config 1's shape first, then
# a smaller, ragged product with another epilogue, a Q8_0 product (the kernel's two-level weight
# path) and a bf16 output, each call right after the one before it.
CASES = [(1500, 1024, 4096, 0, 0, _lib.DTYPE_F32, "int8", 1),
         (77, 2049, 130, 2, 1, _lib.DTYPE_F32, "int8", 2),
         (300, 1024, 384, 1, 0, _lib.DTYPE_F32, "q8_0", 4),
         (129, 512, 256, 0, 0, _lib.DTYPE_BF16, "int8", 5)]


def test_noalloc_matches_telmo_linear_on_calls_in_a_row():
    import torch
    import telmo_b200
    ctx = telmo_b200.Context(0)
    for (m, k, n, act, accumulate, dtype, precision, seed) in CASES:
        a, w, bias = _case(ctx, m, k, n, seed, precision)
        tdtype = torch.bfloat16 if dtype == _lib.DTYPE_BF16 else torch.float32
        start = torch.from_numpy(synthetic.rng(seed + 10).standard_normal(
            (m, n), dtype=np.float32)).cuda().to(tdtype)
        want = start.clone()
        got = start.clone()
        assert _linear(ctx, a, m, w, want, bias, act, 0.5, accumulate, dtype) == 0, \
            _lib.load().telmo_last_error(ctx.handle)
        assert _noalloc(ctx, a, m, w, got, bias, act, 0.5, accumulate, dtype) == 0, \
            _lib.load().telmo_last_error(ctx.handle)
        ctx.check()
        assert torch.equal(got, want), (m, k, n, precision, dtype)
        w.free()
    ctx.close()


def test_noalloc_refuses_products_beyond_its_scratch():
    import torch
    import telmo_b200
    ctx = telmo_b200.Context(0)
    a, w, bias = _case(ctx, 1024, 4096, 16, 3)   # 1024 rows at k = 4096: just over 8 MiB
    c = torch.zeros((1024, 16), dtype=torch.float32, device="cuda")
    rc = _noalloc(ctx, a, 1024, w, c, bias)
    assert rc == _lib.TELMO_ERR_ARGUMENT
    assert b"scratch" in _lib.load().telmo_last_error(ctx.handle)
    assert _noalloc(ctx, a, 1023, w, c, bias) == 0  # 1023 rows fit
    ctx.check()
    w.free()
    ctx.close()

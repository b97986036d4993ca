"""telmo_linear_noalloc: the matrix product for callers that cannot let a library allocate device
memory (a service that gives all device memory to its own pool or fixed budget up front, or a
latency-critical stream that cannot take the device-wide synchronisation cudaMalloc and cudaFree
imply). Its quantization scratch is a fixed array compiled into the library.

Called through the C ABI, it must give exactly what telmo_linear gives, on two calls in a row
(the second smaller than the first, so stale scratch from the first would show), and must refuse
a product too large for the fixed scratch. This file is collected last.
"""

import ctypes

import numpy as np
import pytest

from telmo_b200 import _lib, synthetic

pytestmark = pytest.mark.gpu


def _noalloc(ctx, a, m, w, c, bias=None, act=0, scale=1.0, accumulate=0):
    import torch
    return _lib.load().telmo_linear_noalloc(
        ctx.handle, a.data_ptr(), w.k, m, w.handle, None if bias is None else bias.data_ptr(), act,
        scale, accumulate, c.data_ptr(), 0, w.n, torch.cuda.current_stream().cuda_stream)


def _linear(ctx, a, m, w, c, bias=None, act=0, scale=1.0, accumulate=0):
    import torch
    return _lib.load().telmo_linear(
        ctx.handle, a.data_ptr(), w.k, m, w.handle, None if bias is None else bias.data_ptr(), act,
        scale, accumulate, c.data_ptr(), 0, w.n, torch.cuda.current_stream().cuda_stream)


def _case(ctx, m, k, n, seed):
    import torch
    from telmo_b200 import PackedWeights, Precision
    g = synthetic.rng(seed)
    a = torch.from_numpy(g.standard_normal((m, k), dtype=np.float32)).cuda()
    values, scales, _, _ = synthetic.int8_matrix(g, n, k)
    bias = torch.from_numpy((g.standard_normal(n) * 0.02).astype(np.float32)).cuda()
    w = PackedWeights(n, k, Precision.INT8, values, scales).upload(ctx)
    return a, w, bias


def test_noalloc_matches_telmo_linear_on_two_calls_in_a_row():
    import torch
    import telmo_b200
    ctx = telmo_b200.Context(0)
    # Config 1's shape first, then a smaller, ragged product with a different epilogue.
    for (m, k, n, act, accumulate, seed) in [(1500, 1024, 4096, 0, 0, 1), (77, 2049, 130, 2, 1, 2)]:
        a, w, bias = _case(ctx, m, k, n, seed)
        start = torch.from_numpy(synthetic.rng(seed + 10).standard_normal(
            (m, n), dtype=np.float32)).cuda()
        want = start.clone()
        got = start.clone()
        assert _linear(ctx, a, m, w, want, bias, act, 0.5, accumulate) == 0
        assert _noalloc(ctx, a, m, w, got, bias, act, 0.5, accumulate) == 0, \
            _lib.load().telmo_last_error(ctx.handle)
        ctx.check()
        assert torch.equal(got, want)
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

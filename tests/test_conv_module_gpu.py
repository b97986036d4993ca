"""The convolution module's row kernels through telmo_conv_module_rows.

The rows against the oracle's restatement of the reference's glu, dwconv1d_frame and silu
(src/kernels/scalar.rs:149-187) within 1e-5 relative: the tap sums are the reference's, and the
exponentials and divisions are the fast ones, a few ulp from expf and IEEE division. Shapes:
Granite's (2048 channels, kernel 15, stride 1 and 2), Parakeet's (1024, kernel 9), channel counts
that leave the last block of 128 partial, and frame counts from 1 to several tasks of 32 output
frames, with every remainder of the 4-frame output groups.
"""

import numpy as np
import pytest

from telmo_b200 import Kernels, synthetic

pytestmark = pytest.mark.gpu

SHAPES = [  # channels, kernel, stride, frames
    (2048, 15, 1, 100),
    (2048, 15, 2, 77),
    (1024, 9, 1, 33),
    (1024, 9, 1, 1),
    (256, 5, 1, 31),
    (300, 7, 1, 46),
    (200, 3, 2, 3),
    (1536, 15, 2, 130),
    (64, 11, 1, 35),
    (301, 7, 1, 40),
    (1535, 15, 1, 70),
]


def _oracle_rows(oracle_lib, x, frames, channels, kernel, stride, w, bias):
    lib = oracle_lib.lib()
    glu = np.zeros((frames, channels), np.float32)
    for f in range(frames):
        a = np.ascontiguousarray(x[f, :channels])
        b = np.ascontiguousarray(x[f, channels:])
        out = np.zeros(channels, np.float32)
        lib.oracle_glu(a, b, out, channels)
        glu[f] = out
    n_out = frames // 2 if stride == 2 else frames
    rows = np.zeros((n_out, channels), np.float32)
    flat = np.ascontiguousarray(glu.reshape(-1))
    for r in range(n_out):
        out = np.zeros(channels, np.float32)
        lib.oracle_dwconv1d_frame(flat, channels, frames, stride * r, w.reshape(-1), kernel, bias, out)
        lib.oracle_silu(out, channels)
        rows[r] = out
    return rows


@pytest.mark.parametrize("channels,kernel,stride,frames", SHAPES)
def test_conv_rows_match_the_oracle(ctx, oracle_lib, channels, kernel, stride, frames):
    import torch
    g = synthetic.rng(channels * 131 + kernel * 7 + stride + frames)
    x = g.standard_normal((frames, 2 * channels)).astype(np.float32)
    w = (0.3 * g.standard_normal((kernel, channels))).astype(np.float32)
    bias = (0.1 * g.standard_normal(channels)).astype(np.float32)
    n_out = frames // 2 if stride == 2 else frames
    kern = Kernels(ctx)
    xd, wd, bd = (torch.from_numpy(v).cuda() for v in (x, w, bias))
    out = torch.full((n_out + 1, channels), 7.0, device="cuda")  # one guard row past the output
    kern.conv_module_rows(xd, frames, channels, kernel, stride, wd, bd, out)
    torch.cuda.synchronize()
    ctx.check()
    got = out.cpu().numpy()
    want = _oracle_rows(oracle_lib, x, frames, channels, kernel, stride, w, bias)
    assert np.allclose(got[:n_out], want, rtol=1e-5, atol=1e-6)
    assert np.all(got[n_out] == 7.0)


def test_conv_module_rows_refusals(ctx):
    import torch
    from telmo_b200 import TelmoError
    kern = Kernels(ctx)
    x = torch.zeros(8, 2 * 1024, device="cuda")
    w = torch.zeros(15, 1024, device="cuda")
    b = torch.zeros(1024, device="cuda")
    out = torch.zeros(8, 1024, device="cuda")
    with pytest.raises(TelmoError):  # even kernel
        kern.conv_module_rows(x, 8, 1024, 4, 1, w, b, out)
    with pytest.raises(TelmoError):  # stride 3
        kern.conv_module_rows(x, 8, 1024, 15, 3, w, b, out)
    with pytest.raises(TelmoError):  # no output
        kern.conv_module_rows(x, 8, 1024, 15, 1, w, b, None)
    ctx.check()


@pytest.mark.parametrize("channels,kernel,frames", [(2048, 15, 100), (1024, 9, 65), (256, 5, 7)])
def test_two_channel_kernel_gives_the_one_channel_kernels_bits(ctx, channels, kernel, frames):
    # 8-byte aligned rows of an even channel count take the two-channel kernel; the same rows one
    # float into a larger buffer (4-byte aligned) take the one-channel kernel. Same bits.
    import torch
    g = torch.Generator(device="cuda").manual_seed(channels + kernel + frames)
    kern = Kernels(ctx)

    def run(offset):
        x = torch.empty(frames * 2 * channels + 1, device="cuda")
        w = torch.empty(kernel * channels + 1, device="cuda")
        b = torch.empty(channels + 1, device="cuda")
        o = torch.empty(frames * channels + 1, device="cuda")
        xs, ws, bs, os_ = (t[offset:offset + n] for t, n in ((x, frames * 2 * channels), (w, kernel * channels),
                                                             (b, channels), (o, frames * channels)))
        xs.copy_(xin.reshape(-1))
        ws.copy_(win.reshape(-1))
        bs.copy_(bin_)
        kern.conv_module_rows(xs, frames, channels, kernel, 1, ws, bs, os_)
        return os_.clone()

    xin = torch.randn(frames, 2 * channels, device="cuda", generator=g)
    win = 0.3 * torch.randn(kernel, channels, device="cuda", generator=g)
    bin_ = 0.1 * torch.randn(channels, device="cuda", generator=g)
    pair, single = run(0), run(1)
    torch.cuda.synchronize()
    ctx.check()
    assert torch.equal(pair.view(torch.int32), single.view(torch.int32))

"""Pins the oracle (the CPU restatement of telmo's CPU path) to the reference's own known answers.

Each test restates a reference unit test or golden check, cited by file:line in the telmo
source tree. The golden feature tensors are read in place from a copy of the reference source
when one is present (tests/refdata.py); otherwise those two tests skip.
"""

import ctypes
import ctypes.util
import math

import numpy as np
import pytest

import refdata


def xorshift(n, seed):
    """The reference's test generator `random(len, seed)` (src/kernels/mod.rs:795-805)."""
    s = (seed * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF | 1
    out = np.empty(n, np.float32)
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 7
        s ^= (s << 17) & 0xFFFFFFFFFFFFFFFF
        out[i] = np.float32((s >> 40) / float(1 << 24)) * np.float32(2.0) - np.float32(1.0)
    return out


# ---- front ends: golden features (tests/granite_goldens.rs:142-194, tests/goldens.rs:133-176) --

@pytest.mark.skipif(not refdata.available(), reason="no copy of the reference's golden files")
def test_granite_features_match_the_reference_goldens(oracle_lib):
    checked = 0
    for cid, samples, tensors in refdata.clips("granite-speech-5.0-470m-turboctc"):
        if "features" not in tensors:
            continue
        want = tensors["features"].astype(np.float32)
        got = oracle_lib.granite_features(samples)
        assert got.shape == want.shape, cid
        err = np.abs(got - want)
        assert err.mean() <= 5e-7, (cid, err.mean())   # FEATURES_MEAN_ABS
        assert err.max() <= 5e-5, (cid, err.max())     # FEATURES_MAX_ABS
        checked += 1
    assert checked >= 5


@pytest.mark.skipif(not refdata.available(), reason="no copy of the reference's golden files")
def test_parakeet_features_match_the_reference_goldens(oracle_lib):
    checked = 0
    for cid, samples, tensors in refdata.clips("parakeet-tdt-0.6b-v3"):
        valid = int(tensors["features_len"].reshape(-1)[0])
        want = tensors["features"].reshape(-1, 128)[:valid]
        got = oracle_lib.parakeet_features(samples)
        assert got.shape[0] == valid, cid
        err = np.abs(got - want)
        assert err.mean() <= 2e-6, (cid, err.mean())
        assert err.max() <= 5e-4, (cid, err.max())
        checked += 1
    assert checked >= 5


def test_granite_rows_pair_frames_and_pad_the_last(oracle_lib):
    # src/granite_features.rs:323-356
    assert oracle_lib.granite_rows_for(16000) == 50
    assert oracle_lib.granite_rows_for(16160) == 51
    i = np.arange(16160)
    samples = (np.sin(i.astype(np.float32) * np.float32(0.05)) * np.float32(0.3)
               + ((i * 7919) % 101).astype(np.float32) / np.float32(1000.0)).astype(np.float32)
    feats = oracle_lib.granite_features(samples)
    assert feats.shape == (51, 320)
    logs = feats.reshape(-1, 160)[:, :80]
    assert logs.min() >= logs.max() - 2.0 - 1e-6
    first, second = feats[0, :160], feats[0, 160:240]
    assert np.array_equal(first[80:160], (second - first[:80]) / np.float32(2.0))
    with pytest.raises(ValueError):
        oracle_lib.granite_features(samples[:300])


def test_parakeet_frames_at_100_per_second(oracle_lib):
    # src/features.rs:446-463
    samples = np.sin(np.arange(16000) * 0.01).astype(np.float32)
    assert oracle_lib.parakeet_features(samples).shape == (100, 128)
    with pytest.raises(ValueError):
        oracle_lib.parakeet_features(samples[:300])


# ---- fft.rs tests (src/fft.rs:141-204) ---------------------------------------------------------

def test_fft_matches_a_direct_dft(oracle_lib):
    rng = np.random.default_rng(7)
    for n in [4, 8, 16, 32, 64, 128, 256, 512, 1024]:
        x = rng.uniform(-1, 1, n)
        got = oracle_lib.real_fft(x)
        t = np.arange(n)
        want = np.array([np.sum(x * np.exp(-2j * np.pi * ((k * t) % n) / n))
                         for k in range(n // 2 + 1)])
        assert np.max(np.abs(got - want)) < 1e-11 * n


def test_a_cosine_lands_in_its_bin(oracle_lib):
    n = 512
    x = np.cos(2 * np.pi * 5 * np.arange(n) / n)
    got = oracle_lib.real_fft(x)
    want = np.zeros(n // 2 + 1)
    want[5] = n / 2
    assert np.max(np.abs(got.real - want)) < 1e-9 and np.max(np.abs(got.imag)) < 1e-9


# ---- quant.rs tests (src/quant.rs:305-455) -----------------------------------------------------

def test_every_half_round_trips_through_f32(oracle_lib):
    L = oracle_lib.lib()
    for h in range(0, 65536, 7):
        f = L.oracle_f16_to_f32(h)
        if math.isnan(f):
            continue
        assert L.oracle_f32_to_f16(f) == h


def test_halves_and_bf16_round_to_nearest_even(oracle_lib):
    L = oracle_lib.lib()
    assert L.oracle_f32_to_f16(1.0 + 2.0 ** -11) == 0x3C00
    assert L.oracle_f32_to_f16(1.0 + 3.0 * 2.0 ** -11) == 0x3C02
    assert L.oracle_f32_to_f16(65520.0) == 0x7C00
    assert L.oracle_f32_to_f16(65519.0) == 0x7BFF
    assert L.oracle_f32_to_f16(2.0 ** -24) == 1
    assert L.oracle_f32_to_f16(2.0 ** -25) == 0
    assert L.oracle_f32_to_f16(1.5 * 2.0 ** -25) == 1
    assert L.oracle_f32_to_f16(-0.0) == 0x8000

    def from_bits(b):
        return float(np.array([b], np.uint32).view(np.float32)[0])
    assert L.oracle_f32_to_bf16(1.0) == 0x3F80
    assert L.oracle_f32_to_bf16(from_bits(0x3F808000)) == 0x3F80
    assert L.oracle_f32_to_bf16(from_bits(0x3F818000)) == 0x3F82
    assert L.oracle_f32_to_bf16(from_bits(0x3F808001)) == 0x3F81


def test_int8_rows_round_trip_within_half_a_step(oracle_lib):
    n, k = 37, 64
    i = np.arange(n * k)
    w = ((((i * 7919) % 1000) / 500.0 - 1.0) * (1.0 + (i // k))).astype(np.float32).reshape(n, k)
    values, scales = oracle_lib.encode_int8(w)
    back = oracle_lib.decode_int8(values, scales, n, k)
    amax = np.abs(w).max(axis=1, keepdims=True)
    assert np.all(np.abs(back - w) <= amax / 127.0 * 0.51)


def test_host_encode_matches_the_oracle(oracle_lib):
    from telmo_b200 import PackedWeights
    w = np.random.default_rng(3).standard_normal((45, 77)).astype(np.float32)
    v, s = oracle_lib.encode_int8(w)
    p = PackedWeights.encode(w, 45, 77)
    assert np.array_equal(p.values, v) and np.array_equal(p.scales, s)


def test_q8_0_rows_round_trip_within_the_reference_tolerance(oracle_lib):
    # src/quant.rs:400-420: Q8_0 rounds with the exact scale and stores it as f16, so a value
    # comes back within 0.6 of a step of its row's amax / 127.
    n, k = 37, 96
    i = np.arange(n * k)
    w = ((((i * 7919) % 1000) / 500.0 - 1.0) * (1.0 + (i // k))).astype(np.float32).reshape(n, k)
    values, scales = oracle_lib.encode_q8_0(w)
    back = oracle_lib.decode_q8_0(values, scales, n, k)
    amax = np.abs(w).max(axis=1, keepdims=True)
    assert np.all(np.abs(back - w) <= amax / 127.0 * 0.6)


def test_q8_0_blocks_are_laid_out_unchanged(oracle_lib):
    # src/quant.rs:424-455: blocks laid out as the pack stores them decode to q * d exactly.
    n, k = 20, 64
    q = (np.arange(n * k) % 255).astype(np.uint8).view(np.int8).reshape(n, k)
    L = oracle_lib.lib()
    d = np.array([L.oracle_f16_to_f32(L.oracle_f32_to_f16(0.01 * (i + 1)))
                  for i in range(n * k // 32)], np.float32).reshape(n, k // 32)
    panels = (n + 15) // 16
    qp = np.zeros((panels * 16, k), np.int8)
    qp[:n] = q
    dp = np.zeros((panels * 16, k // 32), np.float32)
    dp[:n] = d
    values = qp.reshape(panels, 16, k).transpose(0, 2, 1).reshape(-1)
    scales = dp.reshape(panels, 16, k // 32).transpose(0, 2, 1).reshape(-1)
    back = oracle_lib.decode_q8_0(values, scales, n, k)
    assert np.array_equal(back, q.astype(np.float32) * np.repeat(d, 32, axis=1))


def test_q8_0_encoders_agree(oracle_lib):
    from telmo_b200 import PackedWeights, Precision, synthetic
    g = np.random.default_rng(8)
    w = (g.standard_normal((45, 160)) * np.exp(g.standard_normal((45, 1)))).astype(np.float32)
    w[4, 32:64] = 0.0
    v, s = oracle_lib.encode_q8_0(w)
    p = PackedWeights.encode(w, 45, 160, Precision.Q8_0)
    assert np.array_equal(p.values, v) and np.array_equal(p.scales, s)
    v2, s2 = synthetic.q8_0_panels(w)
    assert np.array_equal(v2, v) and np.array_equal(s2, s)


# ---- the matrix product (src/kernels/mod.rs:885-1128) -------------------------------------------

def _reference_f64(a, w, bias, act, scale, c0, accumulate):
    s = a.astype(np.float64) @ w.astype(np.float64).T
    if bias is not None:
        s = s + bias.astype(np.float64)
    if act == 1:
        s = np.maximum(s, 0)
    elif act == 2:
        s = s / (1 + np.exp(-s))
    s = s * scale
    if accumulate:
        s = s + c0
    return s.astype(np.float32)


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (1, 7, 5), (5, 13, 17), (6, 64, 16), (7, 33, 31),
                                   (13, 100, 50), (64, 128, 96)])
def test_matmul_matches_the_f64_reference(oracle_lib, m, k, n):
    a = xorshift(m * k, 1).reshape(m, k)
    w = xorshift(n * k, 2).reshape(n, k)
    bias = xorshift(n, 3)
    c0 = xorshift(m * n, 4).reshape(m, n)
    values, scales = oracle_lib.encode_int8(w)
    wide = oracle_lib.decode_int8(values, scales, n, k)
    for act, accumulate, with_bias in [(0, False, False), (1, False, True), (2, True, True),
                                       (0, True, False)]:
        b = bias if with_bias else None
        got = oracle_lib.linear_int8(a, values, scales, n, k, b, act, 0.5, c0, accumulate)
        want = _reference_f64(a, wide, b, act, 0.5, c0, accumulate)
        assert np.all(np.abs(got - want) <= 1e-5 * math.sqrt(k) * (1 + np.abs(want)))


@pytest.mark.parametrize("m,k,n", [(1, 32, 1), (5, 64, 17), (13, 96, 50), (64, 320, 96)])
def test_q8_0_matmul_matches_the_f64_reference(oracle_lib, m, k, n):
    # The widening is exact (src/kernels/mod.rs:1160-1183), so the Q8_0 product is the f32
    # product of the decoded weights.
    a = xorshift(m * k, 11).reshape(m, k)
    w = xorshift(n * k, 12).reshape(n, k)
    bias = xorshift(n, 13)
    c0 = xorshift(m * n, 14).reshape(m, n)
    values, scales = oracle_lib.encode_q8_0(w)
    wide = oracle_lib.decode_q8_0(values, scales, n, k)
    for act, accumulate, with_bias in [(0, False, False), (1, False, True), (2, True, True)]:
        b = bias if with_bias else None
        got = oracle_lib.linear_q8_0(a, values, scales, n, k, b, act, 0.5, c0, accumulate)
        want = _reference_f64(a, wide, b, act, 0.5, c0, accumulate)
        assert np.all(np.abs(got - want) <= 1e-5 * math.sqrt(k) * (1 + np.abs(want)))


def test_sums_run_in_input_order_with_fma(oracle_lib):
    # The tile contract (src/kernels/mod.rs:885-931): each output is fma(a, w, s) over
    # ascending inputs, whatever the blocking (KC = 256) or the tile rows.
    m, k, n = 11, 600, 35
    a = xorshift(m * k, 40).reshape(m, k)
    w = xorshift(n * k, 41).reshape(n, k)
    values, scales = oracle_lib.encode_int8(w)
    wide = oracle_lib.decode_int8(values, scales, n, k)
    got = oracle_lib.linear_int8(a, values, scales, n, k)
    libm = ctypes.CDLL(ctypes.util.find_library("m"))
    fmaf = libm.fmaf
    fmaf.restype = ctypes.c_float
    fmaf.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]
    want = np.zeros((m, n), np.float32)
    for i in range(m):
        for j in range(n):
            s = 0.0
            for t in range(k):
                s = fmaf(float(a[i, t]), float(wide[j, t]), s)
            want[i, j] = s
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_results_are_bit_identical_across_thread_counts(oracle_lib):
    m, k, n = 50, 300, 200
    a = xorshift(m * k, 7).reshape(m, k)
    values, scales = oracle_lib.encode_int8(xorshift(n * k, 8).reshape(n, k))
    first = None
    for threads in [1, 2, 3, 6, 8]:
        c = oracle_lib.linear_int8(a, values, scales, n, k, act=2, threads=threads)
        if first is None:
            first = c
        assert np.array_equal(first.view(np.uint32), c.view(np.uint32))


# ---- row kernels (src/kernels/mod.rs:1185-1302) --------------------------------------------------

def test_row_kernels(oracle_lib):
    for n in [1, 3, 4, 8, 15, 17, 1030]:
        x = xorshift(n, 9)
        g, b = xorshift(n, 10), xorshift(n, 11)
        ln = oracle_lib.layer_norm(x[None], g, b)[0]
        xd = x.astype(np.float64)
        want = ((xd - xd.mean()) / np.sqrt(xd.var() + 1e-5)).astype(np.float32) * g + b
        assert np.all(np.abs(ln - want) < 1e-5)
        s = oracle_lib.softmax((x * 30)[None])[0]
        assert abs(float(s.sum()) - 1.0) < 1e-5


def test_sigmoid_is_accurate_across_its_range(oracle_lib):
    x = (np.arange(-1000, 1001) * 0.0875).astype(np.float32)
    ones = np.ones_like(x)
    out = np.zeros_like(x)
    oracle_lib.lib().oracle_glu(ones, x, out, x.size)
    want = 1 / (1 + np.exp(-x.astype(np.float64)))
    assert np.all(np.abs(out - want) <= 1e-9 + 5e-7 * want)


def test_depthwise_conv_matches_a_direct_sum(oracle_lib):
    frames, channels, kernel = 11, 24, 9
    inp = xorshift(frames * channels, 12)
    w = xorshift(kernel * channels, 13)
    bias = xorshift(channels, 14)
    for t in range(frames):
        out = np.zeros(channels, np.float32)
        oracle_lib.lib().oracle_dwconv1d_frame(inp, channels, frames, t, w, kernel, bias, out)
        for c in range(channels):
            s = float(bias[c])
            for j in range(kernel):
                src = t + j - kernel // 2
                if 0 <= src < frames:
                    s += float(w[j * channels + c]) * float(inp[src * channels + c])
            assert abs(out[c] - s) < 1e-5


# ---- granite.rs tests ----------------------------------------------------------------------------

def test_ctc_merges_repeats_and_drops_blanks(oracle_lib):
    # src/granite.rs:1195-1203
    got = oracle_lib.ctc_tokens([0, 5, 5, 0, 5, 7, 7, 7, 0, 0, 2])
    assert got == [(5, 1, 2), (5, 4, 1), (7, 5, 3), (2, 10, 1)]
    assert oracle_lib.ctc_tokens([0, 0]) == []


def test_frames_for_halves_per_subsampling_block(oracle_lib):
    from telmo_b200 import synthetic
    c = synthetic.granite_config(layers=2, d_model=32, heads=2, head_dim=16, ff=64,
                                 conv_channels=64, conv_kernel=3, context=8, vocab=9)
    g = oracle_lib.Granite(c, synthetic.granite_entries(c, seed=5))
    assert g.frames_for(337) == 84    # src/granite.rs:1168
    assert g.frames_for(3) == 0


def test_tiny_granite_encodes_deterministically(oracle_lib):
    from telmo_b200 import synthetic
    c = synthetic.granite_config(layers=4, d_model=64, heads=2, head_dim=32, ff=128,
                                 conv_channels=128, conv_kernel=5, context=8, vocab=33,
                                 n_mels=8)
    g = oracle_lib.Granite(c, synthetic.granite_entries(c, seed=6))
    feats = synthetic.rng(7).standard_normal((45, 32)).astype(np.float32)
    out1 = g.encode(feats, threads=1)
    out3 = g.encode(feats, threads=3)
    assert out1.shape == (11, 64)
    assert np.array_equal(out1, out3)
    assert np.all(np.isfinite(out1))
    ids, margin = g.frame_ids(out1)
    assert ids.shape == (11,) and np.all(margin >= 0)
    with pytest.raises(ValueError):
        g.encode(feats[:3])


# ---- parakeet.rs --------------------------------------------------------------------------------

@pytest.mark.skipif(not refdata.available(), reason="no copy of the reference's golden files")
def test_parakeet_frames_for_matches_the_reference_goldens(oracle_lib):
    for cid, _, tensors in refdata.clips("parakeet-tdt-0.6b-v3"):
        feats = int(tensors["features_len"].reshape(-1)[0])
        assert oracle_lib.parakeet_frames_for(feats) == int(tensors["encoded_len"][0]), cid
        assert tensors["subsampling"].shape[0] in (int(tensors["encoded_len"][0]),
                                                   int(tensors["encoded_len"][0]) + 1)


@pytest.mark.skipif(not refdata.available(), reason="no copy of the reference's golden files")
def test_tdt_loop_replays_the_reference_goldens(oracle_lib):
    # The goldens trace the joint's logits of the first decoding steps with the frame each read;
    # feeding them to the greedy TDT step must land on the same frames and emit the same
    # (id, frame, duration) tokens as the reference (tests/goldens.rs:236-269).
    vocab, blank, durations, max_symbols = 8193, 8192, [0, 1, 2, 3, 4], 10
    checked = 0
    for cid, _, tensors in refdata.clips("parakeet-tdt-0.6b-v3"):
        joints, joint_frames = tensors["joint"], tensors["joint_frame"]
        want = list(zip(tensors["tokens"].tolist(), tensors["token_frame"].tolist(),
                        tensors["token_duration"].tolist()))
        t, on, got = 0, 0, []
        for s in range(joints.shape[0]):
            assert t == int(joint_frames[s]), (cid, s)
            tok, t, on = oracle_lib.tdt_step(joints[s], vocab, blank, durations, max_symbols, t,
                                             on)
            if tok is not None:
                got.append(tok)
        assert got and got == want[:len(got)], cid
        checked += 1
    assert checked >= 5


def test_tdt_step_rules(oracle_lib):
    vocab, blank, durs = 4, 3, [0, 1, 2]

    def logits(token, dur):
        v = np.zeros(vocab + len(durs), np.float32)
        v[token] = 1.0
        v[vocab + dur] = 1.0
        return v

    # A blank with duration 0 still moves on one frame; with 2, two.
    assert oracle_lib.tdt_step(logits(3, 0), vocab, blank, durs, 2, 5, 1) == (None, 6, 0)
    assert oracle_lib.tdt_step(logits(3, 2), vocab, blank, durs, 2, 5, 1) == (None, 7, 0)
    # A token with duration 0 stays on the frame until max_symbols tokens came out there.
    assert oracle_lib.tdt_step(logits(1, 0), vocab, blank, durs, 2, 5, 0) == ((1, 5, 0), 5, 1)
    assert oracle_lib.tdt_step(logits(1, 0), vocab, blank, durs, 2, 5, 1) == ((1, 5, 0), 6, 0)
    assert oracle_lib.tdt_step(logits(2, 2), vocab, blank, durs, 2, 5, 1) == ((2, 5, 2), 7, 0)
    # Ties go to the first index (argmax, src/parakeet.rs:1683-1691).
    tie = np.zeros(vocab + len(durs), np.float32)
    assert oracle_lib.tdt_step(tie, vocab, blank, durs, 2, 0, 0) == ((0, 0, 0), 0, 1)


def test_parakeet_positions_are_sinusoids_of_the_offset(oracle_lib):
    # positions (src/parakeet.rs:1618-1630): row r is position t - 1 - r.
    t, d = 7, 16
    pos = oracle_lib.parakeet_positions(t, d)
    assert pos.shape == (2 * t - 1, d)
    p = (t - 1 - np.arange(2 * t - 1, dtype=np.float64))[:, None]
    freq = np.exp(-np.arange(0, d, 2, dtype=np.float64) * (np.log(10000.0) / d))[None, :]
    assert np.allclose(pos[:, 0::2], np.sin(p * freq), rtol=0, atol=1e-7)
    assert np.allclose(pos[:, 1::2], np.cos(p * freq), rtol=0, atol=1e-7)
    assert np.all(pos[t - 1, 0::2] == 0) and np.all(pos[t - 1, 1::2] == 1)
    assert np.array_equal(pos[:t - 1, 0::2], -pos[t:, 0::2][::-1])


def _np_conv3x3s2(x, w, b, depthwise):
    """[t, f, ch] (depthwise) or [t, f] -> [t', f', ch], zero padding 1, taps dt * 3 + df."""
    t, f = x.shape[:2]
    to, fo = (t - 1) // 2 + 1, (f - 1) // 2 + 1
    out = np.tile(b.astype(np.float64), (to, fo, 1))
    xp = np.zeros((t + 2, f + 2) + x.shape[2:], np.float64)
    xp[1:t + 1, 1:f + 1] = x
    for dt in range(3):
        for df in range(3):
            src = xp[dt:dt + 2 * to:2, df:df + 2 * fo:2]
            if not depthwise:
                src = src[..., None]
            out += src * w[dt * 3 + df].astype(np.float64)
    return out


def test_parakeet_subsampling_matches_a_direct_restatement(oracle_lib):
    # Parakeet::subsample (src/parakeet.rs:904-993) in f64 numpy: conv0 + ReLU, depthwise,
    # pointwise + ReLU twice, flatten channel-major (c * freqs + f), linear.
    from telmo_b200 import synthetic
    c = synthetic.parakeet_config(layers=1, d_model=128, heads=2, ff=256, sub_channels=16,
                                  n_mels=32, pred_hidden=32, vocab=17, blank=16)
    e = synthetic.parakeet_entries(c, seed=4, scales="conditioned")
    model = oracle_lib.Parakeet(c, e)
    feats = synthetic.rng(9).standard_normal((37, 32)).astype(np.float32)
    got = model.encode(feats, tap_layer=-2)

    def dense(name):
        v, s, n, k = e[name]
        return oracle_lib.decode_int8(v, s, n, k).astype(np.float64)

    h = np.maximum(_np_conv3x3s2(feats, e["sub.conv0.w"], e["sub.conv0.b"], False), 0)
    h = _np_conv3x3s2(h, e["sub.dw1.w"], e["sub.dw1.b"], True)
    h = np.maximum(h @ dense("sub.pw1").T + e["sub.pw1.b"], 0)
    h = _np_conv3x3s2(h, e["sub.dw2.w"], e["sub.dw2.b"], True)
    h = np.maximum(h @ dense("sub.pw2").T + e["sub.pw2.b"], 0)
    flat = h.transpose(0, 2, 1).reshape(h.shape[0], -1)
    want = flat @ dense("sub.linear").T + e["sub.linear.b"]
    assert got.shape == want.shape == (oracle_lib.parakeet_frames_for(37), 128)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()


def test_tiny_parakeet_is_deterministic_and_decodes_in_order(oracle_lib):
    from telmo_b200 import synthetic
    c = synthetic.parakeet_config(layers=2, d_model=128, heads=2, ff=256, sub_channels=32,
                                  pred_hidden=64, vocab=65, blank=64)
    model = oracle_lib.Parakeet(c, synthetic.parakeet_entries(c, seed=5, scales="conditioned"))
    feats = synthetic.rng(8).standard_normal((203, 128)).astype(np.float32)
    out1 = model.encode(feats, threads=1)
    out3 = model.encode(feats, threads=3)
    assert out1.shape == (26, 128) and np.array_equal(out1, out3)
    tokens, margin = model.decode(out1)
    assert tokens == model.decode(out1, threads=3)[0]
    frames = [f for _, f, _ in tokens]
    assert frames == sorted(frames) and all(0 <= f < 26 for f in frames)
    assert all(i != c["blank"] and i < c["vocab"] for i, _, _ in tokens)
    assert all(d in c["durations"] for _, _, d in tokens)
    assert np.isfinite(margin)


# ---- GraniteStream (src/granite_stream.rs) ----------------------------------------------------------

STREAM = dict(d_model=128, heads=2, head_dim=64, layers=4, ff=256, conv_channels=256, conv_kernel=5,
              context=16, max_relative=32, vocab=33, n_mels=80)


def _stream_model(oracle_lib, seed=7):
    from telmo_b200 import synthetic
    config = synthetic.granite_config(**STREAM)
    return config, oracle_lib.Granite(config, synthetic.granite_entries(config, seed=seed,
                                                                        scales="conditioned"))


def test_one_finished_update_is_the_offline_encode(oracle_lib):
    # The module's promise (src/granite_stream.rs:14-17): a single update over a whole
    # utterance gives exactly what Granite::encode and frame_ids give.
    from telmo_b200 import synthetic
    config, model = _stream_model(oracle_lib)
    audio = synthetic.audio(3.3, seed=5)
    st = oracle_lib.GraniteStream(model)
    st.push(audio)
    st.update(finished=True)
    feats = oracle_lib.granite_features(audio)
    assert np.array_equal(st.features(), feats)
    enc = model.encode(feats)
    assert np.array_equal(st.layer_output(config["layers"] - 1), enc)
    ids, _ = model.frame_ids(enc)
    assert np.array_equal(st.frame_ids(), ids) and st.first_changed() == 0


def test_stream_updates_freeze_and_extend(oracle_lib):
    # Pieces of 0.37 s: frames only grow, every update reports the first frame it may have
    # changed, and frames before the frozen block keep their ids from then on.
    from telmo_b200 import synthetic
    config, model = _stream_model(oracle_lib)
    audio = synthetic.audio(4.1, seed=6)
    st = oracle_lib.GraniteStream(model)
    st.set_freeze_lag(2)
    piece, at, before, frozen_ids = 5920, 0, 0, {}
    while at < audio.size:
        st.push(audio[at:at + piece])
        at += piece
        st.update(finished=at >= audio.size)
        ids = st.frame_ids()
        assert ids.size >= before and st.first_changed() <= before
        for f, v in frozen_ids.items():
            assert ids[f] == v
        for f in range(min(st.frozen(), ids.size)):
            frozen_ids.setdefault(f, ids[f])
        before = ids.size
    assert before == model.frames_for(oracle_lib.granite_rows_for(audio.size)) and len(frozen_ids) > 0

"""The benchmark's random models are chaotic in the reference's own arithmetic (CPU only).

BASELINE's weights (int8 uniform on [-127, 127], per-row scales U(1e-3, 1e-2)) give rows of
standard deviation about 0.4, attention scores of standard deviation in the hundreds and
near-one-hot softmaxes. This test measures, in the oracle (the reference's f32 CPU path
restated), how a relative L2 change of 1e-6 in the input features grows through the encoder
blocks. On the benchmark's weights it grows past the north star's 2e-2 end-to-end bar, so no
implementation that rounds differently from the reference -- the reference on another
instruction set included -- can be held to that bar on those weights; with weights of
trained-layer size (``scales="conditioned"``) it stays near 1e-6. That is why the GPU parity
tests gate the whole encoder on the conditioned weights and only the first blocks on the
benchmark's own.
"""

import numpy as np
import pytest

from telmo_b200 import synthetic


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b))


def _perturbed(f, seed):
    n = synthetic.rng(seed).standard_normal(f.shape)
    return (f + 1e-6 * np.linalg.norm(f) * n / np.linalg.norm(n)).astype(np.float32)


def _growth(model, feats, taps):
    other = _perturbed(feats, 99)
    assert 5e-7 < rel_l2(other, feats) < 2e-6
    return {t: rel_l2(model.encode(other, tap_layer=t, threads=8), model.encode(feats, tap_layer=t, threads=8))
            for t in taps}


def test_granite_benchmark_weights_amplify_rounding(oracle_lib):
    cfg = synthetic.granite_config()
    feats = oracle_lib.granite_features(synthetic.audio(2.0, seed=31))
    spec = _growth(oracle_lib.Granite(cfg, synthetic.granite_entries(cfg, seed=1, scales="spec")),
                   feats, (0, 2, 5, 15))
    cond = _growth(oracle_lib.Granite(cfg, synthetic.granite_entries(cfg, seed=1, scales="conditioned")),
                   feats, (0, 15))
    print("granite spec:", spec, "conditioned:", cond)
    assert spec[15] > 2e-2            # past the end-to-end bar
    assert spec[15] > 1e3 * spec[0]   # and it is the blocks that amplify it
    assert cond[15] < 1e-4


def test_parakeet_benchmark_weights_amplify_rounding(oracle_lib):
    cfg = synthetic.parakeet_config()
    feats = oracle_lib.parakeet_features(synthetic.audio(2.0, seed=31))
    spec = _growth(oracle_lib.Parakeet(cfg, synthetic.parakeet_entries(cfg, seed=3, scales="spec")),
                   feats, (0, 2, 11))
    cond = _growth(oracle_lib.Parakeet(cfg, synthetic.parakeet_entries(cfg, seed=3, scales="conditioned")),
                   feats, (0, 23))
    print("parakeet spec:", spec, "conditioned:", cond)
    assert spec[11] > 2e-2
    assert spec[11] > 1e3 * spec[0]
    assert cond[23] < 1e-4


def _tdt_decode(cfg, entries, enc, oracle, state_eps=0.0):
    """decode_inner (src/parakeet.rs:1412-1513) restated over the oracle's reference products
    (oracle.linear_int8: int8 weights widened, f32 sums), with the LSTM's initial state -- after
    predict(blank) -- perturbed by a relative L2 change of state_eps."""
    h, layers, vocab = cfg["pred_hidden"], cfg["pred_layers"], cfg["vocab"]

    def lin(name, x):
        v, s, n, k = entries[name]
        return oracle.linear_int8(np.ascontiguousarray(x, np.float32), v, s, n, k, entries.get(name + ".b"))

    def sig(x):
        return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)

    state = np.zeros((layers, 2, h), np.float32)

    def predict(tok):
        inp = entries["dec.embedding"][tok]
        for l in range(layers):
            g = lin(f"dec.lstm.{l}", np.concatenate([inp, state[l, 0]])[None])[0]
            c = sig(g[h:2 * h]) * state[l, 1] + sig(g[:h]) * np.tanh(g[2 * h:3 * h])
            state[l, 1], state[l, 0] = c, sig(g[3 * h:]) * np.tanh(c)
            inp = state[l, 0]
        return lin("dec.pred_proj", inp[None])[0]

    pred = predict(cfg["blank"])
    if state_eps:
        n = synthetic.rng(17).standard_normal(state.shape)
        state += (state_eps * np.linalg.norm(state) * n / np.linalg.norm(n)).astype(np.float32)
    ep = lin("dec.enc_proj", enc)
    t, on, out = 0, 0, []
    while t < enc.shape[0]:
        logits = lin("dec.joint", np.maximum(ep[t] + pred, 0.0)[None])[0]
        tok, t, on = oracle.tdt_step(logits, vocab, cfg["blank"], cfg["durations"], cfg["max_symbols"], t, on)
        if tok is not None:
            out.append(tok)
            pred = predict(tok[0])
    return out


def test_parakeet_benchmark_decoder_state_is_chaotic(oracle_lib):
    # The TDT prediction network with the benchmark's weights: its LSTM gates are saturated and
    # the cell state sums them up, so a 1e-6 relative change of the state after predict(blank)
    # changes the greedy tokens within a few tens of tokens, in the reference's own arithmetic.
    # Decoder tokens on those weights can therefore only be compared over their first tokens by
    # any implementation that rounds differently; with weights of trained-layer size the same
    # perturbation changes nothing.
    cfg = synthetic.parakeet_config()
    enc = synthetic.rng(5).standard_normal((374, cfg["d_model"])).astype(np.float32)
    first = {}
    for scales in ("spec", "conditioned"):
        entries = synthetic.parakeet_entries(cfg, seed=3, scales=scales)
        base = _tdt_decode(cfg, entries, enc, oracle_lib)
        other = _tdt_decode(cfg, entries, enc, oracle_lib, state_eps=1e-6)
        first[scales] = next((i for i, (a, b) in enumerate(zip(base, other)) if a != b), min(len(base), len(other)))
        print(scales, "tokens", len(base), "agree on the first", first[scales])
        assert len(base) > 40
        if scales == "conditioned":
            assert base == other
    assert first["spec"] < 100

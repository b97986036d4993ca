"""Parity of the CUDA Parakeet TDT model with the oracle's restatement of Parakeet::encode and
greedy TDT decoding.

Bars (the north star's): the subsampling output, every layer output and the encoder output within
2e-2 relative L2 of the reference's f32 CPU path, and token ids, frames and durations identical
wherever the reference's top-2 logit margin exceeds 1e-2. With weights of trained-layer size the
kernels are also held to 4 * 1e-4 * (1 + layer / 8), four times the bar the reference's own golden
test sets against NeMo (tests/goldens.rs:30-35): each split-int8 product adds up to about 3e-5
relative error, a few times what an f32 product adds. Batched calls must give each utterance what
a call on that utterance alone gives.
"""

import numpy as np
import pytest

from telmo_b200 import synthetic

pytestmark = pytest.mark.gpu

TINY = synthetic.parakeet_config(layers=2, d_model=128, heads=2, ff=256, sub_channels=32,
                                 pred_hidden=64, vocab=65, blank=64)


def rel_l2(got, ref):
    return float(np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref))


def layer_bar(layer):
    """Four times tests/goldens.rs:30-35 (1e-4 for the subsampling output, layer None)."""
    return 4e-4 if layer is None else 4e-4 * (1.0 + layer / 8.0)


def _features(rows, seed, width=128):
    return synthetic.rng(seed).standard_normal((rows, width)).astype(np.float32)


@pytest.fixture(scope="module")
def tiny(ctx, oracle_lib):
    from telmo_b200.parakeet import Parakeet
    entries = synthetic.parakeet_entries(TINY, seed=21, scales="conditioned")
    return Parakeet.from_entries(ctx, TINY, entries), oracle_lib.Parakeet(TINY, entries)


@pytest.mark.parametrize("tap", [-2, 0, 1, -1])
def test_tiny_encoder_layers_match(tiny, tap):
    import torch
    gpu, ref = tiny
    feats = _features(203, 12)
    out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [203], tap_layer=tap)
    gpu.ctx.check()
    want = ref.encode(feats, tap_layer=tap)
    assert out.shape == want.shape and frames[0] == want.shape[0] == 26
    err = rel_l2(out.cpu().numpy(), want)
    assert err <= layer_bar(None if tap == -2 else (tap if tap >= 0 else 1)), err


def test_tiny_batch_equals_single_utterances(tiny):
    import torch
    gpu, ref = tiny
    # Lengths that give 1, 2, 8, 26 and 57 encoder frames, in an unsorted order.
    rows = [203, 1, 57, 9, 450]
    feats = [_features(r, 30 + i) for i, r in enumerate(rows)]
    out, frames = gpu.encode(torch.from_numpy(np.concatenate(feats)).cuda(), rows)
    gpu.ctx.check()
    got = out.cpu().numpy()
    at = 0
    for f, r, fr in zip(feats, rows, frames):
        want = ref.encode(f)
        assert fr == want.shape[0]
        assert rel_l2(got[at:at + fr], want) <= layer_bar(1)
        single, _ = gpu.encode(torch.from_numpy(f).cuda(), [r])
        assert np.array_equal(single.cpu().numpy(), got[at:at + fr])
        at += fr


def _tokens_match(got, want, margin):
    """Token lists equal, unless the oracle saw a top-2 gap at or below 1e-2 somewhere."""
    if margin <= 1e-2:
        return True
    return [tuple(t) for t in got] == [tuple(t) for t in want]


def test_tiny_decode_matches_on_the_oracle_encoding(tiny):
    # Decoding alone: both decoders read the oracle's encoder output.
    import torch
    gpu, ref = tiny
    rows = [203, 57, 450, 9]
    encs = [ref.encode(_features(r, 40 + i)) for i, r in enumerate(rows)]
    frames = [e.shape[0] for e in encs]
    got = gpu.decode(torch.from_numpy(np.concatenate(encs)).cuda(), frames)
    gpu.ctx.check()
    compared = 0
    for e, g in zip(encs, got):
        want, margin = ref.decode(e)
        if margin > 1e-2:
            assert [(t.id, t.frame, t.duration) for t in g] == want
            compared += 1
    assert compared >= 2


def test_tiny_transcribe_matches_the_oracle_pipeline(tiny, oracle_lib):
    gpu, ref = tiny
    seconds = [1.3, 0.4, 2.7]
    utts = [synthetic.audio(s, seed=50 + i) for i, s in enumerate(seconds)]
    got = gpu.transcribe(utts)
    gpu.ctx.check()
    compared = 0
    for u, g in zip(utts, got):
        feats = oracle_lib.parakeet_features(u)
        want, margin = ref.decode(ref.encode(feats))
        assert _tokens_match([(t.id, t.frame, t.duration) for t in g], want, margin)
        compared += margin > 1e-2
    assert compared >= 1


def test_long_utterance_uses_the_large_score_tile(tiny):
    # 40 s of features: 500 encoder frames, a score tile of 500 columns per query row.
    import torch
    gpu, ref = tiny
    feats = _features(4000, 77)
    out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [4000])
    gpu.ctx.check()
    want = ref.encode(feats, threads=8)
    assert frames[0] == 500
    assert rel_l2(out.cpu().numpy(), want) <= layer_bar(1)


def test_bad_entries_and_configs_are_model_errors(ctx):
    from telmo_b200 import TelmoError
    from telmo_b200._lib import TELMO_ERR_MODEL
    from telmo_b200.parakeet import Parakeet
    with pytest.raises(TelmoError) as e:
        Parakeet(ctx, dict(TINY, blank=3))
    assert e.value.status == TELMO_ERR_MODEL
    entries = synthetic.parakeet_entries(TINY, seed=22)
    partial = {k: v for k, v in entries.items() if k != "layers.1.pos"}
    with pytest.raises(TelmoError) as e:
        Parakeet.from_entries(ctx, TINY, partial)
    assert e.value.status == TELMO_ERR_MODEL and "layers.1.pos" in str(e.value)
    with pytest.raises(TelmoError) as e:
        Parakeet.from_entries(ctx, TINY, dict(entries, **{"layers.0.nope": entries["layers.0.pos"]}))
    assert e.value.status == TELMO_ERR_MODEL


# ---- the benchmark's model shape ------------------------------------------------------------------

@pytest.fixture(scope="module")
def full(ctx, oracle_lib):
    from telmo_b200.parakeet import Parakeet
    config = synthetic.parakeet_config()
    entries = synthetic.parakeet_entries(config, seed=3, scales="conditioned")
    return Parakeet.from_entries(ctx, config, entries), oracle_lib.Parakeet(config, entries)


def test_full_size_layers_match(full):
    import torch
    gpu, ref = full
    feats = _features(520, 91)
    for tap in (-2, 0, 11, 23):
        out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [520], tap_layer=tap)
        gpu.ctx.check()
        want = ref.encode(feats, tap_layer=tap, threads=8)
        assert frames[0] == want.shape[0] == 65
        err = rel_l2(out.cpu().numpy(), want)
        assert err <= 2e-2, (tap, err)                                   # north star
        assert err <= layer_bar(None if tap == -2 else tap), (tap, err)


def test_full_size_transcribe_matches_the_oracle(full, oracle_lib):
    gpu, ref = full
    utts = [synthetic.audio(s, seed=60 + i) for i, s in enumerate([3.1, 1.2])]
    got = gpu.transcribe(utts)
    gpu.ctx.check()
    compared = 0
    for u, g in zip(utts, got):
        want, margin = ref.decode(ref.encode(oracle_lib.parakeet_features(u), threads=8), threads=8)
        assert len(want) > 0
        assert _tokens_match([(t.id, t.frame, t.duration) for t in g], want, margin)
        compared += margin > 1e-2
    assert compared >= 1


# ---- the benchmark's own weight distribution --------------------------------------------------------

@pytest.fixture(scope="module")
def full_spec(ctx, oracle_lib):
    from telmo_b200.parakeet import Parakeet
    config = synthetic.parakeet_config()
    entries = synthetic.parakeet_entries(config, seed=3, scales="spec")
    return Parakeet.from_entries(ctx, config, entries), oracle_lib.Parakeet(config, entries)


def test_benchmark_model_matches_the_oracle_before_it_diverges(full_spec, oracle_lib):
    # The config-4 model exactly as bench.py builds it (per-row scales U(1e-3, 1e-2)). Like the
    # Granite benchmark model it is chaotic: in the oracle itself a 1e-6 relative change of the
    # features grows to 2.9e-4 relative L2 after layer 2, 7e-2 after layer 5 and 0.48 after
    # layer 11, so no implementation that rounds differently from the reference can meet 2e-2 at
    # its output. The subsampling and the first layer, before the divergence builds up, are held
    # to the north star's bar (by layer 2 the GPU's split-int8 rounding has grown to about 4e-2).
    import torch
    gpu, ref = full_spec
    utts = [synthetic.audio(s, seed=70 + i) for i, s in enumerate([4.0, 9.5])]
    feats = [oracle_lib.parakeet_features(u) for u in utts]
    rows = [f.shape[0] for f in feats]
    for tap in (-2, 0):
        out, frames = gpu.encode(torch.from_numpy(np.concatenate(feats)).cuda(), rows, tap_layer=tap)
        gpu.ctx.check()
        got = out.cpu().numpy()
        at = 0
        for f, fr in zip(feats, frames):
            want = ref.encode(f, tap_layer=tap, threads=8)
            assert rel_l2(got[at:at + fr], want) <= 2e-2, tap
            at += fr


# ---- the two decoders -------------------------------------------------------------------------

def _decode_both(gpu, enc, frames):
    gpu.set_decoder(True)
    tok_p, cnt_p, total_p = gpu.decode_packed(enc, frames)
    assert gpu.last_decoder() == 1
    gpu.set_decoder(False)
    try:
        tok_g, cnt_g, total_g = gpu.decode_packed(enc, frames)
        assert gpu.last_decoder() == 0
    finally:
        gpu.set_decoder(True)
    gpu.ctx.check()
    return (tok_p.cpu().numpy(), cnt_p.cpu().numpy(), total_p), (tok_g.cpu().numpy(), cnt_g.cpu().numpy(), total_g)


def test_persistent_decoder_equals_the_per_phase_decoder(tiny):
    # Same products, same epilogue, same quantization: the same tokens bit for bit, including
    # for an utterance with no frames and one that finishes on the first pass.
    import torch
    gpu, ref = tiny
    rows = [203, 57, 450, 9, 320, 1]
    encs = [ref.encode(_features(r, 90 + i)) for i, r in enumerate(rows)]
    frames = [e.shape[0] for e in encs[:-1]] + [0]
    enc = torch.from_numpy(np.concatenate(encs[:-1])).cuda()
    (tp, cp, np_), (tg, cg, ng) = _decode_both(gpu, enc, frames)
    assert np_ == ng > 0 and np.array_equal(cp, cg) and cp[-1] == 0
    assert np.array_equal(tp, tg)


def test_persistent_decoder_on_the_benchmark_model(full_spec):
    # The config-4 decoder at its full size on 48 utterances of 1..374 frames: many passes, the
    # live and predicting rows shrinking as utterances finish, both row halves of the stage ring.
    import torch
    gpu, _ = full_spec
    rng = synthetic.rng(5)
    frames = [int(x) for x in rng.integers(1, 375, 48)] + [374]
    enc = torch.from_numpy(rng.standard_normal((sum(frames), 1024)).astype(np.float32)).cuda()
    (tp, cp, np_), (tg, cg, ng) = _decode_both(gpu, enc, frames)
    assert np_ == ng > 0 and np.array_equal(cp, cg)
    assert np.array_equal(tp, tg)


def test_decoder_choice_is_checked(tiny):
    from telmo_b200 import TelmoError
    gpu, _ = tiny
    with pytest.raises(TelmoError):
        gpu.set_decoder(2)


# ---- Q8_0 weights, the reference's recommended Parakeet precision (src/model.rs:94-102) --------

@pytest.fixture(scope="module")
def tiny_q8(ctx, oracle_lib):
    from telmo_b200.parakeet import Parakeet
    entries = synthetic.parakeet_entries(TINY, seed=21, scales="conditioned", precision="q8_0")
    return Parakeet.from_entries(ctx, TINY, entries), oracle_lib.Parakeet(TINY, entries)


@pytest.mark.parametrize("tap", [-2, 0, -1])
def test_q8_0_tiny_encoder_matches(tiny_q8, tap):
    import torch
    gpu, ref = tiny_q8
    feats = _features(203, 12)
    out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [203], tap_layer=tap)
    gpu.ctx.check()
    want = ref.encode(feats, tap_layer=tap)
    err = rel_l2(out.cpu().numpy(), want)
    assert err <= layer_bar(None if tap == -2 else (tap if tap >= 0 else 1)), err


def test_q8_0_tiny_transcribe_matches_and_uses_the_phase_decoder(tiny_q8, oracle_lib):
    # Two-level weights do not fit the persistent decoder's shared memory plan: the per-phase
    # decoder runs them.
    gpu, ref = tiny_q8
    utts = [synthetic.audio(s, seed=80 + i) for i, s in enumerate([1.3, 2.7])]
    got = gpu.transcribe(utts)
    gpu.ctx.check()
    assert gpu.last_decoder() == 0
    compared = 0
    for u, g in zip(utts, got):
        want, margin = ref.decode(ref.encode(oracle_lib.parakeet_features(u)))
        assert _tokens_match([(t.id, t.frame, t.duration) for t in g], want, margin)
        compared += margin > 1e-2
    assert compared >= 1


def test_q8_0_full_size_layers_and_tokens_match(ctx, oracle_lib):
    import torch
    from telmo_b200.parakeet import Parakeet
    config = synthetic.parakeet_config()
    entries = synthetic.parakeet_entries(config, seed=4, scales="conditioned", precision="q8_0")
    gpu, ref = Parakeet.from_entries(ctx, config, entries), oracle_lib.Parakeet(config, entries)
    feats = _features(520, 91)
    for tap in (-2, 0, 23):
        out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [520], tap_layer=tap)
        gpu.ctx.check()
        want = ref.encode(feats, tap_layer=tap, threads=8)
        err = rel_l2(out.cpu().numpy(), want)
        assert err <= 2e-2, (tap, err)
        assert err <= layer_bar(None if tap == -2 else tap), (tap, err)
    utts = [synthetic.audio(3.1, seed=64)]
    got = gpu.transcribe(utts)
    gpu.ctx.check()
    want, margin = ref.decode(ref.encode(oracle_lib.parakeet_features(utts[0]), threads=8), threads=8)
    assert len(want) > 0 and _tokens_match([(t.id, t.frame, t.duration) for t in got[0]], want, margin)


# ---- the networks the biased beam search reads (src/parakeet.rs:1641-1676) ---------------------

@pytest.mark.parametrize("which", ["tiny", "full"])
def test_beam_search_networks_match_the_oracle(request, which):
    # enc_proj, joint at one frame for many hypotheses, and predict_rows over caller-held
    # states, against the oracle's restatement of the reference's Networks; each within the
    # north star's 1e-3 max-relative per product.
    import torch
    gpu, ref = request.getfixturevalue(which)
    c = gpu.config
    h, L = c["pred_hidden"], c["pred_layers"]
    g = synthetic.rng(33)
    enc = g.standard_normal((37, c["d_model"])).astype(np.float32)
    ep = gpu.enc_proj(torch.from_numpy(enc).cuda())
    gpu.ctx.check()
    want_ep = ref.enc_proj(enc)
    assert np.max(np.abs(ep.cpu().numpy() - want_ep)) <= 1e-3 * np.max(np.abs(want_ep))
    rows = 29
    preds = g.standard_normal((rows, h)).astype(np.float32)
    out = gpu.joint(ep[5], torch.from_numpy(preds).cuda())
    gpu.ctx.check()
    want = ref.joint(want_ep[5], preds)
    assert np.max(np.abs(out.cpu().numpy() - want)) <= 1e-3 * np.max(np.abs(want))
    tokens = g.integers(0, c["vocab"], rows)
    states = (g.standard_normal((rows, L * 2 * h)) * 0.5).astype(np.float32)
    st = torch.from_numpy(states).cuda()
    pr = torch.empty((rows, h), dtype=torch.float32, device="cuda")
    gpu.predict(tokens, st, pr)
    gpu.ctx.check()
    want_st, want_pr = ref.predict(tokens, states)
    assert np.max(np.abs(st.cpu().numpy() - want_st)) <= 1e-3 * np.max(np.abs(want_st))
    assert np.max(np.abs(pr.cpu().numpy() - want_pr)) <= 1e-3 * np.max(np.abs(want_pr))


def test_predict_rejects_tokens_outside_the_vocabulary(tiny):
    import torch
    from telmo_b200 import TelmoError
    gpu, _ = tiny
    h, L = gpu.config["pred_hidden"], gpu.config["pred_layers"]
    st = torch.zeros((2, L * 2 * h), device="cuda")
    pr = torch.zeros((2, h), device="cuda")
    with pytest.raises(TelmoError):
        gpu.predict([0, gpu.config["vocab"]], st, pr)


def test_decoder_barrier_timeout_is_reported_and_the_context_recovers(tiny):
    # The persistent decoder's grid barriers wait at most about a second. One CTA withholds its
    # arrival at the first barrier (a flag nothing else sets; no copies or MMAs are in flight
    # there): every CTA's wait runs out, the kernel returns, and the decode reports
    # TELMO_ERR_DEVICE_TIMEOUT. The same context then checks clean and decodes as before.
    import time
    import torch
    from telmo_b200 import TelmoError
    from telmo_b200._lib import TELMO_ERR_DEVICE_TIMEOUT
    gpu, ref = tiny
    encs = [ref.encode(_features(r, 95 + i)) for i, r in enumerate([203, 57])]
    frames = [e.shape[0] for e in encs]
    enc = torch.from_numpy(np.concatenate(encs)).cuda()
    gpu.set_decoder(True)
    want = gpu.decode(enc, frames)
    assert gpu.last_decoder() == 1
    gpu.test_barrier_timeout(0)
    t0 = time.perf_counter()
    with pytest.raises(TelmoError) as e:
        gpu.decode(enc, frames)
    assert e.value.status == TELMO_ERR_DEVICE_TIMEOUT and "barrier" in str(e.value)
    assert 0.5 < time.perf_counter() - t0 < 30.0
    gpu.ctx.check()
    got = gpu.decode(enc, frames)
    gpu.ctx.check()
    assert gpu.last_decoder() == 1
    assert [[(t.id, t.frame, t.duration) for t in u] for u in got] == \
        [[(t.id, t.frame, t.duration) for t in u] for u in want]
    with pytest.raises(TelmoError):
        gpu.test_barrier_timeout(-1)

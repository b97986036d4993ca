"""Parity of the CUDA Granite encoder with the oracle's restatement of Granite::encode.

Bars (the north star's): every block output and the encoder output within 2e-2 relative L2
(||got - ref|| / ||ref||) of the reference's f32 CPU path, and greedy CTC ids identical wherever
the reference's top-2 logit margin exceeds 1e-2. Batched calls must give each utterance what a
call on that utterance alone gives (the reference has no batch API; its oracle is one run per
utterance).
"""

import numpy as np
import pytest

from telmo_b200 import synthetic

pytestmark = pytest.mark.gpu

TINY = synthetic.granite_config(d_model=128, heads=2, head_dim=64, layers=4, ff=256,
                                conv_channels=256, conv_kernel=5, context=16, max_relative=32,
                                vocab=33, n_mels=8)


def rel_l2(got, ref):
    return float(np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref))


def _models(ctx, oracle_lib, config, seed):
    from telmo_b200.granite import Granite
    entries = synthetic.granite_entries(config, seed=seed)
    return Granite.from_entries(ctx, config, entries), oracle_lib.Granite(config, entries)


def _features(rows, width, seed):
    return synthetic.rng(seed).standard_normal((rows, width)).astype(np.float32)


@pytest.fixture(scope="module")
def tiny(ctx, oracle_lib):
    return _models(ctx, oracle_lib, TINY, seed=11)


@pytest.mark.parametrize("tap", [0, 1, 2, 3, -1])
def test_tiny_encoder_layers_match(tiny, tap):
    import torch
    gpu, ref = tiny
    feats = _features(45, 32, 12)
    out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [45], tap_layer=tap)
    gpu.ctx.check()
    want = ref.encode(feats, tap_layer=tap)
    assert out.shape == want.shape and frames[0] == want.shape[0]
    assert rel_l2(out.cpu().numpy(), want) <= 2e-2


def test_tiny_batch_equals_single_utterances(tiny):
    import torch
    gpu, ref = tiny
    rows = [45, 61, 4, 130]
    feats = [_features(r, 32, 20 + i) for i, r in enumerate(rows)]
    out, frames = gpu.encode(torch.from_numpy(np.concatenate(feats)).cuda(), rows)
    gpu.ctx.check()
    got = out.cpu().numpy()
    at = 0
    for f, r, fr in zip(feats, rows, frames):
        want = ref.encode(f)
        assert fr == want.shape[0] == gpu.frames_for(r)
        assert rel_l2(got[at:at + fr], want) <= 2e-2
        single, _ = gpu.encode(torch.from_numpy(f).cuda(), [r])
        assert np.array_equal(single.cpu().numpy(), got[at:at + fr])
        at += fr


def test_too_short_audio_is_a_model_error(tiny):
    import torch
    from telmo_b200 import TelmoError
    from telmo_b200._lib import TELMO_ERR_MODEL
    gpu, _ = tiny
    with pytest.raises(TelmoError) as e:
        gpu.encode(torch.zeros((3, 32), device="cuda"), [3])
    assert e.value.status == TELMO_ERR_MODEL and "too short" in str(e.value)


def test_incomplete_or_wrong_entries_are_errors(ctx):
    from telmo_b200 import TelmoError
    from telmo_b200.granite import Granite
    entries = synthetic.granite_entries(TINY, seed=3)
    del entries["blocks.2.dw.b"]
    with pytest.raises(TelmoError, match="blocks.2.dw.b"):
        Granite.from_entries(ctx, TINY, entries)
    bad = dict(TINY, conv_kernel=4)
    with pytest.raises(TelmoError):
        Granite(ctx, bad)
    g = Granite(ctx, TINY)
    with pytest.raises(TelmoError):
        Granite.from_entries(ctx, TINY, {"blocks.0.qkv": synthetic.int8_matrix(
            synthetic.rng(1), 10, 128)})
    g.close()


def test_q8_0_linears_match_the_oracle(ctx, oracle_lib):
    # Every linear whose inputs come in whole blocks of 32 as Q8_0 (the relative tables stay
    # Int8): each block within the north star's bar of the reference's f32 path.
    import torch
    from telmo_b200.granite import Granite
    config = dict(TINY, n_mels=16)
    entries = synthetic.granite_entries(config, seed=15, scales="conditioned", precision="q8_0")
    assert sum(isinstance(v, tuple) and len(v) == 5 for v in entries.values()) > 10
    gpu, ref = Granite.from_entries(ctx, config, entries), oracle_lib.Granite(config, entries)
    feats = _features(61, 64, 16)
    for tap in (0, 3):
        out, frames = gpu.encode(torch.from_numpy(feats).cuda(), [61], tap_layer=tap)
        gpu.ctx.check()
        want = ref.encode(feats, tap_layer=tap)
        assert rel_l2(out.cpu().numpy(), want) <= 2e-2


def test_q8_0_relative_tables_are_refused(ctx):
    from telmo_b200 import TelmoError
    from telmo_b200._lib import TELMO_ERR_UNSUPPORTED
    from telmo_b200.granite import Granite
    entries = synthetic.granite_entries(TINY, seed=3)
    v, s, n, k = entries["blocks.1.rel"]
    entries["blocks.1.rel"] = synthetic.as_q8_0((v, s, n, k))
    with pytest.raises(TelmoError) as e:
        Granite.from_entries(ctx, TINY, entries)
    assert e.value.status == TELMO_ERR_UNSUPPORTED


def test_ctc_tokens_match_the_oracle(ctx, oracle_lib):
    import torch
    from telmo_b200.granite import ctc_tokens
    g = synthetic.rng(5)
    frames = [11, 0, 1, 77, 300, 33]
    ids = [np.array([0, 5, 5, 0, 5, 7, 7, 7, 0, 0, 2], np.uint32)] + [
        g.integers(0, 4, size=f).astype(np.uint32) for f in frames[1:]]
    dev = torch.from_numpy(np.concatenate(ids).astype(np.int32)).cuda()
    got = ctc_tokens(ctx, dev, frames, blank=0)
    for u, want_ids in enumerate(ids):
        want = oracle_lib.ctc_tokens(want_ids)
        assert [(t.id, t.frame, t.duration) for t in got[u]] == want
    assert [(t.id, t.frame, t.duration) for t in got[0]] == [(5, 1, 2), (5, 4, 1), (7, 5, 3),
                                                               (2, 10, 1)]


def _full(ctx, oracle_lib, scales):
    from telmo_b200.granite import Granite
    cfg = synthetic.granite_config()
    entries = synthetic.granite_entries(cfg, seed=1, scales=scales)
    return Granite.from_entries(ctx, cfg, entries), oracle_lib.Granite(cfg, entries)


def test_full_size_encoder_and_ids_match(ctx, oracle_lib):
    """Granite-shaped model (config 2 sizes, weights of trained-layer size) on two synthetic
    utterances in one batch: every block within 2e-2 relative L2 (measured: below 1e-4, so the
    test also holds it to 1e-3) and identical ids where the margin exceeds 1e-2."""
    import torch
    gpu, ref = _full(ctx, oracle_lib, "conditioned")
    audio = [synthetic.audio(2.0, seed=31), synthetic.audio(3.3, seed=32)]
    feats = [oracle_lib.granite_features(a) for a in audio]
    rows = [f.shape[0] for f in feats]
    dfeats = torch.from_numpy(np.concatenate(feats)).cuda()
    for tap in [0, 1, 7, 15]:
        out, frames = gpu.encode(dfeats, rows, tap_layer=tap)
        got = out.cpu().numpy()
        at = 0
        for f, fr in zip(feats, frames):
            want = ref.encode(f, tap_layer=tap, threads=8)
            err = rel_l2(got[at:at + fr], want)
            assert err <= 2e-2 and err <= 1e-3, (tap, err)
            at += fr
    ids = gpu.frame_ids(out).cpu().numpy()
    gpu.ctx.check()
    at = 0
    for f, fr in zip(feats, frames):
        want_ids, margin = ref.frame_ids(ref.encode(f, threads=8), threads=8)
        sure = margin > 1e-2
        assert sure.mean() > 0.5
        assert np.array_equal(ids[at:at + fr][sure], want_ids[sure].astype(np.int32))
        at += fr
    gpu.close()


def test_full_size_spec_model_tracks_the_reference_until_it_diverges(ctx, oracle_lib):
    """With the benchmark's weight distribution (scales U(1e-3, 1e-2)) the model is chaotic: a
    1e-6 input change grows about 3x per block in the reference's own arithmetic, so only the
    first blocks can be compared; they stay within 2e-2."""
    import torch
    gpu, ref = _full(ctx, oracle_lib, "spec")
    f = oracle_lib.granite_features(synthetic.audio(2.0, seed=31))
    for tap in [0, 1, 2]:
        out, _ = gpu.encode(torch.from_numpy(f).cuda(), [f.shape[0]], tap_layer=tap)
        assert rel_l2(out.cpu().numpy(), ref.encode(f, tap_layer=tap, threads=8)) <= 2e-2
    gpu.ctx.check()
    gpu.close()


# ---- streaming (GraniteStream, src/granite_stream.rs) ---------------------------------------------

STREAM = synthetic.granite_config(d_model=128, heads=2, head_dim=64, layers=4, ff=256,
                                  conv_channels=256, conv_kernel=5, context=16, max_relative=32,
                                  vocab=33, n_mels=80)


@pytest.fixture(scope="module")
def stream_models(ctx, oracle_lib):
    return _models(ctx, oracle_lib, STREAM, seed=7)


def test_one_finished_stream_update_is_the_offline_pass(stream_models, oracle_lib):
    # src/granite_stream.rs:14-17: one update over a whole utterance is Granite::encode and
    # frame_ids -- here, the GPU's own offline front end, encoder and frame ids, bit for bit.
    import torch
    from telmo_b200.granite import GraniteStream, logmel
    from telmo_b200 import _lib
    gpu, ref = stream_models
    audio = synthetic.audio(3.3, seed=5)
    st = GraniteStream(gpu)
    st.push(audio)
    st.update(finished=True)
    feats, rows = logmel(gpu.ctx, _lib.FRONTEND_GRANITE, torch.from_numpy(audio).cuda(), [audio.size])
    gpu.ctx.check()
    assert np.array_equal(st.features(), feats.cpu().numpy())
    enc, frames = gpu.encode(feats, rows)
    assert np.array_equal(st.layer_output(STREAM["layers"] - 1), enc.cpu().numpy())
    ids = gpu.frame_ids(enc)
    assert np.array_equal(st.frame_ids(), ids.cpu().numpy().astype(np.uint32))
    assert st.first_changed() == 0
    # And the oracle's stream (the reference's arithmetic) agrees.
    ost = oracle_lib.GraniteStream(ref)
    ost.push(audio)
    ost.update(finished=True)
    want = ost.layer_output(STREAM["layers"] - 1)
    assert rel_l2(st.layer_output(STREAM["layers"] - 1), want) <= 2e-3


def test_stream_updates_match_the_oracle_stream(stream_models, oracle_lib):
    # Pieces of 0.37 s (about 4.6 encoder frames), a freeze lag of 2: after every update the
    # frame count, the first changed frame and the frozen frame equal the oracle stream's, every
    # block's cached outputs agree, and the ids agree wherever the top-2 logit gap is clear.
    from telmo_b200.granite import GraniteStream
    gpu, ref = stream_models
    audio = synthetic.audio(4.1, seed=6)
    st, ost = GraniteStream(gpu), oracle_lib.GraniteStream(ref)
    st.set_freeze_lag(2)
    ost.set_freeze_lag(2)
    piece, at, updates = 5920, 0, 0
    while at < audio.size:
        st.push(audio[at:at + piece])
        ost.push(audio[at:at + piece])
        at += piece
        done = at >= audio.size
        st.update(finished=done)
        ost.update(finished=done)
        gpu.ctx.check()
        assert (st.frames(), st.first_changed(), st.frozen()) == \
            (len(ost.frame_ids()), ost.first_changed(), ost.frozen())
        for layer in range(STREAM["layers"]):
            got, want = st.layer_output(layer), ost.layer_output(layer)
            assert got.shape == want.shape
            if want.size:
                assert rel_l2(got, want) <= 2e-3, (updates, layer)
        last = ost.layer_output(STREAM["layers"] - 1)
        if last.size:
            ids, margin = ref.frame_ids(last)
            clear = margin > 1e-2
            assert np.array_equal(st.frame_ids()[clear], ids[clear])
        updates += 1
    assert updates >= 10 and st.frozen() > 0


def test_stream_misuse_is_an_error(stream_models, ctx):
    from telmo_b200 import TelmoError
    from telmo_b200.granite import GraniteStream
    gpu, _ = stream_models
    st = GraniteStream(gpu)
    st.push(synthetic.audio(0.5, seed=1))
    st.update(finished=True)
    with pytest.raises(TelmoError):
        st.push(np.zeros(10, np.float32))
    with pytest.raises(TelmoError):
        st.update()
    # A model whose first block is not strided cannot stream.
    from telmo_b200.granite import Granite
    bad = dict(STREAM, subsample_layers=[1, 2])
    g2 = Granite.from_entries(ctx, bad, synthetic.granite_entries(bad, seed=3))
    with pytest.raises(TelmoError):
        GraniteStream(g2)

"""Parity of the batched CUDA front ends and of end-to-end transcription with the oracle.

The oracle's front ends match the reference's golden features (tests/test_oracle_pins.py); here
the GPU front ends must match the oracle on synthetic audio -- every feature within 1e-5 (their
f64 spectra follow the same operation order, so most values agree bit for bit) -- with edge
lengths: the shortest accepted audio, a last odd frame, 30 s.
"""

import numpy as np
import pytest

from telmo_b200 import _lib, synthetic

pytestmark = pytest.mark.gpu

LENGTHS = [320, 16000, 16160, 4321, 30 * 16000, 333]


def _audio():
    return [synthetic.audio(n / 16000.0, seed=40 + i)[:n] for i, n in enumerate(LENGTHS)]


@pytest.mark.parametrize("kind", [_lib.FRONTEND_GRANITE, _lib.FRONTEND_PARAKEET])
def test_batched_front_end_matches_the_oracle(ctx, oracle_lib, kind):
    import torch
    from telmo_b200.granite import logmel
    audio = _audio()
    dev = torch.from_numpy(np.concatenate(audio)).cuda()
    feats, rows = logmel(ctx, kind, dev, [len(a) for a in audio])
    ctx.check()
    got = feats.cpu().numpy()
    at = 0
    for a, r in zip(audio, rows):
        want = oracle_lib.granite_features(a) if kind == _lib.FRONTEND_GRANITE else \
            oracle_lib.parakeet_features(a)
        assert r == want.shape[0]
        err = np.abs(got[at:at + r] - want)
        assert err.max() <= 1e-5, err.max()
        assert np.mean(err == 0) > 0.9
        at += r


def test_front_end_rejects_too_short_audio(ctx):
    import torch
    from telmo_b200 import TelmoError
    from telmo_b200.granite import logmel
    with pytest.raises(TelmoError, match="too short"):
        logmel(ctx, _lib.FRONTEND_GRANITE, torch.zeros(319, device="cuda"), [319])


def test_transcribe_matches_the_oracle_pipeline(ctx, oracle_lib):
    """Audio -> tokens for a batch through the public call with host buffers, against the
    oracle's features -> encode -> argmax -> ctc_tokens, on the conditioned Granite-shaped
    model. Token lists must be identical for utterances whose every frame has a margin above
    1e-2, and frame ids identical where the margin exceeds 1e-2 otherwise."""
    from telmo_b200.granite import Granite
    cfg = synthetic.granite_config()
    entries = synthetic.granite_entries(cfg, seed=1, scales="conditioned")
    gpu = Granite.from_entries(ctx, cfg, entries)
    ref = oracle_lib.Granite(cfg, entries)
    audio = [synthetic.audio(s, seed=50 + i) for i, s in enumerate([1.3, 4.0, 2.2])]
    tokens = gpu.transcribe(audio)
    ctx.check()
    for a, got in zip(audio, tokens):
        enc = ref.encode(oracle_lib.granite_features(a), threads=8)
        ids, margin = ref.frame_ids(enc, threads=8)
        want = oracle_lib.ctc_tokens(ids)
        got_t = [(t.id, t.frame, t.duration) for t in got]
        if np.all(margin > 1e-2):
            assert got_t == want
        else:
            assert len(got_t) > 0
    gpu.close()

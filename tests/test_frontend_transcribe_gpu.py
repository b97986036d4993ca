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


def test_host_transcribe_in_pipelined_groups_equals_one_group(ctx):
    """telmo_granite_transcribe splits its utterances into groups and copies the next group's
    audio up while one is transcribed. Each utterance's result does not depend on the others in
    its batch, so any grouping gives the same tokens, counts and frames bit for bit -- with
    pageable or pinned host audio and tokens, and for an utterance longer than a group."""
    import torch
    from telmo_b200.granite import Granite
    cfg = synthetic.granite_config(layers=4)
    entries = synthetic.granite_entries(cfg, seed=1, scales="conditioned")
    gpu = Granite.from_entries(ctx, cfg, entries)
    secs = [0.7, 3.3, 1.1, 6.0, 2.5, 0.3, 4.4, 1.9, 2.2, 5.1]
    audio = [synthetic.audio(s, seed=80 + i) for i, s in enumerate(secs)]
    lengths = np.array([a.size for a in audio], np.int64)
    packed = np.concatenate(audio)
    want = gpu.transcribe_arrays(packed, lengths)
    for group_s in (4.0, 1.0, 9.0):
        gpu.set_transcribe_group(group_s)
        for pinned in (False, True):
            samples = torch.from_numpy(packed).pin_memory() if pinned else packed
            cap = 3 * sum(gpu.frames_for_samples(int(x)) for x in lengths)
            tokens = torch.zeros(cap, dtype=torch.int32).pin_memory() if pinned else None
            got = gpu.transcribe_arrays(samples, lengths, tokens_buf=tokens)
            ctx.check()
            got_tok = (got[0].numpy() if hasattr(got[0], "numpy") else got[0]).view(np.uint32)
            assert np.array_equal(got[2], want[2]) and np.array_equal(got[1], want[1])
            # Utterance u's counts[u] triples start at 3 * (frames before it); the rest of its
            # region is not written.
            at = 0
            for f, c in zip(want[2], want[1]):
                assert np.array_equal(got_tok[3 * at:3 * (at + c)], want[0].view(np.uint32)[3 * at:3 * (at + c)]), \
                    (group_s, pinned)
                at += int(f)
    gpu.set_transcribe_group(2048.0)
    from telmo_b200 import TelmoError
    with pytest.raises(TelmoError):
        gpu.set_transcribe_group(0.0)
    gpu.close()

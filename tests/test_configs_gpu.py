"""Parity at the benchmark configurations' own sizes: full-length utterances and whole batches,
each utterance against one run of the oracle (the reference has no batch API; its oracle for a
batch is Model::transcribe per utterance, src/model.rs:154-159).

* config 2: one 30 s utterance (1500 feature rows, three 128-frame attention blocks after the
  two strided blocks) through the Granite-shaped model, every tapped block within 1e-3 relative
  L2 (the north star's bar is 2e-2) and CTC ids identical wherever the reference's top-2 logit
  margin exceeds 1e-2;
* config 3: 64 utterances, lengths uniform in 1-30 s, in ONE masked batch: per utterance the
  GPU front end, the encoder output, the frame ids and the CTC tokens of the batched call;
* config 4: 32 utterances of 1-30 s (one of 30 s) through the Parakeet-TDT-shaped model in one
  batch, tokens from the persistent decoder against the oracle's greedy decode_inner;
* the persistent decoder at the benchmark's size on oracle-encoded frames.

The encoders use weights of trained-layer size (``scales="conditioned"``): with the benchmark's
scale distribution the random model amplifies any rounding difference about 3x per block in the
reference's own arithmetic (tests/test_chaos.py measures it), so only the first blocks of that
model can be compared (test_granite_gpu.py, test_parakeet_gpu.py). A TDT token is held to the
reference's wherever every joint step before it had a top-2 gap above 1e-2 (``decode_sure``).
"""

import os

import numpy as np
import pytest

from telmo_b200 import synthetic

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1
MARGIN = 1e-2


def rel_l2(got, ref):
    return float(np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref))


def _sure_ids_match(got_ids, want_ids, margin):
    sure = margin > MARGIN
    return bool(np.array_equal(np.asarray(got_ids)[sure], np.asarray(want_ids, np.int64)[sure].astype(
        np.asarray(got_ids).dtype))), float(sure.mean()) if sure.size else 1.0


@pytest.fixture(scope="module")
def granite(ctx, oracle_lib):
    from telmo_b200.granite import Granite
    cfg = synthetic.granite_config()
    entries = synthetic.granite_entries(cfg, seed=1, scales="conditioned")
    gpu, ref = Granite.from_entries(ctx, cfg, entries), oracle_lib.Granite(cfg, entries)
    yield gpu, ref
    gpu.close()


def test_config2_thirty_second_utterance(granite, oracle_lib):
    import torch
    gpu, ref = granite
    audio = synthetic.audio(30.0, seed=41)
    feats = oracle_lib.granite_features(audio)
    assert feats.shape == (1500, 320)
    dfeats = torch.from_numpy(feats).cuda()
    for tap in (0, 1, 7, 15):
        out, frames = gpu.encode(dfeats, [1500], tap_layer=tap)
        gpu.ctx.check()
        want = ref.encode(feats, tap_layer=tap, threads=THREADS)
        assert out.shape == want.shape, tap
        err = rel_l2(out.cpu().numpy(), want)
        assert err <= 1e-3, (tap, err)
    assert frames[0] == 375
    ids = gpu.frame_ids(out).cpu().numpy()
    want_ids, margin = ref.frame_ids(want, threads=THREADS)
    same, frac = _sure_ids_match(ids, want_ids, margin)
    assert same and frac > 0.5, frac


def _config3_set():
    secs = synthetic.lengths_uniform(64, 1.0, 30.0, seed=3)
    secs[17] = 30.0  # the config's longest utterance is in the batch
    return [synthetic.audio(float(s), seed=300 + i) for i, s in enumerate(secs)]


def test_config3_masked_batch_matches_one_oracle_run_per_utterance(granite, oracle_lib):
    import torch
    from telmo_b200 import _lib
    from telmo_b200.granite import logmel
    gpu, ref = granite
    utts = _config3_set()
    lengths = [u.size for u in utts]
    packed = np.concatenate(utts)
    feats, rows = logmel(gpu.ctx, _lib.FRONTEND_GRANITE, torch.from_numpy(packed).cuda(), lengths)
    enc, frames = gpu.encode(feats, rows)
    ids = gpu.frame_ids(enc).cpu().numpy()
    feats = feats.cpu().numpy()
    enc = enc.cpu().numpy()
    tokens = gpu.transcribe(utts)  # the same batch through the host-buffer entry point
    gpu.ctx.check()
    fa = ea = 0
    sure_frames = total_frames = 0
    for u, a in enumerate(utts):
        want_f = oracle_lib.granite_features(a)
        assert rows[u] == want_f.shape[0]
        got_f = feats[fa:fa + rows[u]]
        assert np.max(np.abs(got_f - want_f)) <= 1e-5 * max(1.0, float(np.max(np.abs(want_f)))), u
        fa += rows[u]
        want = ref.encode(want_f, threads=THREADS)
        assert frames[u] == want.shape[0]
        got = enc[ea:ea + frames[u]]
        err = rel_l2(got, want)
        assert err <= 1e-3, (u, err)
        want_ids, margin = ref.frame_ids(want, threads=THREADS)
        got_ids = ids[ea:ea + frames[u]]
        same, _ = _sure_ids_match(got_ids, want_ids, margin)
        assert same, u
        sure_frames += int((margin > MARGIN).sum())
        total_frames += int(frames[u])
        # The reference's tokens of the reference's ids, with the frames too close to call taken
        # as the GPU decided them, are the batched transcription's tokens.
        merged = np.where(margin > MARGIN, want_ids.astype(np.int64), got_ids.astype(np.int64))
        want_tok = oracle_lib.ctc_tokens(merged.astype(np.uint32))
        assert [(t.id, t.frame, t.duration) for t in tokens[u]] == want_tok, u
        ea += frames[u]
    assert sure_frames > 0.5 * total_frames


@pytest.fixture(scope="module")
def parakeet(ctx, oracle_lib):
    from telmo_b200.parakeet import Parakeet
    cfg = synthetic.parakeet_config()
    entries = synthetic.parakeet_entries(cfg, seed=3, scales="conditioned")
    gpu, ref = Parakeet.from_entries(ctx, cfg, entries), oracle_lib.Parakeet(cfg, entries)
    yield gpu, ref
    gpu.close()


def _prefix_matches(got, want, sure):
    got = [(t.id, t.frame, t.duration) for t in got]
    if got[:sure] == want[:sure]:
        return True
    first = next(i for i in range(min(sure, len(got)) + 1) if i >= len(got) or got[i] != want[i])
    print(f"first difference at token {first} of {sure} sure, {len(want)} in all: "
          f"got {got[max(0, first - 3):first + 3]} want {want[max(0, first - 3):first + 3]}")
    return False


def test_config4_batch_tokens_match_the_oracle(parakeet, oracle_lib):
    import torch
    gpu, ref = parakeet
    secs = synthetic.lengths_uniform(32, 1.0, 30.0, seed=4)
    secs[5] = 30.0
    utts = [synthetic.audio(float(s), seed=400 + i) for i, s in enumerate(secs)]
    gpu.set_decoder(True)
    got = gpu.transcribe(utts)
    gpu.ctx.check()
    assert gpu.last_decoder() == 1
    feats = [oracle_lib.parakeet_features(a) for a in utts]
    enc, frames = gpu.encode(torch.from_numpy(np.concatenate(feats)).cuda(), [f.shape[0] for f in feats])
    enc = enc.cpu().numpy()
    at = 0
    sure_total = want_total = 0
    for u, f in enumerate(feats):
        want_enc = ref.encode(f, threads=THREADS)
        assert frames[u] == want_enc.shape[0]
        err = rel_l2(enc[at:at + frames[u]], want_enc)
        assert err <= 4e-4 * (1.0 + 23 / 8.0), (u, err)
        at += frames[u]
        want, sure = ref.decode_sure(want_enc, MARGIN, threads=THREADS)
        assert _prefix_matches(got[u], want, sure), (u, sure, len(want))
        sure_total += sure
        want_total += len(want)
    assert want_total > 0 and sure_total > 0.5 * want_total, (sure_total, want_total)


def test_persistent_decoder_at_benchmark_size_matches_the_oracle(parakeet, oracle_lib):
    # The config-4 decoder at its full size (joint 8198 x 640, two LSTM layers of 640) on frames
    # the oracle encoded from 24 utterances of 1-30 s: the GPU's persistent kernel and the
    # reference's decode_inner read the same encoder output. With the benchmark's own weights the
    # prediction network's recurrent state is chaotic in the reference's own arithmetic (a 1e-6
    # change of the state changes the tokens within a few tens of tokens; tests/test_chaos.py),
    # so its tokens are compared on the weights of trained-layer size; the benchmark's weights
    # run the same kernel, which test_parakeet_gpu.py holds bit for bit to the per-phase decoder.
    import torch
    gpu, ref = parakeet
    secs = synthetic.lengths_uniform(24, 1.0, 30.0, seed=6)
    secs[0] = 30.0
    encs = [ref.encode(oracle_lib.parakeet_features(synthetic.audio(float(s), seed=600 + i)),
                       threads=THREADS) for i, s in enumerate(secs)]
    frames = [e.shape[0] for e in encs]
    assert max(frames) == 375
    gpu.set_decoder(True)
    got = gpu.decode(torch.from_numpy(np.concatenate(encs)).cuda(), frames)
    gpu.ctx.check()
    assert gpu.last_decoder() == 1
    sure_total = want_total = 0
    for u, e in enumerate(encs):
        want, sure = ref.decode_sure(e, MARGIN, threads=THREADS)
        assert _prefix_matches(got[u], want, sure), (u, sure, len(want))
        sure_total += sure
        want_total += len(want)
    assert want_total > 0 and sure_total > 0.5 * want_total, (sure_total, want_total)

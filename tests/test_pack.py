"""The pack reader and config.json parsers (src/pack.rs, Config::from_json) -- host code, no
GPU -- and models loaded from packs (GPU)."""

import json
import struct

import numpy as np
import pytest

from telmo_b200 import synthetic

from telmo_b200.pack import granite_config_json, parakeet_config_json, write_pack


def _sample():
    # src/pack.rs:618-631: one entry of each kind.
    w = np.array([(i % 17) * 0.1 - 0.8 for i in range(40 * 64)], np.float32).reshape(40, 64)
    from telmo_b200 import PackedWeights, Precision
    w8 = PackedWeights.encode(w, 40, 64, Precision.INT8)
    wq = PackedWeights.encode(w, 40, 64, Precision.Q8_0)
    return {"w8": (w8.values, w8.scales, 40, 64), "wq": (wq.values, wq.scales, 40, 64, "q8_0"),
            "bias": np.array([[1, 2, 3], [4, 5, 6]], np.float32), "config.json": b'{"a":1}'}


def test_a_pack_reads_back():
    from telmo_b200.pack import Pack
    p = Pack(data=write_pack("test", _sample(), {"source": "x"}))
    assert p.model == "test" and p.meta("source") == "x" and p.meta("nope") is None
    got = {e["name"]: e for e in p.entries()}
    assert got["w8"]["kind"] == "matrix" and got["w8"]["precision"] == "int8"
    assert (got["w8"]["n"], got["w8"]["k"], got["w8"]["bytes"]) == (40, 64, 48 * 64)
    assert got["wq"]["precision"] == "q8_0"
    assert got["bias"]["kind"] == "f32" and got["bias"]["bytes"] == 24
    assert p.bytes("config.json") == b'{"a":1}'
    from telmo_b200 import TelmoError
    with pytest.raises(TelmoError, match="missing"):
        p.bytes("missing")


def _damaged(good, **changes):
    data = bytearray(good)
    for at, value in changes.get("set", []):
        data[at] = value
    return bytes(data[:changes.get("cut", len(data))])


def test_damaged_packs_are_refused():
    # src/pack.rs:694-706, and the index checks of Pack::parse.
    from telmo_b200 import TelmoError
    from telmo_b200.pack import Pack
    good = write_pack("test", _sample())
    Pack(data=good)
    for bad in (good[:-1], _damaged(good, set=[(8, 2)]), _damaged(good, set=[(0, 0)]), b"",
                write_pack("test", _sample(), version=2)):
        with pytest.raises(TelmoError):
            Pack(data=bad)
    # Index problems: a wrong size, a misplaced or overlapping range, two entries of one name.
    idx_at, idx_len = struct.unpack("<QQ", good[-24:-8])
    index = json.loads(good[idx_at:idx_at + idx_len])

    def with_index(change):
        ix = json.loads(json.dumps(index))
        change(ix)
        blob = json.dumps(ix).encode()
        return good[:idx_at] + blob + struct.pack("<QQ", idx_at, len(blob)) + b"TELMOIDX"

    def entry(ix, name):
        return next(e for e in ix["entries"] if e["name"] == name)

    cases = [
        lambda ix: entry(ix, "w8").update(bytes=10),
        lambda ix: entry(ix, "w8").update(offset=entry(ix, "w8")["offset"] + 1),
        lambda ix: entry(ix, "bias").update(offset=entry(ix, "w8")["offset"]),
        lambda ix: ix["entries"].append(dict(entry(ix, "bias"))),
        lambda ix: entry(ix, "w8").update(precision="int4"),
        lambda ix: entry(ix, "wq").update(k=48),
        lambda ix: entry(ix, "w8").update(scales_bytes=4),
        lambda ix: entry(ix, "bias").update(type="tensor"),
        lambda ix: ix.pop("model"),
    ]
    with_index(lambda ix: None)  # the unchanged rewrite reads
    Pack(data=with_index(lambda ix: None))
    for change in cases:
        with pytest.raises(TelmoError):
            Pack(data=with_index(change))


# ---- device-layout packs (this build's extension; host only) ------------------------------------

def _panel_rows(values, n, k):
    """The panel layout's [n, k] int8 values (output o in panel o // 16, lane o % 16)."""
    p = (n + 15) // 16
    return np.asarray(values, np.int8).reshape(p, k, 16).transpose(0, 2, 1).reshape(p * 16, k)[:n]


def _device_planes(values, scales, n, k, precision, perm=None):
    """The device layout restated: rows of round_up(k, 16) values, one scale per row; Q8_0 rows
    re-encoded as s (hi + lo / 254) with s = amax / 127, each level rounded half to even."""
    ld = (k + 15) // 16 * 16
    q = _panel_rows(values, n, k).astype(np.int32)
    perm = np.arange(k) if perm is None else np.asarray(perm)
    hi = np.zeros((n, ld), np.int8)
    lo = np.zeros((n, ld), np.int8)
    if precision == "int8":
        hi[:, :k] = q[:, perm]
        sc = np.asarray(scales, np.float32).reshape(-1)[:n]
        return hi, None, sc
    blocks = k // 32
    d = np.asarray(scales, np.float32).reshape(-1, blocks, 16).transpose(0, 2, 1).reshape(-1, blocks)[:n]
    w = (q.astype(np.float32) * np.repeat(d, 32, axis=1))[:, perm]
    amax = np.abs(w).max(axis=1)
    s = (amax / np.float32(127)).astype(np.float32)
    inv = np.where(s != 0, np.float32(1) / np.where(s != 0, s, 1), 0).astype(np.float32)
    h = np.clip(np.rint(w * inv[:, None]), -127, 127).astype(np.float32)
    e = (w.astype(np.float64) - h.astype(np.float64) * s[:, None].astype(np.float64)).astype(np.float32)
    l = np.clip(np.rint(e * (inv * np.float32(254))[:, None]), -127, 127)
    hi[:, :k] = h.astype(np.int8)
    lo[:, :k] = l.astype(np.int8)
    return hi, lo, s


def _read_index(data):
    at, n = struct.unpack("<QQ", data[-24:-8])
    return json.loads(data[at:at + n])


def test_device_layout_pack(tmp_path):
    # The converted pack holds each 8-bit matrix as the upload would build it on the host, keeps
    # the other entries, reads back through the same checks, and converts again to itself.
    from telmo_b200.pack import Pack
    sample = _sample()
    src = Pack(data=write_pack("test", sample, {"source": "x"}))
    dev = src.to_device()
    assert dev.model == "test" and dev.meta("source") == "x"
    got = {e["name"]: e for e in dev.entries()}
    assert got["w8"]["kind"] == "device" and got["w8"]["precision"] == "int8"
    assert (got["w8"]["n"], got["w8"]["k"], got["w8"]["bytes"]) == (40, 64, 40 * 64)
    assert got["wq"]["kind"] == "device" and got["wq"]["precision"] == "q8_0"
    assert got["bias"]["kind"] == "f32" and dev.bytes("config.json") == b'{"a":1}'
    dev.save(tmp_path / "dev.pack")
    data = (tmp_path / "dev.pack").read_bytes()
    index = {e["name"]: e for e in _read_index(data)["entries"]}
    assert np.array_equal(np.frombuffer(data, np.float32, 6, index["bias"]["offset"]), sample["bias"].reshape(-1))
    for name, prec in (("w8", "int8"), ("wq", "q8_0")):
        values, scales, n, k = sample[name][:4]
        hi, lo, sc = _device_planes(values, scales, n, k, prec)
        e = index[name]
        assert e["type"] == "device" and all(e[f] % 64 == 0 for f in e if f.endswith("offset"))
        assert np.array_equal(np.frombuffer(data, np.int8, e["bytes"], e["offset"]).reshape(n, -1), hi)
        assert np.array_equal(np.frombuffer(data, np.float32, n, e["scales_offset"]), sc)
        if lo is not None:
            assert np.array_equal(np.frombuffer(data, np.int8, e["lo_bytes"], e["lo_offset"]).reshape(n, -1), lo)
        else:
            assert "lo_offset" not in e
    again = Pack(path=tmp_path / "dev.pack").to_device()
    again.save(tmp_path / "again.pack")
    assert (tmp_path / "again.pack").read_bytes() == data


@pytest.mark.parametrize("precision", ["int8", "q8_0"])
def test_device_layout_pack_orders_parakeet_columns(tmp_path, precision):
    # Parakeet's subsampling output matrix is stored with its columns in the kernels' order
    # (frequency-major); every other matrix keeps the pack's order.
    from telmo_b200.pack import Pack
    pc = synthetic.parakeet_config(layers=1, d_model=64, heads=2, ff=128, sub_channels=32, pred_hidden=32,
                                   vocab=17, blank=16)
    pe = synthetic.parakeet_entries(pc, seed=3, precision=precision)
    Pack(data=write_pack("parakeet-tdt", dict(pe, **{"config.json": parakeet_config_json(pc)}))).to_device().save(
        tmp_path / "p.pack")
    data = (tmp_path / "p.pack").read_bytes()
    index = {e["name"]: e for e in _read_index(data)["entries"]}
    ch, freqs = pc["sub_channels"], pc["n_mels"] // 8
    perm = [c * freqs + f for f in range(freqs) for c in range(ch)]
    for name, order in (("sub.linear", perm), ("sub.pw1", None)):
        values, scales, n, k = pe[name][:4]
        hi, lo, sc = _device_planes(values, scales, n, k, precision, order)
        e = index[name]
        assert np.array_equal(np.frombuffer(data, np.int8, e["bytes"], e["offset"]).reshape(n, -1), hi)
        assert np.array_equal(np.frombuffer(data, np.float32, n, e["scales_offset"]), sc)
        if lo is not None:
            assert np.array_equal(np.frombuffer(data, np.int8, e["lo_bytes"], e["lo_offset"]).reshape(n, -1), lo)
    # A Parakeet pack without its config cannot be converted (the column order depends on it).
    from telmo_b200 import TelmoError
    with pytest.raises(TelmoError, match="config.json"):
        Pack(data=write_pack("parakeet-tdt", pe)).to_device()


def test_damaged_device_entries_are_refused(tmp_path):
    from telmo_b200 import TelmoError
    from telmo_b200.pack import Pack
    Pack(data=write_pack("test", _sample())).to_device().save(tmp_path / "d.pack")
    good = (tmp_path / "d.pack").read_bytes()
    idx_at, idx_len = struct.unpack("<QQ", good[-24:-8])
    index = json.loads(good[idx_at:idx_at + idx_len])

    def with_index(change):
        ix = json.loads(json.dumps(index))
        change(ix)
        blob = json.dumps(ix).encode()
        return good[:idx_at] + blob + struct.pack("<QQ", idx_at, len(blob)) + b"TELMOIDX"

    def entry(ix, name):
        return next(e for e in ix["entries"] if e["name"] == name)

    Pack(data=with_index(lambda ix: None))
    cases = [
        lambda ix: entry(ix, "w8").update(precision="f32"),
        lambda ix: entry(ix, "w8").update(bytes=40 * 48),
        lambda ix: entry(ix, "w8").update(scales_bytes=4),
        lambda ix: entry(ix, "wq").pop("lo_offset"),
        lambda ix: entry(ix, "wq").update(lo_bytes=64),
        lambda ix: entry(ix, "wq").update(lo_offset=entry(ix, "wq")["offset"]),
        lambda ix: entry(ix, "wq").update(k=48),
    ]
    for change in cases:
        with pytest.raises(TelmoError):
            Pack(data=with_index(change))


def test_config_json_round_trips():
    from telmo_b200.pack import granite_config_from_json, parakeet_config_from_json
    g = synthetic.granite_config()
    assert granite_config_from_json(granite_config_json(g)) == \
        {k: g[k] for k in ("d_model", "heads", "head_dim", "layers", "ff", "conv_kernel", "conv_channels",
                           "n_mels", "context", "max_relative", "vocab", "blank", "subsample_layers")}
    p = synthetic.parakeet_config()
    assert parakeet_config_from_json(parakeet_config_json(p)) == \
        {k: p[k] for k in ("d_model", "heads", "layers", "ff", "conv_kernel", "sub_channels", "n_mels",
                           "pred_hidden", "pred_layers", "vocab", "blank", "max_symbols", "durations")}


def test_unsupported_configs_are_refused():
    from telmo_b200 import TelmoError
    from telmo_b200.pack import granite_config_from_json, parakeet_config_from_json
    g = json.loads(granite_config_json(synthetic.granite_config()))
    for change in (lambda c: c.update(model_type="llama"),
                   lambda c: c["encoder_config"].update(hidden_act="gelu"),
                   lambda c: c["encoder_config"].update(num_key_value_heads=2),
                   lambda c: c["encoder_config"].pop("context_size"),
                   lambda c: c.update(pad_token_id=5000)):
        bad = json.loads(json.dumps(g))
        change(bad)
        with pytest.raises(TelmoError):
            granite_config_from_json(json.dumps(bad))
    p = json.loads(parakeet_config_json(synthetic.parakeet_config()))
    for change in (lambda c: c["encoder_config"].update(subsampling_factor=4),
                   lambda c: c.update(blank_token_id=7),
                   lambda c: c.pop("durations")):
        bad = json.loads(json.dumps(p))
        change(bad)
        with pytest.raises(TelmoError):
            parakeet_config_from_json(json.dumps(bad))
    with pytest.raises(TelmoError):
        granite_config_from_json("{not json")


# ---- models from packs (GPU) ------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["int8", "q8_0"])
def test_models_load_from_packs(ctx, precision):
    # A pack of each model (plus an entry neither knows) loads into the same model as its
    # entries: identical encoder outputs bit for bit; a missing entry is named.
    import torch
    from telmo_b200 import TelmoError
    from telmo_b200.granite import Granite
    from telmo_b200.pack import Pack
    from telmo_b200.parakeet import Parakeet
    gc = synthetic.granite_config(d_model=128, heads=2, head_dim=64, layers=4, ff=256, conv_channels=256,
                                  conv_kernel=5, context=16, max_relative=32, vocab=33, n_mels=8)
    ge = synthetic.granite_entries(gc, seed=2, scales="conditioned", precision=precision)
    pack = Pack(data=write_pack("granite-speech-ctc",
                                dict(ge, **{"config.json": granite_config_json(gc), "extra": np.ones(3, np.float32)})))
    a, b = Granite.from_entries(ctx, gc, ge), Granite.from_pack(ctx, pack)
    feats = torch.from_numpy(synthetic.rng(4).standard_normal((61, 32)).astype(np.float32)).cuda()
    want = a.encode(feats, [61])[0].cpu().numpy()
    assert np.array_equal(want, b.encode(feats, [61])[0].cpu().numpy())
    # The device-layout pack (matrices copied, not repacked) loads into the same model.
    assert np.array_equal(want, Granite.from_pack(ctx, pack.to_device()).encode(feats, [61])[0].cpu().numpy())
    pc = synthetic.parakeet_config(layers=2, d_model=128, heads=2, ff=256, sub_channels=32, pred_hidden=64,
                                   vocab=65, blank=64)
    pe = synthetic.parakeet_entries(pc, seed=5, scales="conditioned", precision=precision)
    pack = Pack(data=write_pack("parakeet-tdt", dict(pe, **{"config.json": parakeet_config_json(pc)})))
    a, b = Parakeet.from_entries(ctx, pc, pe), Parakeet.from_pack(ctx, pack)
    f = torch.from_numpy(synthetic.rng(6).standard_normal((203, 128)).astype(np.float32)).cuda()
    want = a.encode(f, [203])[0].cpu().numpy()
    assert np.array_equal(want, b.encode(f, [203])[0].cpu().numpy())
    assert np.array_equal(want, Parakeet.from_pack(ctx, pack.to_device()).encode(f, [203])[0].cpu().numpy())
    gone = {k: v for k, v in pe.items() if k != "layers.1.pos"}
    pack = Pack(data=write_pack("parakeet-tdt", dict(gone, **{"config.json": parakeet_config_json(pc)})))
    with pytest.raises(TelmoError, match="layers.1.pos"):
        Parakeet.from_pack(ctx, pack)
    with pytest.raises(TelmoError):
        Granite.from_pack(ctx, pack)  # the pack holds another model

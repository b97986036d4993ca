"""Writes packs in the reference's file format (src/pack.rs:1-16, FileSink :470-620) for the tests:
"TELMOPAK", u32 version, 4 zero bytes; entry data at 64-byte multiples; a JSON index; the index's
offset and length as u64s and "TELMOIDX"."""

import json
import struct

import numpy as np


def write_pack(model, entries, metadata=None, version=1):
    """entries: name -> (values, scales, n, k[, "q8_0"]) matrix in panels, an f32 array, or bytes."""
    data = bytearray(b"TELMOPAK" + struct.pack("<I", version) + b"\0" * 4)
    index = []

    def put(blob):
        while len(data) % 64:
            data.append(0)
        at = len(data)
        data.extend(blob)
        return at

    for name, e in entries.items():
        if isinstance(e, (bytes, bytearray)):
            at = put(bytes(e))
            index.append({"name": name, "type": "bytes", "offset": at, "bytes": len(e)})
        elif isinstance(e, tuple):
            values, scales, n, k = e[:4]
            precision = e[4] if len(e) > 4 else "int8"
            v = np.ascontiguousarray(values, np.int8).tobytes()
            s = np.ascontiguousarray(scales, np.float32).tobytes()
            at = put(v)
            s_at = put(s)
            index.append({"name": name, "type": "matrix", "precision": precision, "n": n, "k": k,
                          "offset": at, "bytes": len(v), "scales_offset": s_at, "scales_bytes": len(s)})
        else:
            a = np.ascontiguousarray(e, np.float32)
            at = put(a.tobytes())
            index.append({"name": name, "type": "f32", "shape": list(a.shape), "offset": at,
                          "bytes": a.nbytes})
    idx = json.dumps({"model": model, "metadata": metadata or {}, "entries": index}).encode()
    at = len(data)
    data.extend(idx)
    data.extend(struct.pack("<QQ", at, len(idx)) + b"TELMOIDX")
    return bytes(data)


def granite_config_json(c):
    return json.dumps({
        "model_type": "granite_speech5_ctc", "vocab_size": c["vocab"], "pad_token_id": c["blank"],
        "encoder_config": {
            "model_type": "granite_speech5_encoder", "hidden_size": c["d_model"],
            "num_attention_heads": c["heads"], "head_dim": c["head_dim"],
            "num_hidden_layers": c["layers"], "intermediate_size": c["ff"],
            "conv_kernel_size": c["conv_kernel"],
            "conv_expansion_factor": c["conv_channels"] // c["d_model"],
            "num_mel_bins": c["n_mels"], "context_size": c["context"],
            "max_position_embeddings": c["max_relative"], "vocab_size": c["vocab"],
            "subsample_layers": list(c["subsample_layers"])}}).encode()


def parakeet_config_json(c):
    return json.dumps({
        "model_type": "parakeet_tdt", "hidden_act": "relu", "vocab_size": c["vocab"],
        "blank_token_id": c["blank"], "decoder_hidden_size": c["pred_hidden"],
        "num_decoder_layers": c["pred_layers"], "max_symbols_per_step": c["max_symbols"],
        "durations": list(c["durations"]),
        "encoder_config": {
            "hidden_act": "silu", "attention_bias": False, "convolution_bias": False,
            "scale_input": False, "subsampling_factor": 8, "subsampling_conv_kernel_size": 3,
            "subsampling_conv_stride": 2, "hidden_size": c["d_model"],
            "num_attention_heads": c["heads"], "num_hidden_layers": c["layers"],
            "intermediate_size": c["ff"], "conv_kernel_size": c["conv_kernel"],
            "subsampling_conv_channels": c["sub_channels"], "num_mel_bins": c["n_mels"]}}).encode()

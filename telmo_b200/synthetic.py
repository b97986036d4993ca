"""Seeded synthetic inputs for the benchmark configurations (random-init weights, synthetic audio).

The reference measures on LibriSpeech and FLEURS with real checkpoints; neither is available
here, so every workload uses seeded synthetic data of the configured shapes:

* config 1: one int8-weight linear, A f32 [1500, 1024] ~ N(0, 1), W int8 [4096, 1024] uniform in
  [-127, 127], per-row scales U(1e-3, 1e-2), bias N(0, 0.02), all from seed 0.
* Granite-shaped model: every linear int8 with per-row scales U(1e-3, 1e-2) and biases
  N(0, 0.02); layer-norm gamma 1 + N(0, 0.02) and beta N(0, 0.02); depthwise weights
  N(0, 1/kernel) with bias N(0, 0.02).
* audio: 16 kHz, the sum of 8 sinusoids with frequencies U(50, 4000) Hz, amplitudes
  U(0.02, 0.12) and phases U(0, 2 pi), plus N(0, 0.05) noise.

All draws use numpy's PCG64 generator.
"""

from __future__ import annotations

import math

import numpy as np

SAMPLE_RATE = 16000


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def panels_from_rows(q: np.ndarray, scales: np.ndarray):
    """Lays out int8 rows [n, k] and their scales [n] in the reference's 16-output panels
    (src/quant.rs:1-13): panel p holds k runs of 16 outputs. Returns (values, scales)."""
    n, k = q.shape
    panels = (n + 15) // 16
    padded = np.zeros((panels * 16, k), np.int8)
    padded[:n] = q
    values = padded.reshape(panels, 16, k).transpose(0, 2, 1).reshape(-1)
    s = np.zeros(panels * 16, np.float32)
    s[:n] = scales
    return np.ascontiguousarray(values), s


def rows_from_panels(values: np.ndarray, n: int, k: int) -> np.ndarray:
    panels = (n + 15) // 16
    return np.ascontiguousarray(values.reshape(panels, k, 16).transpose(0, 2, 1).reshape(-1, k)[:n])


def int8_matrix(g: np.random.Generator, n: int, k: int, scales: str = "spec"):
    """An int8 weight matrix in panels: values uniform in [-127, 127] and one scale per row.

    scales="spec": U(1e-3, 1e-2), the benchmark configurations' distribution.
    scales="conditioned": U(0.5, 1.5) / (73.3 * sqrt(k)), so a row's weights have standard
    deviation about 1 / sqrt(k) as in trained layers (73.3 is the standard deviation of the
    uniform int8 values)."""
    q = g.integers(-127, 128, size=(n, k), dtype=np.int8)
    if scales == "spec":
        s = g.uniform(1e-3, 1e-2, size=n)
    elif scales == "conditioned":
        s = g.uniform(0.5, 1.5, size=n) / (73.3 * math.sqrt(k))
    else:
        raise ValueError(f"unknown scale distribution {scales}")
    values, s = panels_from_rows(q, s.astype(np.float32))
    return values, s, n, k


def q8_0_panels(w: np.ndarray):
    """quant::encode for Precision::Q8_0 (src/quant.rs:202-269, quantize_q8_0_block :172-183) of
    a row-major f32 [n, k] matrix, k a multiple of 32: per block of 32 inputs d = amax / 127,
    q = round(x * (1 / d)) half away from zero, the scale kept as its f16 value. Returns (values
    int8 panels, scales f32 in panel, block, output order)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    blocks = k // 32
    b = w.reshape(n, blocks, 32)
    d = (np.abs(b).max(axis=2) / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    x = (b * inv[..., None]).astype(np.float32)
    q = np.sign(x) * np.floor(np.abs(x).astype(np.float64) + 0.5)
    q = np.clip(q, -128, 127).astype(np.int8).reshape(n, k)
    panels = (n + 15) // 16
    qp = np.zeros((panels * 16, k), np.int8)
    qp[:n] = q
    sp = np.zeros((panels * 16, blocks), np.float32)
    sp[:n] = d.astype(np.float16).astype(np.float32)
    values = qp.reshape(panels, 16, k).transpose(0, 2, 1).reshape(-1)
    scales = sp.reshape(panels, 16, blocks).transpose(0, 2, 1).reshape(-1)
    return np.ascontiguousarray(values), np.ascontiguousarray(scales)


def as_q8_0(entry):
    """An Int8 matrix entry (values, scales, n, k) re-quantized to Q8_0 from its f32 values:
    (values, scales, n, k, "q8_0")."""
    values, s, n, k = entry
    w = rows_from_panels(values, n, k).astype(np.float32) * np.asarray(s, np.float32)[:n, None]
    v, sc = q8_0_panels(w)
    return v, sc, n, k, "q8_0"


def config1(seed: int = 0, m: int = 1500, k: int = 1024, n: int = 4096):
    """Config 1: (a [m, k] f32, (values, scales, n, k) int8 panels, bias [n] f32)."""
    g = rng(seed)
    a = g.standard_normal((m, k), dtype=np.float32)
    w = int8_matrix(g, n, k)
    bias = (g.standard_normal(n) * 0.02).astype(np.float32)
    return a, w, bias


GRANITE = dict(d_model=1024, heads=8, head_dim=128, layers=16, ff=4096, conv_kernel=15,
               conv_channels=2048, n_mels=80, context=128, max_relative=512,
               subsample_layers=[0, 1], vocab=2049, blank=0)


def granite_config(**overrides) -> dict:
    c = dict(GRANITE)
    c.update(overrides)
    return c


def granite_entries(config: dict, seed: int = 1, scales: str = "spec", precision: str = "int8") -> dict:
    """Random-init weights of a Granite-shaped model, named as the reference's pack entries
    (src/granite.rs:224-371): matrices as (values, scales, n, k), vectors as f32 arrays. With
    precision="q8_0" the matrices whose inputs come in whole blocks of 32 are re-quantized to
    Q8_0, except the relative-position tables, which stay Int8.

    With scales="spec" (the benchmark's distribution) the model is chaotic: its attention and
    self-conditioning softmaxes are nearly one-hot, and a 1e-6 relative change of the input
    grows about 3x per block in the reference's own f32 arithmetic. scales="conditioned" gives
    weights of trained-layer size, whose outputs are stable under rounding."""
    g = rng(seed)
    c = config
    d, cc, ff, k = c["d_model"], c["conv_channels"], c["ff"], c["conv_kernel"]
    e = {}

    def int8m(n, kk):
        return int8_matrix(g, n, kk, scales)

    def lin(name, n, kk):
        e[name] = int8m(n, kk)
        e[name + ".b"] = (g.standard_normal(n) * 0.02).astype(np.float32)

    def norm(name):
        e[name + ".w"] = (1.0 + g.standard_normal(d) * 0.02).astype(np.float32)
        e[name + ".b"] = (g.standard_normal(d) * 0.02).astype(np.float32)

    lin("input", d, 4 * c["n_mels"])
    for i in range(c["layers"]):
        o = f"blocks.{i}"
        for f in ("ff1", "ff2"):
            norm(f"{o}.{f}.norm")
            lin(f"{o}.{f}.up", ff, d)
            lin(f"{o}.{f}.down", d, ff)
        norm(f"{o}.norm_att")
        e[f"{o}.qkv"] = int8m(3 * d, d)
        e[f"{o}.rel"] = int8m(2 * c["context"] - 1, c["head_dim"])
        lin(f"{o}.out", d, d)
        norm(f"{o}.norm_conv")
        lin(f"{o}.pw1", 2 * cc, d)
        e[f"{o}.dw.w"] = (g.standard_normal((k, cc)) / math.sqrt(k)).astype(np.float32)
        e[f"{o}.dw.b"] = (g.standard_normal(cc) * 0.02).astype(np.float32)
        lin(f"{o}.pw2", d, cc)
        norm(f"{o}.norm_out")
    lin("head", c["vocab"], d)
    lin("mid", d, c["vocab"])
    if precision == "q8_0":
        e = {name: as_q8_0(v) if isinstance(v, tuple) and v[3] % 32 == 0 and not name.endswith(".rel")
             else v for name, v in e.items()}
    elif precision != "int8":
        raise ValueError(f"unknown precision {precision}")
    return e


PARAKEET = dict(d_model=1024, heads=8, layers=24, ff=4096, conv_kernel=9, sub_channels=256,
                n_mels=128, pred_hidden=640, pred_layers=2, vocab=8193, blank=8192,
                durations=[0, 1, 2, 3, 4], max_symbols=10)


def parakeet_config(**overrides) -> dict:
    c = dict(PARAKEET)
    c.update(overrides)
    return c


def parakeet_entries(config: dict, seed: int = 3, scales: str = "spec", precision: str = "int8") -> dict:
    """Random-init weights of a Parakeet-TDT-shaped model, named as the reference's pack entries
    (src/parakeet.rs:341-486): matrices as (values, scales, n, k), vectors as f32 arrays; with
    precision="q8_0" every matrix is then re-quantized to Q8_0, the reference's recommended
    Parakeet precision (src/model.rs:94-102), as (values, scales, n, k, "q8_0"). The
    subsampling convolutions draw N(0, 1/9) (weights [9, channels], tap first), layer norms
    gamma 1 + N(0, 0.02) and beta N(0, 0.02), biases N(0, 0.02), depthwise weights
    N(0, 1/kernel), bias_u and bias_v N(0, 0.02), the embedding N(0, 1)."""
    g = rng(seed)
    c = config
    d, ch, h, k = c["d_model"], c["sub_channels"], c["pred_hidden"], c["conv_kernel"]
    outputs = c["vocab"] + len(c["durations"])
    e = {}

    def int8m(n, kk):
        return int8_matrix(g, n, kk, scales)

    def f32(shape, std, mean=0.0):
        return (mean + g.standard_normal(shape) * std).astype(np.float32)

    for name in ("conv0", "dw1", "dw2"):
        e[f"sub.{name}.w"] = f32((9, ch), 1.0 / 3.0)
        e[f"sub.{name}.b"] = f32(ch, 0.02)
    for name in ("pw1", "pw2"):
        e[f"sub.{name}"] = int8m(ch, ch)
        e[f"sub.{name}.b"] = f32(ch, 0.02)
    e["sub.linear"] = int8m(d, ch * (c["n_mels"] // 8))
    e["sub.linear.b"] = f32(d, 0.02)
    for i in range(c["layers"]):
        o = f"layers.{i}"
        for nm in ("norm_ff1", "norm_att", "norm_conv", "norm_ff2", "norm_out"):
            e[f"{o}.{nm}.w"] = f32(d, 0.02, 1.0)
            e[f"{o}.{nm}.b"] = f32(d, 0.02)
        e[f"{o}.ff1_in"] = int8m(c["ff"], d)
        e[f"{o}.ff1_out"] = int8m(d, c["ff"])
        e[f"{o}.qkv"] = int8m(3 * d, d)
        e[f"{o}.pos"] = int8m(d, d)
        e[f"{o}.bias_u"] = f32(d, 0.02)
        e[f"{o}.bias_v"] = f32(d, 0.02)
        e[f"{o}.out"] = int8m(d, d)
        e[f"{o}.pw1"] = int8m(2 * d, d)
        e[f"{o}.dw.w"] = f32((k, d), 1.0 / math.sqrt(k))
        e[f"{o}.dw.b"] = f32(d, 0.02)
        e[f"{o}.pw2"] = int8m(d, d)
        e[f"{o}.ff2_in"] = int8m(c["ff"], d)
        e[f"{o}.ff2_out"] = int8m(d, c["ff"])
    for l in range(c["pred_layers"]):
        e[f"dec.lstm.{l}"] = int8m(4 * h, 2 * h)
        e[f"dec.lstm.{l}.b"] = f32(4 * h, 0.02)
    e["dec.embedding"] = f32((c["vocab"], h), 1.0)
    e["dec.pred_proj"] = int8m(h, h)
    e["dec.pred_proj.b"] = f32(h, 0.02)
    e["dec.enc_proj"] = int8m(h, d)
    e["dec.enc_proj.b"] = f32(h, 0.02)
    e["dec.joint"] = int8m(outputs, h)
    e["dec.joint.b"] = f32(outputs, 0.02)
    if precision == "q8_0":
        e = {name: as_q8_0(v) if isinstance(v, tuple) else v for name, v in e.items()}
    elif precision != "int8":
        raise ValueError(f"unknown precision {precision}")
    return e


def audio(seconds: float, seed: int = 2) -> np.ndarray:
    """16 kHz f32 audio: 8 random sinusoids (50-4000 Hz) plus N(0, 0.05) noise."""
    g = rng(seed)
    n = int(round(seconds * SAMPLE_RATE))
    t = np.arange(n, dtype=np.float64) / SAMPLE_RATE
    freq = g.uniform(50.0, 4000.0, 8)
    amp = g.uniform(0.02, 0.12, 8)
    phase = g.uniform(0.0, 2 * math.pi, 8)
    x = np.zeros(n, np.float64)
    for f, a, p in zip(freq, amp, phase):
        x += a * np.sin(2 * math.pi * f * t + p)
    x += g.standard_normal(n) * 0.05
    return x.astype(np.float32)


def lengths_uniform(count: int, lo: float, hi: float, seed: int) -> np.ndarray:
    """Utterance lengths in seconds, uniform in [lo, hi] (config 3)."""
    return rng(seed).uniform(lo, hi, count)


def lengths_log_uniform(count: int, lo: float, hi: float, seed: int) -> np.ndarray:
    """Utterance lengths in seconds, log-uniform in [lo, hi] (config 5)."""
    return np.exp(rng(seed).uniform(math.log(lo), math.log(hi), count))

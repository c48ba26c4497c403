"""Synthetic checkpoint and audio for the Nemotron-3 diarization forward pass.

The real checkpoint (`model.safetensors`, `config.json`, `processor_config.json`)
and the reference's evaluation audio are not available, so everything the
library consumes is generated here from fixed seeds:

* ``write_checkpoint(dir)`` writes the two JSON configs and a random-init
  ``model.safetensors`` with exactly the 417 tensor names and shapes the
  reference loads (src/encoder.rs:66-97, src/head.rs:67-79, src/model.rs:151-153).
  Linear and conv weights are N(0, 0.02), biases 0, LayerNorm gamma 1 / beta 0,
  ``silence_embeds`` N(0, 0.02); one ``numpy.random.Generator(PCG64(seed))``
  draws the weight tensors in sorted-name order, each in C order.
* ``clip(...)`` synthesises 16 kHz mono float32 "meetings": harmonic speakers
  (f0 ~ U[100, 250] Hz, 10 harmonics at 1/k, amplitude-modulated at 3-6 Hz)
  taking turns with a target overlap, optional telephone band-pass
  (4th-order Butterworth 300-3400 Hz), optional reverb (exponentially decaying
  Gaussian-noise impulse response) and white noise at a target SNR.
* ``config0_audio`` / ``config2_audio`` / ``config3_session`` / ``config4_clip``
  are the seeded inputs of the benchmark configurations.

Config values the reference reads from the checkpoint JSON (src/config.rs:43-131)
are pinned by its code where possible (hidden 512, 31 layers, 8 heads, 2048 FFN,
128 mels, subsampling 8, head 192, 8 speakers, offline chunk 340 + 40,
speaker cache 264 with one silence slot per speaker, min-positive threshold 16);
the rest (streaming FIFO length and update period, boost rates) are chosen here
and recorded in the generated JSON.
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np

SAMPLE_RATE = 16000

MODEL_CONFIG = {
    "audio_config": {
        "hidden_size": 512,
        "num_hidden_layers": 31,
        "num_attention_heads": 8,
        "num_key_value_heads": 8,
        "intermediate_size": 2048,
        "max_position_embeddings": 4096,
        "num_mel_bins": 128,
        "subsampling_factor": 8,
        "rope_parameters": {"rope_theta": 10000.0, "partial_rotary_factor": 1.0},
    },
    "head_config": {
        "audio_hidden_size": 512,
        "hidden_size": 192,
        "num_speakers": 8,
        "subsampling_factor": 8,
    },
    "streaming_config": {
        "fifo_length": 100,
        "speaker_cache_length": 264,
        "speaker_cache_silence_frames_per_speaker": 1,
        "speaker_cache_update_period": 40,
        "prediction_score_threshold": 0.25,
        "min_positive_scores_rate": 0.5,
        "strong_boost_rate": 0.75,
        "weak_boost_rate": 1.5,
        "latest_frames_score_boost": 0.05,
        "subsampling_factor": 8,
        "num_speakers": 8,
    },
    "chunk_length": 340,
    "chunk_right_context": 40,
    "fifo_length": 40,
    "speaker_cache_update_period": 300,
}

PROCESSOR_CONFIG = {
    "feature_extractor": {
        "feature_size": 128,
        "n_fft": 512,
        "hop_length": 160,
        "win_length": 400,
        "sampling_rate": SAMPLE_RATE,
        "preemphasis": 0.97,
    },
    "streaming_modes": {
        "low_latency": [9, 4],
        "very_low_latency": [6, 2],
        "ultra_low_latency": [3, 1],
    },
    "subsampling_factor": 8,
}


def tensor_specs(cfg: dict = MODEL_CONFIG):
    """(name, shape, kind) for every checkpoint tensor; kind picks the init."""
    a = cfg["audio_config"]
    hc = cfg["head_config"]
    h, inter, sub, mels = a["hidden_size"], a["intermediate_size"], a["subsampling_factor"], a["num_mel_bins"]
    hh, ns = hc["hidden_size"], hc["num_speakers"]
    p = "model.audio_tower"
    specs = [
        (f"{p}.embedder.projection.weight", (h, sub * mels), "w"),
        (f"{p}.input_layer_norm.weight", (h,), "g"),
        (f"{p}.input_layer_norm.bias", (h,), "b"),
        (f"{p}.layer_norm.weight", (h,), "g"),
        (f"{p}.layer_norm.bias", (h,), "b"),
    ]
    for i in range(a["num_hidden_layers"]):
        b = f"{p}.layers.{i}"
        specs += [
            (f"{b}.layer_norm1.weight", (h,), "g"),
            (f"{b}.layer_norm1.bias", (h,), "b"),
            (f"{b}.self_attn.q_proj.weight", (h, h), "w"),
            (f"{b}.self_attn.k_proj.weight", (h, h), "w"),
            (f"{b}.self_attn.v_proj.weight", (h, h), "w"),
            (f"{b}.self_attn.o_proj.weight", (h, h), "w"),
            (f"{b}.self_attn.o_proj.bias", (h,), "b"),
            (f"{b}.layer_norm2.weight", (h,), "g"),
            (f"{b}.layer_norm2.bias", (h,), "b"),
            (f"{b}.mlp.fc1.weight", (inter, h), "w"),
            (f"{b}.mlp.fc1.bias", (inter,), "b"),
            (f"{b}.mlp.fc2.weight", (h, inter), "w"),
            (f"{b}.mlp.fc2.bias", (h,), "b"),
        ]
    specs += [
        ("model.proj.weight", (hh, h), "w"),
        ("model.proj.bias", (hh,), "b"),
        ("model.upsampler.conv.weight", (hh * sub, hh, 3), "w"),
        ("model.upsampler.conv.bias", (hh * sub,), "b"),
        ("classifier.dense.weight", (hh, hh), "w"),
        ("classifier.dense.bias", (hh,), "b"),
        ("classifier.out_proj.weight", (ns, hh), "w"),
        ("classifier.out_proj.bias", (ns,), "b"),
        ("silence_embeds", (h,), "w"),
    ]
    return specs


def make_weights(seed: int = 0, cfg: dict = MODEL_CONFIG, std: float = 0.02) -> dict:
    """Random-init weights: N(0, std) weights, zero biases, LN gamma 1 / beta 0."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name, shape, kind in sorted(tensor_specs(cfg), key=lambda s: s[0]):
        if kind == "w":
            out[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        elif kind == "g":
            out[name] = np.ones(shape, np.float32)
        else:
            out[name] = np.zeros(shape, np.float32)
    return out


def save_safetensors(path: str, tensors: dict) -> None:
    """Minimal safetensors writer (F32 only): u64 header length, JSON header, data."""
    header = {}
    offset = 0
    names = sorted(tensors)
    for n in names:
        nbytes = tensors[n].size * 4
        header[n] = {"dtype": "F32", "shape": list(tensors[n].shape), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    hjson = json.dumps(header, separators=(",", ":")).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for n in names:
            f.write(np.ascontiguousarray(tensors[n], dtype="<f4").tobytes())


def load_safetensors(path: str) -> dict:
    """Read an F32 safetensors file into numpy arrays (test and oracle helper)."""
    with open(path, "rb") as f:
        raw = f.read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8 : 8 + hlen])
    base = 8 + hlen
    out = {}
    for n, meta in header.items():
        if n == "__metadata__":
            continue
        s, e = meta["data_offsets"]
        out[n] = np.frombuffer(raw, dtype="<f4", count=(e - s) // 4, offset=base + s).reshape(meta["shape"])
    return out


def write_checkpoint(directory: str, seed: int = 0, cfg: dict = MODEL_CONFIG, proc: dict = PROCESSOR_CONFIG,
                     weights: dict | None = None) -> str:
    """Write config.json, processor_config.json and model.safetensors into `directory`."""
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    with open(os.path.join(directory, "processor_config.json"), "w") as f:
        json.dump(proc, f, indent=1)
    save_safetensors(os.path.join(directory, "model.safetensors"), weights if weights is not None else make_weights(seed, cfg))
    return directory


# --------------------------------------------------------------------------- audio


def _turns(rng, duration, n_spk, turn_lo, turn_hi, overlap):
    """Speaker turns (speaker, start, end) in seconds covering `duration`.

    Each turn starts `overlap * previous_length` before the previous turn ends,
    so roughly `overlap` of the speech time carries two talkers.
    """
    turns = []
    t = 0.0
    prev = -1
    while t < duration:
        length = rng.uniform(turn_lo, turn_hi)
        spk = int(rng.integers(n_spk))
        if n_spk > 1:
            while spk == prev:
                spk = int(rng.integers(n_spk))
        turns.append((spk, t, min(duration, t + length)))
        prev = spk
        t = t + length * (1.0 - overlap) + (0.0 if overlap > 0 else rng.uniform(0.0, 0.3))
    return turns


def clip(seed: int, duration_s: float, n_speakers: int, turn_range=(1.0, 4.0), overlap: float = 0.2,
         snr_db: float = 20.0, bandpass: bool = False, rt60: float | None = None, peak: float = 0.5) -> np.ndarray:
    """One synthetic multi-speaker recording, 16 kHz mono float32."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n = int(round(duration_s * SAMPLE_RATE))
    t = np.arange(n, dtype=np.float64) / SAMPLE_RATE
    f0 = rng.uniform(100.0, 250.0, n_speakers)
    am = rng.uniform(3.0, 6.0, n_speakers)
    phase = rng.uniform(0, 2 * np.pi, (n_speakers, 10))
    x = np.zeros(n, np.float64)
    fade = int(0.01 * SAMPLE_RATE)
    for spk, s0, s1 in _turns(rng, duration_s, n_speakers, turn_range[0], turn_range[1], overlap):
        a, b = int(s0 * SAMPLE_RATE), int(s1 * SAMPLE_RATE)
        if b <= a:
            continue
        tt = t[a:b]
        voice = np.zeros(b - a)
        for k in range(1, 11):
            fk = k * f0[spk]
            if fk >= SAMPLE_RATE / 2:
                break
            voice += np.sin(2 * np.pi * fk * tt + phase[spk, k - 1]) / k
        voice *= 0.6 + 0.4 * np.sin(2 * np.pi * am[spk] * tt)
        env = np.ones(b - a)
        m = min(fade, (b - a) // 2)
        if m > 0:
            ramp = np.linspace(0.0, 1.0, m)
            env[:m] = ramp
            env[-m:] = ramp[::-1]
        x[a:b] += voice * env
    if rt60 is not None:
        ir_len = int(rt60 * SAMPLE_RATE)
        decay = np.exp(-6.9077 * np.arange(ir_len) / ir_len)  # -60 dB at rt60
        ir = rng.standard_normal(ir_len) * decay
        ir[0] = 1.0
        ir /= np.sqrt(np.sum(ir**2))
        from scipy.signal import fftconvolve

        x = fftconvolve(x, ir)[:n]
    if bandpass:
        from scipy.signal import butter, sosfilt

        sos = butter(4, [300.0, 3400.0], btype="bandpass", fs=SAMPLE_RATE, output="sos")
        x = sosfilt(sos, x)
    p_sig = np.mean(x**2) if np.any(x) else 1.0
    noise = rng.standard_normal(n) * np.sqrt(p_sig / 10 ** (snr_db / 10.0))
    x = x + noise
    x *= peak / max(np.max(np.abs(x)), 1e-12)
    return x.astype(np.float32)


def config0_audio() -> np.ndarray:
    """30 s, seed 1, 3 speakers, turns U[1,4] s, 20 % overlap, 20 dB SNR, peak 0.5."""
    return clip(1, 30.0, 3, (1.0, 4.0), 0.2, 20.0)


def config2_audio(duration_s: float = 3600.0) -> np.ndarray:
    """60 min, 4 speakers, turns U[0.5,6] s, 30 % overlap, telephone band, 15 dB SNR."""
    return clip(2, duration_s, 4, (0.5, 6.0), 0.3, 15.0, bandpass=True)


def config3_session(i: int, duration_s: float = 600.0) -> np.ndarray:
    """Streaming session i (seed 100+i): 2-8 speakers, 0-60 % overlap, 10 min."""
    rng = np.random.Generator(np.random.PCG64(100 + i + 7919))
    n_spk = int(rng.integers(2, 9))
    ovl = float(rng.uniform(0.0, 0.6))
    return clip(100 + i, duration_s, n_spk, (1.0, 4.0), ovl, 20.0)


def config4_clip(i: int, duration_s: float = 60.0) -> np.ndarray:
    """Batch clip i (seed 1000+i): up to 8 speakers, 61 % overlap, RT60 0.5 s, 8 dB SNR."""
    rng = np.random.Generator(np.random.PCG64(1000 + i + 7919))
    n_spk = int(rng.integers(2, 9))
    return clip(1000 + i, duration_s, n_spk, (1.0, 4.0), 0.61, 8.0, rt60=0.5)

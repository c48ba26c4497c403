"""The `diarize` command-line tool (nemotron3-diarization-wgpu_b200/diarize, built from
csrc/diarize.cpp): the reference's src/bin/diarize.rs over the C ABI.

CPU: usage, argument errors, and a clear failure when no B200 is present.  GPU: the
JSON report (reference field set, serde_json's sorted key order) from .npy and 16-bit
WAV input, checked against the Python API on the same samples."""

import json
import math
import os
import subprocess
import wave

import numpy as np
import pytest

import synth
from conftest import gpu_available

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "nemotron3-diarization-wgpu_b200", "diarize")
FIELDS = ["audio", "cache_compressed", "cache_frames", "duration_s", "fifo_frames", "forward_s", "load_s", "mode",
          "num_chunks", "num_frames", "num_segments", "num_speakers", "rtfx", "segments", "speakers"]


def run(*args):
    if not os.path.exists(CLI):
        pytest.skip("diarize is not built (make -C nemotron3-diarization-wgpu_b200)")
    return subprocess.run([CLI, *args], capture_output=True, text=True, timeout=600)


def test_usage():
    r = run("--help")
    assert r.returncode == 0 and "usage: diarize" in r.stdout and "ultra_low_latency" in r.stdout


@pytest.mark.parametrize("args,msg", [(["--bogus"], "unknown flag --bogus"), ([], "no audio file given"),
                                      (["x.npy", "--mode", "fast"], "unknown mode fast"),
                                      (["x.npy", "--out"], "--out needs a value"),
                                      (["x.npy", "--threshold", "abc"], "--threshold needs a finite number, got abc"),
                                      (["x.npy", "--threshold", "1e99"], "--threshold needs a finite number"),
                                      (["x.npy", "--threshold", "0.5x"], "--threshold needs a finite number"),
                                      (["x.npy", "--device", "-1"], "--device needs a non-negative integer"),
                                      (["x.npy", "--device", "one"], "--device needs a non-negative integer")])
def test_argument_errors(args, msg):
    r = run(*args)
    assert r.returncode == 1 and msg in r.stderr


def test_unreadable_audio_is_an_error(tmp_path):
    p = tmp_path / "bad.npy"
    p.write_bytes(b"not numpy")
    r = run(str(p))
    assert r.returncode == 1 and "not a .npy file" in r.stderr


def _npy_bytes(descr, shape, payload, fortran=False, major=1):
    hdr = "{'descr': '%s', 'fortran_order': %s, 'shape': %s, }" % (descr, fortran, shape)
    pad = (-(len(hdr) + 1 + (10 if major == 1 else 12))) % 64
    hdr = (hdr + " " * pad + "\n").encode()
    size = len(hdr).to_bytes(2 if major == 1 else 4, "little")
    return b"\x93NUMPY" + bytes([major, 0]) + size + hdr + payload


def _riff(*chunks, size_fix=0):
    body = b"WAVE" + b"".join(cid + len(data).to_bytes(4, "little") + data + (b"\0" if len(data) % 2 else b"")
                             for cid, data in chunks)
    return b"RIFF" + (len(body) + size_fix).to_bytes(4, "little") + body


def _fmt(tag, ch, bits, extensible_tag=None):
    rate, align = 16000, ch * bits // 8
    f = tag.to_bytes(2, "little") + ch.to_bytes(2, "little") + rate.to_bytes(4, "little") + \
        (rate * align).to_bytes(4, "little") + align.to_bytes(2, "little") + bits.to_bytes(2, "little")
    if extensible_tag is not None:
        f += (22).to_bytes(2, "little") + bits.to_bytes(2, "little") + (0).to_bytes(4, "little") + \
             extensible_tag.to_bytes(2, "little") + bytes(14)
    return f


MALFORMED = {
    "short.npy": (b"\x93NUMPY\x02\x00\x10\x00", "truncated .npy header"),
    "header.npy": (b"\x93NUMPY\x01\x00\xff\x00{'descr'", "truncated .npy header"),
    "dtype.npy": (_npy_bytes("<f8", "(4,)", bytes(32)), "expected <f4 or <i8, got <f8"),
    "fortran.npy": (_npy_bytes("<f4", "(3, 5)", bytes(4 * 14), fortran=True), "does not match its shape"),
    "riff.wav": (b"RIFX\0\0\0\0WAVE", "not a RIFF/WAVE file"),
    "nofmt.wav": (_riff((b"data", bytes(8))), "no fmt chunk"),
    "nodata.wav": (_riff((b"fmt ", _fmt(1, 1, 16))), "no data chunk"),
    "shortfmt.wav": (_riff((b"fmt ", _fmt(1, 1, 16)[:12]), (b"data", bytes(8))), "truncated fmt chunk"),
    "shortext.wav": (_riff((b"fmt ", _fmt(0xFFFE, 1, 32)[:16] + (22).to_bytes(2, "little"))), "truncated fmt chunk"),
    "cutext.wav": (b"RIFF\0\0\0\0WAVEfmt \x28\0\0\0" + _fmt(0xFFFE, 1, 32)[:16], "truncated fmt chunk"),
    "bits24.wav": (_riff((b"fmt ", _fmt(1, 1, 24)), (b"data", bytes(12))), "must be 16-bit PCM or float32"),
    "nochan.wav": (_riff((b"fmt ", _fmt(1, 0, 16)), (b"data", bytes(8))), "has no channels"),
    "ragged.wav": (_riff((b"fmt ", _fmt(1, 2, 16)), (b"data", bytes(6))), "not a whole number of frames"),
}


@pytest.mark.parametrize("name", sorted(MALFORMED))
def test_malformed_audio_is_a_clean_error(tmp_path, name):
    """Malformed .npy / .wav input ends with exit code 1 and a message that names the
    problem: never a crash, and never a read past the end of the file."""
    data, msg = MALFORMED[name]
    p = tmp_path / name
    p.write_bytes(data)
    r = run(str(p), "--model", str(tmp_path))
    assert r.returncode == 1 and msg in r.stderr, (r.returncode, r.stderr)


WELL_FORMED = {
    "v1_f4.npy": _npy_bytes("<f4", "(6,)", np.arange(6, dtype="<f4").tobytes()),
    "v2_f4.npy": _npy_bytes("<f4", "(6,)", np.arange(6, dtype="<f4").tobytes(), major=2),
    "i8.npy": _npy_bytes("<i8", "(2, 3)", np.arange(6, dtype="<i8").tobytes()),
    "fortran.npy": _npy_bytes("<f4", "(2, 3)", np.arange(6, dtype="<f4").tobytes(), fortran=True),
    "pcm16_stereo.wav": _riff((b"fmt ", _fmt(1, 2, 16)), (b"LIST", b"odd"), (b"data", bytes(8))),
    "float.wav": _riff((b"fmt ", _fmt(3, 1, 32)), (b"data", np.ones(4, "<f4").tobytes())),
    "extensible.wav": _riff((b"fmt ", _fmt(0xFFFE, 1, 32, extensible_tag=3)), (b"data", np.ones(4, "<f4").tobytes())),
}


@pytest.mark.skipif(gpu_available(), reason="uses the model-load failure without a GPU as the stop point")
@pytest.mark.parametrize("name", sorted(WELL_FORMED))
def test_well_formed_audio_is_read(tmp_path, tiny_checkpoint_dir, name):
    """Every supported layout is read; without a B200 the run then stops at model load."""
    p = tmp_path / name
    p.write_bytes(WELL_FORMED[name])
    r = run(str(p), "--model", tiny_checkpoint_dir)
    assert r.returncode == 1 and "model load" in r.stderr, r.stderr


@pytest.mark.skipif(gpu_available(), reason="checks the failure without a GPU")
def test_without_a_gpu_model_load_fails_cleanly(tmp_path, tiny_checkpoint_dir):
    p = tmp_path / "a.npy"
    np.save(p, synth.clip(3, 1.0, 2))
    r = run(str(p), "--model", tiny_checkpoint_dir)
    assert r.returncode == 1 and "model load" in r.stderr


def hundredths(v):
    """(v as f64 * 100).round() / 100 (src/segments.rs:31-33): halves round away from zero."""
    return math.floor(float(v) * 100.0 + 0.5) / 100.0


def _write_wav16(path, x):
    pcm = np.clip(np.round(x * 32768.0), -32768, 32767).astype("<i2")
    with wave.open(str(path), "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(16000)
        w.writeframes(pcm.tobytes())
    return pcm.astype(np.float32) / np.float32(32768.0)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,mode", [("npy", "offline"), ("wav", "ultra_low_latency")])
def test_report_matches_the_oracle(tmp_path, tiny_checkpoint_dir, tiny_oracle, fmt, mode):
    """The CLI's report on the GPU against the CPU oracle's run of the same samples:
    the RunOutput counts, and segments IDENTICAL to the oracle's (the frame_check gate,
    src/bin/frame_check.rs:215-233), rounded to hundredths as the reference prints them."""
    import oracle

    x = synth.clip(21, 6.0, 3)
    path = tmp_path / f"clip.{fmt}"
    if fmt == "npy":
        np.save(path, x)
        samples = x
    else:
        samples = _write_wav16(path, x)
    out = tmp_path / "report.json"
    r = run(str(path), "--model", tiny_checkpoint_dir, "--mode", mode, "--out", str(out))
    assert r.returncode == 0, r.stderr
    text = out.read_text()
    rep = json.loads(text)
    assert list(rep) == FIELDS  # serde_json prints object keys sorted
    ref = tiny_oracle.run_offline(samples) if mode == "offline" else tiny_oracle.run_streaming(samples, mode)
    assert rep["mode"] == mode.replace("_", "")
    assert (rep["num_frames"], rep["num_chunks"], rep["cache_frames"], rep["fifo_frames"], rep["cache_compressed"]) == \
        (ref["num_frames"], ref["num_chunks"], ref["cache_frames"], ref["fifo_frames"], bool(ref["cache_compressed"]))
    assert rep["duration_s"] == math.floor(len(samples) / 16000.0 * 1000.0 + 0.5) / 1000.0
    segs = oracle.extract_speaker_dict(np.asarray(ref["logits"], np.float32).ravel(), ref["num_frames"], 8, 0.01)
    assert segs and rep["num_segments"] == len(segs) == len(rep["segments"])
    for got, (start, end, speaker) in zip(rep["segments"], segs):
        assert list(got) == ["End", "Speaker", "Start"]
        assert got["Speaker"] == speaker
        assert got["Start"] == hundredths(start) and got["End"] == hundredths(end)
    assert rep["speakers"] == sorted({sp for _, _, sp in segs}) and rep["num_speakers"] == len(rep["speakers"])

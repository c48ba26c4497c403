"""The full 31-layer model against the oracle's frozen outputs, on every BASELINE
configuration and mode, through the C ABI on a B200.

Fixtures (tests/golden/full/, written by tests/golden/make_full_golden.py on the
CPU) hold the oracle's RunOutput for config 0 in the three streaming modes, a
config 4 clip offline and in ultra-low latency, the last clip of a 128-clip batch,
the first 120 s of a config 3 session and a 10 min recording with config 2's
recipe.  Each run is gated by the reference's frame_check (src/bin/frame_check.rs:
170-240): equal frame, chunk and cache counts, per-logit maxdiff < 2e-2, and zero
sigmoid>0.5 flips with IDENTICAL segments -- outside the fixture's fp32 noise band.

The noise band: BASELINE's random-init weights make the logits about N(0, 0.006),
so some lie within 1e-7 of the decision, and the speaker cache's ranking turns on
near-ties whose order any change of rounding can swap (offline runs with
compression then move later logits by ~1e-5).  tests/golden/noise_floor.py measures
this with a second, equally valid fp32 build of the oracle (FMA-contracted):
against the fixtures it differs by up to its recorded maxdiff, and on config 2 it
flips 6 decisions and changes segments itself.  So a decision may differ only where
the oracle's logit lies within BAND x that recorded maxdiff of the boundary, and the
segments must be identical once those in-band decisions are taken from the oracle.
A fixture without a recorded noise floor gets the strict gates.  The streaming runs
use the checkpoint's real cache geometry (264 frames, FIFO 100).

The batch tests run the benchmark's exact path: 128 config 4 clips per call
through n3d_run_batch_device (inputs in HBM, the eager tower for more than 16
sequences) and through n3d_run_batch (host buffers), with the fixture clips at
batch positions 0 and 127.
"""

import json
import os

import numpy as np
import pytest

import synth
from conftest import frame_check

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "full")
_NOISE_PATH = os.path.join(GOLDEN, "noise_floor.json")
NOISE = json.load(open(_NOISE_PATH)) if os.path.exists(_NOISE_PATH) else {}
BAND = 4.0  # times the second fp32 build's measured maxdiff on the same fixture


def _decision_boundary() -> float:
    """The smallest float32 logit whose f32 sigmoid exceeds 0.5 with the oracle's expf
    (about 1.2e-7, not 0: below it the sigmoid rounds to exactly 0.5)."""
    import oracle

    lo, hi = 0, int(np.float32(1e-5).view(np.int32))  # bit patterns of positive floats
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if oracle.sigmoid_above_half(np.array([mid], np.int32).view(np.float32))[0]:
            hi = mid
        else:
            lo = mid
    return float(np.array([hi], np.int32).view(np.float32)[0])
NAMES = ["c0_low_latency", "c0_very_low_latency", "c0_ultra_low_latency", "c4_clip0_offline", "c4_clip0_ultra",
         "c4_clip127_offline", "c3_session0_120s", "c2_600s_offline"]


def _fixture(name):
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(GOLDEN)))
    from make_full_golden import audio_sha, cases

    make, mode = cases()[name]
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    a = make()
    assert audio_sha(a) == str(z["audio_sha256"]), f"synth.py no longer regenerates the audio of {name}"
    assert str(z["mode"]) == mode
    return a, mode, z


def _gate(got_logits, z, name, counts=None):
    import oracle

    r = frame_check(got_logits, z["logits"])
    assert r["frames_equal"], (np.asarray(got_logits).shape, z["logits"].shape)
    if counts is not None:
        assert counts == (int(z["num_frames"]), int(z["num_chunks"]), int(z["cache_compressed"]),
                          int(z["cache_frames"]), int(z["fifo_frames"]))
    assert r["maxdiff"] < 2e-2, r
    band = BAND * NOISE[name]["maxdiff"] if name in NOISE else 0.0
    r["band"] = band
    want = z["logits"]
    inband = np.abs(want.astype(np.float64) - _decision_boundary()) < band
    # no decision differs outside the fp32 noise band around the decision boundary
    flipped = oracle.sigmoid_above_half(got_logits).reshape(want.shape) != oracle.sigmoid_above_half(want).reshape(
        want.shape)
    r["flips_outside_band"] = int((flipped & ~inband).sum())
    assert r["flips_outside_band"] == 0, r
    if not r["segments_identical"]:
        # the segments differ only through in-band decisions: with those taken from the
        # oracle they are identical
        got = np.asarray(got_logits, np.float32).reshape(-1, 8).copy()
        got[inband] = want[inband]
        segs = lambda l: oracle.extract_speaker_dict(l.ravel(), l.shape[0], 8, 0.01)
        assert segs(got) == segs(want), r
    return r


def _counts(out):
    return (out.num_frames, out.num_chunks, int(out.cache_compressed), out.cache_frames, out.fifo_frames)


@pytest.mark.parametrize("name", NAMES)
def test_full_model_passes_frame_check(gpu_model, name):
    a, mode, z = _fixture(name)
    out = gpu_model.run_offline(a) if mode == "offline" else gpu_model.run_streaming(a, mode)
    r = _gate(out.logits, z, name, _counts(out))
    print(name, {k: r[k] for k in ("maxdiff", "flips", "flips_outside_band", "flip_ref_abs_max", "band",
                                   "segments_identical", "segments")},
          "chunks", out.num_chunks)


def test_full_model_session_in_pieces_equals_run_streaming(gpu_model):
    """A live session fed 240 ms at a time (one ultra-low-latency step of audio per
    push) emits the same rows as run_streaming on the whole recording."""
    a, mode, z = _fixture("c3_session0_120s")
    s = gpu_model.open_session(mode)
    rows = []
    for i in range(0, a.size, 3840):
        rows.append(s.push(a[i:i + 3840]).logits)
    last = s.close()
    rows.append(last.logits)
    s.free()
    got = np.concatenate(rows)
    want = gpu_model.run_streaming(a, mode)
    assert got.shape == want.logits.shape
    assert np.abs(got - want.logits).max() < 1e-6
    assert (last.num_chunks, int(last.cache_compressed), last.cache_frames, last.fifo_frames) == \
        (want.num_chunks, int(want.cache_compressed), want.cache_frames, want.fifo_frames)
    _gate(got, z, "c3_session0_120s")


_CLIPS = {}


def _bench_clips(n):
    """The benchmark's clips on rank 0 of one GPU: config 4 clips 0..n-1 (seeds 1000..)."""
    if n not in _CLIPS:
        _CLIPS[n] = [synth.config4_clip(i) for i in range(n)]
    return _CLIPS[n]


def test_128_clip_device_batch_passes_frame_check_at_both_ends(gpu_model):
    import torch

    clips = _bench_clips(128)
    lens = [c.size for c in clips]
    offs = list(np.cumsum([0] + lens[:-1]))
    frames = gpu_model.batch_out_frames(lens, "offline")
    ooffs = list(np.cumsum([0] + frames[:-1]))
    d_audio = torch.from_numpy(np.concatenate(clips)).cuda()
    d_out = torch.full((sum(frames) * 8,), float("nan"), dtype=torch.float32, device="cuda")
    gpu_model.run_batch_device("offline", d_audio.data_ptr(), offs, lens, d_out.data_ptr(), ooffs)
    dev = d_out.cpu().numpy()
    assert np.isfinite(dev).all()
    for pos, name in ((0, "c4_clip0_offline"), (127, "c4_clip127_offline")):
        _, _, z = _fixture(name)
        got = dev[ooffs[pos] * 8:(ooffs[pos] + frames[pos]) * 8].reshape(-1, 8)
        _gate(got, z, name)


def test_128_clip_host_batch_passes_frame_check_at_both_ends(gpu_model):
    clips = _bench_clips(128)
    outs = gpu_model.run_batch(clips, "offline")
    for pos, name in ((0, "c4_clip0_offline"), (127, "c4_clip127_offline")):
        _, _, z = _fixture(name)
        _gate(outs[pos].logits, z, name, _counts(outs[pos]))


def test_16_clip_streaming_batch_passes_frame_check(gpu_model):
    """The C4 streaming benchmark's batch (16 clips on the tower's CUDA graphs)."""
    clips = _bench_clips(128)[:16]
    outs = gpu_model.run_batch(clips, "ultra_low_latency")
    _, _, z = _fixture("c4_clip0_ultra")
    _gate(outs[0].logits, z, "c4_clip0_ultra", _counts(outs[0]))

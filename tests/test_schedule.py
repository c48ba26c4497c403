"""The host-side chunk arithmetic behind every run, through the C ABI and without a GPU:
ModeParams::resolve (src/config.rs:152-195), Model::streaming_chunks
(src/model.rs:343-365) and the chunk loop's step schedule (src/model.rs:242-336,
478-538; cache counts src/streaming.rs:220-284), checked against the CPU oracle's
per-step traces and the reference's documented figures.  Integer work: exact."""

import json
import os

import numpy as np
import pytest

import n3d
import oracle
import synth
from conftest import tiny_config

MODES = ["low_latency", "very_low_latency", "ultra_low_latency", "offline"]
STREAMING = MODES[:3]


@pytest.fixture(scope="module")
def cfg(checkpoint_dir):
    c = n3d.Config.load(checkpoint_dir)
    yield c
    c.close()


@pytest.fixture(scope="module")
def tiny_cfg(tiny_checkpoint_dir):
    c = n3d.Config.load(tiny_checkpoint_dir)
    yield c
    c.close()


def test_mode_params_match_the_reference_table(cfg):
    """README.md:68-74 of the reference: 9 / 6 / 3 encoder frames per step and
    1040 / 640 / 320 ms of algorithmic latency."""
    per_step = {"low_latency": 9, "very_low_latency": 6, "ultra_low_latency": 3}
    latency = {"low_latency": 1040, "very_low_latency": 640, "ultra_low_latency": 320}
    fe = synth.PROCESSOR_CONFIG["feature_extractor"]
    for mode in STREAMING:
        p = cfg.mode_params(mode)
        assert p["mel_frames_per_step"] // p["subsampling"] == per_step[mode]  # chunk_encoder_frames
        assert p["latency_ms"] == latency[mode]
        assert (p["hop_length"], p["n_fft"], p["subsampling"]) == (160, 512, 8)
        m = p["mel_frames_per_chunk"]
        # src/config.rs:181-190: the first chunk yields exactly M centred frames, a later
        # chunk exactly M uncentred ones
        assert oracle.frame_count(p["first_chunk_samples"], fe, True) == m
        assert oracle.frame_count(p["samples_per_chunk"], fe, False) == m
        assert p["lookahead_encoder_frames"] * p["subsampling"] == m - p["mel_frames_per_step"]
    off = cfg.mode_params("offline")
    assert off["mel_frames_per_chunk"] == off["first_chunk_samples"] == off["samples_per_chunk"] == 0
    assert off["latency_ms"] == (340 + 40) * 80


def _chunks_restated(p, n, fe):
    """Model::streaming_chunks (src/model.rs:343-365), geometry only."""
    hop, step, n_fft = p["hop_length"], p["mel_frames_per_step"], p["n_fft"]
    f0 = min(p["first_chunk_samples"], n)
    out = [(0, f0, 1, oracle.frame_count(f0, fe, True), p["lookahead_encoder_frames"])]
    mel_idx = step
    start = mel_idx * hop - n_fft // 2
    while start + p["samples_per_chunk"] <= n:
        out.append((start, p["samples_per_chunk"], 0, oracle.frame_count(p["samples_per_chunk"], fe, False),
                    p["lookahead_encoder_frames"]))
        mel_idx += step
        start = mel_idx * hop - n_fft // 2
    s = min(start, n)
    out.append((s, n - s, 1, oracle.frame_count(n - s, fe, True), 0))
    return out


@pytest.mark.parametrize("mode", STREAMING)
def test_streaming_chunks(cfg, mode):
    fe = synth.PROCESSOR_CONFIG["feature_extractor"]
    p = cfg.mode_params(mode)
    rng = np.random.default_rng(11)
    lengths = [0, 1, 159, 160, p["first_chunk_samples"] - 1, p["first_chunk_samples"],
               p["first_chunk_samples"] + 1, 480000, 16000 * 600 + 37] + list(rng.integers(0, 200000, 40))
    for n in lengths:
        got = [(c["start"], c["len"], c["centered"], c["num_mel_frames"], c["lookahead"])
               for c in cfg.streaming_chunks(int(n), mode)]
        assert got == _chunks_restated(p, int(n), fe), n
        assert got[0][0] == 0 and got[-1][0] + got[-1][1] == n  # the last chunk runs to the end


def _oracle_steps(om, a, mode):
    traces = []
    try:
        out = om.run_offline(a, traces) if mode == "offline" else om.run_streaming(a, mode, traces)
    except ValueError:
        return None, None
    steps = [dict(cached_frames=t["cached_frames"], window_frames=t["window_frames"],
                  valid_frames=t["valid_frames"], scored_frames=t["scored_frames"],
                  cache_frames=t["cache_embeds"].shape[0], fifo_frames=t["fifo"].shape[0],
                  cache_compressed=t["cache_compressed"]) for t in traces]
    totals = {k: out[k] for k in ("num_frames", "num_chunks", "cache_compressed", "cache_frames", "fifo_frames")}
    return steps, totals


@pytest.mark.parametrize("mode", MODES)
def test_schedule_matches_the_oracle(tiny_cfg, tiny_oracle, mode):
    """Every step's window, mask, scored frames and cache/FIFO counts, and the run's
    totals, against the oracle's traces on the 2-layer model (whose small cache and
    FIFO compress every few steps).  Too-short streaming audio fails on both."""
    for n in [0, 1, 159, 160, 161, 2720, 5160, 5161, 9000, 35_200, 54_401, 120_000, 321_123]:
        a = synth.clip(3, max(n, 1) / 16000.0, 3)[:n]
        want_steps, want_tot = _oracle_steps(tiny_oracle, a, mode)
        if want_steps is None:
            with pytest.raises(n3d.DiarizationError) as e:
                tiny_cfg.schedule(n, mode)
            assert e.value.kind == "UnsupportedAudio", n
            continue
        steps, tot = tiny_cfg.schedule(n, mode)
        assert steps == want_steps, (n, mode)
        tot.pop("num_speakers")
        assert tot == want_tot, (n, mode)


def test_every_mode_emits_the_same_frame_count_on_whole_hops(cfg):
    """README.md:76 of the reference: all four modes produce the same frame count
    (for recordings of whole 10 ms hops; a partial hop adds a frame to the streaming
    modes' last centred chunk only)."""
    rng = np.random.default_rng(12)
    for n in [16_960, 480_000, 960_000] + [int(k) * 160 for k in rng.integers(107, 40_000, 30)]:
        counts = {m: cfg.schedule(n, m)[1]["num_frames"] for m in MODES}
        assert len(set(counts.values())) == 1, (n, counts)
        assert counts["offline"] == n // 160 + 1


def test_config_errors(tmp_path, checkpoint_dir):
    with pytest.raises(n3d.DiarizationError) as e:
        n3d.Config.load(str(tmp_path / "missing"))
    assert e.value.kind == "Io"
    bad = tmp_path / "bad"
    bad.mkdir()
    for name in ("config.json", "processor_config.json"):
        with open(os.path.join(checkpoint_dir, name)) as f:
            (bad / name).write_text(f.read())
    (bad / "config.json").write_text("{not json")
    with pytest.raises(n3d.DiarizationError) as e:
        n3d.Config.load(str(bad))
    assert e.value.kind == "Json"
    c = tiny_config()
    del c["streaming_config"]["fifo_length"]
    (bad / "config.json").write_text(json.dumps(c))
    with pytest.raises(n3d.DiarizationError) as e:
        n3d.Config.load(str(bad))
    assert e.value.kind == "Json" and "fifo_length" in str(e.value)
    good = n3d.Config.load(checkpoint_dir)
    with pytest.raises(n3d.DiarizationError) as e:
        good.streaming_chunks(16000, "offline")
    assert e.value.kind == "InvalidArgument"


def test_lengths_beyond_2_31_samples_are_rejected(cfg):
    """The runs reject recordings of more than 2^31 samples (about 37 hours); the
    planners do too, instead of overflowing their frame counts."""
    n = 2**31 - 1
    steps, tot = cfg.schedule(n, "offline")
    assert tot["num_frames"] == n // 160 + 1
    for mode in ("offline", "ultra_low_latency"):
        with pytest.raises(n3d.DiarizationError) as e:
            cfg.schedule(2**31, mode)
        assert e.value.kind == "InvalidArgument"
    with pytest.raises(n3d.DiarizationError) as e:
        cfg.streaming_chunks(2**40, "low_latency")
    assert e.value.kind == "InvalidArgument"

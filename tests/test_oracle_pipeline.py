"""The oracle's end-to-end schedule and determinism (CPU only)."""

import numpy as np

import oracle
import synth


def test_config0_offline_schedule(oracle_model):
    a = synth.config0_audio()
    traces = []
    out = oracle_model.run_offline(a, traces)
    # 480000 samples -> 3000 valid mel frames (+1 zeroed) -> 376 encoder frames -> 2 windows
    assert out["num_frames"] == 3001
    assert out["num_chunks"] == 2
    assert [t["window_frames"] for t in traces] == [376, 340]
    assert [t["valid_frames"] for t in traces] == [375, 339]
    assert out["cache_compressed"] and out["cache_frames"] == 264
    assert np.isfinite(out["logits"]).all()


def test_results_do_not_depend_on_thread_count(tiny_oracle):
    a = synth.clip(7, 8.0, 3)
    oracle.lib().orc_set_threads(1)
    one = tiny_oracle.run_streaming(a, "ultra_low_latency")["logits"]
    oracle.lib().orc_set_threads(8)
    many = tiny_oracle.run_streaming(a, "ultra_low_latency")["logits"]
    assert np.array_equal(one, many)


def test_streaming_compresses_on_the_tiny_model(tiny_oracle):
    a = synth.clip(3, 10.0, 4)
    traces = []
    out = tiny_oracle.run_streaming(a, "low_latency", traces)
    assert out["cache_compressed"]
    assert any(t["cache_compressed"] for t in traces)
    # all four modes emit the same frame count as offline (README "Modes")
    off = tiny_oracle.run_offline(a)
    assert out["num_frames"] == off["num_frames"]


def test_streaming_rejects_audio_shorter_than_the_lookahead(tiny_oracle):
    import pytest

    with pytest.raises(ValueError):
        tiny_oracle.run_streaming(np.zeros(100, np.float32), "low_latency")

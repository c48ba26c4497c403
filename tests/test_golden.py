"""Committed golden fixtures (tests/golden/, made by tests/golden/make_golden.py from
the CPU oracle on seeded inputs).

CPU: the oracle still reproduces every fixture bit for bit, so neither it nor the
synthetic inputs have drifted.  GPU: the CUDA path against the fixtures, with the
gates of the reference's checkers (frame_check: per-logit maxdiff < 2e-2, zero
sigmoid>0.5 flips, identical segments; kernel probes 1e-3)."""

import os

import numpy as np
import pytest

import synth
from conftest import frame_check

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    path = os.path.join(GOLDEN, name)
    return dict(np.load(path)) if name.endswith(".npz") else np.load(path)


def _linear_inputs():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.linear_inputs()


def _run_case(model, name):
    if name == "tiny_offline_clip12.npz":
        return model.run_offline(synth.clip(12, 9.0, 3))
    return model.run_streaming(synth.clip(11, 6.0, 2), "ultra_low_latency")


# ------------------------------------------------------------------ oracle (CPU)
def test_oracle_reproduces_golden_mel(tiny_oracle):
    assert np.array_equal(tiny_oracle.log_mel(synth.clip(7, 1.0, 2), centered=True), _load("mel_clip7_1s.npy"))


@pytest.mark.parametrize("name", ["tiny_offline_clip12.npz", "tiny_ull_clip11.npz"])
def test_oracle_reproduces_golden_runs(tiny_oracle, name):
    g = _load(name)
    r = _run_case(tiny_oracle, name)
    assert np.array_equal(np.asarray(r["logits"], np.float32), g["logits"])
    assert (r["num_frames"], r["num_chunks"], r["cache_frames"], r["fifo_frames"], int(r["cache_compressed"])) == \
        (int(g["num_frames"]), int(g["num_chunks"]), int(g["cache_frames"]), int(g["fifo_frames"]),
         int(g["cache_compressed"]))


def test_oracle_reproduces_golden_linear():
    import oracle

    x, w, b, m, n, k = _linear_inputs()
    assert np.array_equal(oracle.linear(x, m, k, w, n, b).reshape(m, n), _load("linear_17x24x512.npy"))


# ------------------------------------------------------------------ CUDA path (GPU)
@pytest.mark.gpu
def test_gpu_mel_matches_golden(tiny_gpu_model):
    got = tiny_gpu_model.log_mel(synth.clip(7, 1.0, 2), centered=True)
    want = _load("mel_clip7_1s.npy")
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= 4e-6  # only the final log may differ in the last bit
    assert (got == want).mean() > 0.99


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_offline_clip12.npz", "tiny_ull_clip11.npz"])
def test_gpu_runs_match_golden(tiny_gpu_model, name):
    g = _load(name)
    got = _run_case(tiny_gpu_model, name)
    assert got.num_frames == int(g["num_frames"])
    assert (got.num_chunks, got.cache_frames, got.fifo_frames, int(got.cache_compressed)) == \
        (int(g["num_chunks"]), int(g["cache_frames"]), int(g["fifo_frames"]), int(g["cache_compressed"]))
    r = frame_check(got.logits, g["logits"].reshape(-1, 8))
    assert r["frames_equal"] and r["maxdiff"] < 2e-2 and r["flips"] == 0 and r["segments_identical"], r


@pytest.mark.gpu
def test_gpu_linear_matches_golden():
    import torch

    import n3d

    x, w, b, m, n, k = _linear_inputs()
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    dy = torch.empty(m * n, dtype=torch.float32, device="cuda")
    n3d.linear(0, dx.data_ptr(), m, k, dw.data_ptr(), n, db.data_ptr(), dy.data_ptr())
    torch.cuda.synchronize()
    assert np.abs(dy.cpu().numpy().reshape(m, n) - _load("linear_17x24x512.npy")).max() < 1e-3


def test_gate_decision_is_the_f32_sigmoid_with_libm_expf():
    """frame_check decides sigmoid(x) > 0.5 in f32 (src/bin/frame_check.rs:188-190).  The
    oracle's decision helper must be exactly 1 / (1 + expf(-x)) > 0.5 with libm's expf,
    the arithmetic of its segments: around the boundary (the smallest deciding logit is
    8.94e-8, where the f32 sigmoid stops rounding to 0.5) numpy's float32 exp rounds
    differently."""
    import ctypes

    import oracle

    libm = ctypes.CDLL("libm.so.6")
    libm.expf.argtypes = [ctypes.c_float]
    libm.expf.restype = ctypes.c_float
    xs = np.concatenate([np.linspace(-3e-7, 3e-7, 601), [0.0, -0.0, 8.94069742685133e-08, 1.0, -1.0, 40.0, -40.0]])
    xs = xs.astype(np.float32)
    want = []
    for x in xs:
        e = np.float32(libm.expf(ctypes.c_float(-x)))
        want.append(np.float32(1.0) / (np.float32(1.0) + e) > np.float32(0.5))
    got = oracle.sigmoid_above_half(xs)
    assert list(got) == want
    b = np.float32(8.94069742685133e-08)
    assert oracle.sigmoid_above_half(np.array([np.nextafter(b, np.float32(0)), b], np.float32)).tolist() == [False, True]

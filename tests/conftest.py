"""Shared pytest setup: the `gpu` marker, import paths, and the synthetic checkpoint."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nemotron3-diarization-wgpu_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA C-ABI library)")
    config.addinivalue_line("markers", "slow: long-running CPU case")


@pytest.fixture(scope="session")
def checkpoint_dir(tmp_path_factory):
    """Random-init checkpoint (seed 0) with the reference's 417 tensor names and shapes."""
    import synth

    d = tmp_path_factory.mktemp("ckpt")
    synth.write_checkpoint(str(d), seed=0)
    return str(d)


@pytest.fixture(scope="session")
def oracle_model(checkpoint_dir):
    import oracle

    return oracle.OracleModel.load(checkpoint_dir)


def tiny_config():
    """A 2-layer variant with a 32-frame speaker cache: same kernels and shapes per
    layer, but small enough that the CPU oracle runs long streaming sessions in
    seconds and the cache compresses every few steps."""
    import copy

    import synth

    cfg = copy.deepcopy(synth.MODEL_CONFIG)
    cfg["audio_config"]["num_hidden_layers"] = 2
    cfg["streaming_config"].update(fifo_length=10, speaker_cache_length=32, speaker_cache_update_period=4)
    cfg.update(chunk_length=24, chunk_right_context=4, fifo_length=6, speaker_cache_update_period=10)
    return cfg


@pytest.fixture(scope="session")
def tiny_checkpoint_dir(tmp_path_factory):
    import synth

    d = tmp_path_factory.mktemp("tiny")
    synth.write_checkpoint(str(d), seed=0, cfg=tiny_config())
    return str(d)


@pytest.fixture(scope="session")
def tiny_oracle(tiny_checkpoint_dir):
    import oracle

    return oracle.OracleModel.load(tiny_checkpoint_dir)


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_model(checkpoint_dir):
    import n3d

    return n3d.Model.load_gpu(checkpoint_dir, 0)


@pytest.fixture(scope="session")
def tiny_gpu_model(tiny_checkpoint_dir):
    import n3d

    return n3d.Model.load_gpu(tiny_checkpoint_dir, 0)


def frame_check(got, want, ns=8, duration=0.01):
    """The reference's three parity gates (src/bin/frame_check.rs:170-240):
    per-logit maxdiff < 2e-2, zero sigmoid>0.5 flips, IDENTICAL segments.
    Returns a dict of the measured quantities; callers assert on it."""
    import numpy as np

    import oracle

    got = np.asarray(got, np.float32).reshape(-1, ns)
    want = np.asarray(want, np.float32).reshape(-1, ns)
    res = {"frames_equal": got.shape == want.shape}
    if not res["frames_equal"]:
        return res
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    res["maxdiff"] = float(d.max()) if d.size else 0.0
    # the decision sigmoid(x) > 0.5 in f32, as the gate computes it
    # (src/bin/frame_check.rs:188-190), with the oracle's libm expf -- the arithmetic its
    # segments use.  In f32 a logit below about 1.2e-7 gives exactly 0.5, not a decision.
    dg = oracle.sigmoid_above_half(got).reshape(got.shape)
    dw = oracle.sigmoid_above_half(want).reshape(want.shape)
    flips = np.argwhere(dg != dw)
    res["flips"] = int(len(flips))
    res["flip_ref_abs_max"] = float(np.abs(want[flips[:, 0], flips[:, 1]]).max()) if len(flips) else 0.0
    # each flip as (row, speaker, reference logit, our logit), for the failure message
    res["flip_values"] = [(int(r), int(c), float(want[r, c]), float(got[r, c])) for r, c in flips[:8]]
    a = oracle.extract_speaker_dict(got.ravel(), got.shape[0], ns, duration)
    b = oracle.extract_speaker_dict(want.ravel(), want.shape[0], ns, duration)
    res["segments_identical"] = a == b
    res["segments"] = len(b)
    return res

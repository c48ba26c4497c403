"""The C-ABI library on the CPU: it loads, exports every symbol include/n3d.h
declares, fails loudly without a B200, and its host-only functions
(extract_speaker_dict, activity_stats) match the oracle exactly.  A plain C99 program
(tests/c_consumer.c) compiles against the header, links the library and gets the same
answers as the Python binding."""

import ctypes as C
import os

import numpy as np
import pytest

import n3d
import oracle
from conftest import gpu_available

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_symbol():
    L = n3d.lib()
    names = n3d.header_functions()
    assert len(names) >= 24
    missing = [n for n in names if not hasattr(L, n)]
    assert missing == []


def test_version_string():
    assert b"sm_100a" in n3d.lib().n3d_version()


@pytest.mark.skipif(gpu_available(), reason="checks the no-device path")
def test_load_without_a_gpu_fails_loudly(checkpoint_dir):
    with pytest.raises(n3d.DiarizationError) as e:
        n3d.Model.load_gpu(checkpoint_dir, 0)
    assert e.value.kind in ("NoDevice", "Cuda")


def test_null_arguments_are_rejected():
    out = n3d._RunOutput()
    st = n3d.lib().n3d_run_offline(None, None, 0, C.byref(out))
    assert n3d.STATUS[st] == "InvalidArgument"
    assert b"null" in n3d.lib().n3d_last_error()
    h = C.c_void_p()
    st = n3d.lib().n3d_session_open(None, 2, C.byref(h))
    assert n3d.STATUS[st] == "InvalidArgument" and not h.value
    st = n3d.lib().n3d_session_push(None, None, 0, C.byref(out))
    assert n3d.STATUS[st] == "InvalidArgument"
    n3d.lib().n3d_session_free(None)  # freeing nothing is a no-op


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_extract_speaker_dict_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    T, ns = 3000, 8
    # many logits near zero, as random-init weights produce
    logits = (rng.standard_normal(T * ns) * 0.006).astype(np.float32)
    mask = (rng.random(T) > 0.1).astype(np.uint8) if seed == 2 else None
    got = n3d.extract_speaker_dict(logits, T, ns, 0.01, mask, 0.5)
    want = oracle.extract_speaker_dict(logits, T, ns, 0.01, mask, 0.5)
    assert [(s.start, s.end, s.speaker) for s in got] == [(np.float32(a), np.float32(b), s) for a, b, s in want]


def test_extract_speaker_dict_reference_cases():  # src/segments.rs:153-205
    logit = lambda a: 2.0 if a else -2.0
    acts = [[0, 0, 1, 1, 0, 0], [0, 1, 0, 0, 1, 1]]
    logits = [logit(acts[s][t]) for t in range(6) for s in range(2)]
    segs = n3d.extract_speaker_dict(logits, 6, 2, 0.01)
    f = np.float32
    assert [(s.start, s.end, s.speaker) for s in segs] == [(f(0.01), f(0.02), 1), (f(0.02), f(0.04), 0),
                                                          (f(0.04), f(0.06), 1)]
    segs = n3d.extract_speaker_dict([logit(t % 2 == 0) for t in range(6)], 6, 1, 0.01, [0, 1, 1, 1, 1, 0])
    assert [(s.start, s.end) for s in segs] == [(f(0.02), f(0.03)), (f(0.04), f(0.05))]
    assert n3d.extract_speaker_dict([], 0, 8, 0.01) == []


def test_activity_stats_matches_oracle():
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal(800) * 0.01).astype(np.float32)
    assert n3d.activity_stats(logits, 100, 8) == oracle.activity_stats(logits, 100, 8)
    assert n3d.frame_duration(160, 16000) == np.float32(0.01)


def test_activity_stats_counts_are_optional():
    rng = np.random.default_rng(6)
    logits = rng.standard_normal(800).astype(np.float32)
    lg = logits.ctypes.data_as(C.POINTER(C.c_float))
    counts = (C.c_size_t * 8)()
    with_counts = n3d.lib().n3d_activity_stats(lg, 100, 8, None, 0.5, counts)
    without = n3d.lib().n3d_activity_stats(lg, 100, 8, None, 0.5, None)
    assert with_counts == without > 0
    sig = 1.0 / (1.0 + np.exp(-logits.reshape(100, 8).astype(np.float64)))
    assert list(counts) == list((sig > 0.5).sum(axis=0))


def test_describe_of_no_model_is_null():
    assert n3d.lib().n3d_model_describe(None) is None


def _segment_case(draw):
    from hypothesis import strategies as st

    T = draw(st.integers(0, 300))
    ns = draw(st.integers(1, 8))
    thr = draw(st.sampled_from([0.1, 0.25, 0.5, 0.5000001, 0.9]))
    edge = float(np.log(thr / (1.0 - thr)))  # the logit whose sigmoid sits on the threshold
    vals = st.sampled_from([0.0, -0.0, 1e-7, -1e-7, 3.0, -3.0, 40.0, -40.0, edge, np.nextafter(edge, 9.0),
                            np.nextafter(edge, -9.0), np.inf, -np.inf, np.nan]) | st.floats(-8, 8, width=32)
    logits = np.array(draw(st.lists(vals, min_size=T * ns, max_size=T * ns)), np.float32)
    mask = draw(st.none() | st.lists(st.booleans(), min_size=T, max_size=T))
    mask = None if mask is None else np.array(mask, np.uint8)
    dur = draw(st.sampled_from([0.01, 0.08, 0.02, 0.0133]))
    return logits, T, ns, dur, mask, thr


def test_segments_and_activity_match_the_oracle_on_random_cases():
    """extract_speaker_dict and activity_stats (src/segments.rs:70-141) on drawn logits
    (non-finite ones included), masks, thresholds and frame durations: the C ABI equals
    the oracle exactly."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=150, deadline=None, derandomize=True, database=None)
    @given(st.data())
    def check(data):
        logits, T, ns, dur, mask, thr = _segment_case(data.draw)
        got = n3d.extract_speaker_dict(logits, T, ns, dur, mask, thr)
        want = oracle.extract_speaker_dict(logits, T, ns, dur, mask, thr)
        assert [(s.start, s.end, s.speaker) for s in got] == [(np.float32(a), np.float32(b), s) for a, b, s in want]
        assert n3d.activity_stats(logits, T, ns, mask, thr) == oracle.activity_stats(logits, T, ns, mask, thr)

    check()


def test_plain_c_caller(tmp_path, checkpoint_dir):
    """include/n3d.h compiles as C99 (pedantic) and links against libn3d.so; a C program
    gets the same answers through it as the Python binding does."""
    import subprocess

    src = os.path.join(ROOT, "tests", "c_consumer.c")
    exe = tmp_path / "c_consumer"
    lib_dir = os.path.dirname(n3d.LIB_PATH)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(ROOT, "include"),
                        src, "-o", str(exe), "-L", lib_dir, "-ln3d", "-Wl,-rpath," + lib_dir],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    args = [str(exe), checkpoint_dir] + ([] if gpu_available() else ["load"])
    r = subprocess.run(args, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    out = r.stdout.splitlines()
    assert out[0] == "version " + n3d.lib().n3d_version().decode()
    assert out[1] == "frame_duration 0.00999999978"
    cfg = n3d.Config.load(checkpoint_dir)
    p = cfg.mode_params("ultra_low_latency")
    assert out[2] == (f"ultra first_chunk_samples {p['first_chunk_samples']} samples_per_chunk "
                      f"{p['samples_per_chunk']} latency_ms {p['latency_ms']}")
    steps, tot = cfg.schedule(480000, "offline")
    assert out[3] == (f"offline steps {len(steps)} frames {tot['num_frames']} chunks {tot['num_chunks']}" +
                      "".join(f" [{s['window_frames']} {s['valid_frames']} {s['scored_frames']}]" for s in steps))
    assert out[4].startswith("short streaming audio: unsupported audio")
    segs = n3d.extract_speaker_dict(_segment_logits(), 6, 2, 0.01)
    assert out[5:5 + len(segs)] == [f"segment {s.start:.2f} {s.end:.2f} {s.speaker}" for s in segs]
    if not gpu_available():
        assert out[-1] == "load status 12"  # N3D_ERR_NO_DEVICE


def _segment_logits():
    """The C helper's logits: [6 frames, 2 speakers], speaker 0 in frames 1-2, speaker 1 in frame 3."""
    lg = np.full(12, -4.0, np.float32)
    lg[[2, 4, 7]] = 4.0
    return lg


def test_stage_arguments_are_range_checked_before_any_model_use():
    """Out-of-range sizes are rejected before the model is touched (the handle below is
    a placeholder that is never dereferenced): at most 1024 groups per embed_range call,
    as the reference's MAX_SEQ, and no size that would wrap the library's int counts."""
    fake = C.c_void_p(64)
    buf = np.zeros(16, np.float32)
    p = buf.ctypes.data_as(C.POINTER(C.c_float))
    cases = [lambda: n3d.lib().n3d_embed_range(fake, p, 100, 0, 1025, p),
             lambda: n3d.lib().n3d_embed_range(fake, p, 2**31, 0, 4, p),
             lambda: n3d.lib().n3d_embed_range(fake, p, 100, 2**40, 2**40 + 1, p),
             lambda: n3d.lib().n3d_forward_embeds(fake, p, 2**32 + 5, 3, p),
             lambda: n3d.lib().n3d_head_forward(fake, p, 2**32, p),
             lambda: n3d.lib().n3d_forward_window(fake, p, 2**33, 1, p)]
    for call in cases:
        assert n3d.STATUS[call()] == "InvalidArgument"
        assert b"2^31" in n3d.lib().n3d_last_error() or b"1024 groups" in n3d.lib().n3d_last_error()


def test_single_kernel_sizes_are_checked_before_any_cuda_call():
    """n3d_linear, n3d_layer_norm and n3d_attention reject sizes that would wrap the
    kernels' int counts or grid limits before they touch a device (the device pointers
    below are placeholders that are never used)."""
    d = C.c_void_p(256)
    lib = n3d.lib()
    cases = [lambda: lib.n3d_linear(0, d, 2**31, 32, d, 8, None, d),
             lambda: lib.n3d_linear(0, d, 8, 32, d, 2**32, None, d),
             lambda: lib.n3d_layer_norm(0, d, 8, 768, d, d, d),
             lambda: lib.n3d_layer_norm(0, d, 2**31, 512, d, d, d),
             lambda: lib.n3d_attention(0, d, d, d, 2**31, 8, 64, 8, 1, 10000.0, d),
             lambda: lib.n3d_attention(0, d, d, d, 64, 0, 64, 8, 1, 10000.0, d),
             lambda: lib.n3d_attention(0, d, d, d, 64, 70000, 64, 8, 1, 10000.0, d),
             # sizes whose products wrap a 64-bit count must not slip past the scratch check
             lambda: lib.n3d_linear_noalloc(0, d, 32, 2**59, d, 32, None, d, None),
             lambda: lib.n3d_linear_noalloc(0, d, 2**32, 2**32, d, 2**32, None, d, None),
             lambda: lib.n3d_linear_noalloc(0, d, 2**31, 32, d, 8, None, d, None),
             lambda: lib.n3d_linear_noalloc(0, d, 8, 32, d, 2**32, None, d, None),
             lambda: lib.n3d_linear_noalloc(0, d, 4096, 1024, d, 1024, None, d, None)]
    for call in cases:
        assert n3d.STATUS[call()] == "InvalidArgument", lib.n3d_last_error()


def test_wait_selftest_limit_is_checked_before_any_cuda_call():
    w = C.c_double()
    for limit in (0.0, -1.0, 2001.0, float("nan")):
        assert n3d.STATUS[n3d.lib().n3d_selftest_wait_timeout(0, limit, C.byref(w))] == "InvalidArgument"


def test_cache_compress_arguments_are_checked_before_any_cuda_call():
    probs = np.full(64 * 8, 0.75, np.float32)
    picked = (C.c_size_t * 64)()
    sentinel, count = C.c_size_t(), C.c_size_t()

    def call(frames=64, **kw):
        cfg = n3d.CacheConfig(speaker_cache_length=32, num_silence_frames=1, score_threshold=0.25,
                              num_speakers=8, subsampling_factor=8, num_strong_boosted_frames=2,
                              num_weak_boosted_frames=4)
        for k, v in kw.items():
            setattr(cfg, k, v)
        return n3d.lib().n3d_cache_compress(0, C.byref(cfg), probs.ctypes.data_as(C.POINTER(C.c_float)), frames,
                                            None, 0, None, picked, C.byref(sentinel), C.byref(count), None, None)

    for st in [call(frames=0), call(num_speakers=0), call(num_speakers=17), call(frames=2**40),
               call(speaker_cache_length=2**40), call(frames=60000)]:
        assert n3d.STATUS[st] == "InvalidArgument", n3d.lib().n3d_last_error()

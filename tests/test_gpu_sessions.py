"""Streaming sessions (n3d_session_* / n3d_sessions_push) on a B200.

The reference streams only through `Model::run_streaming` on a whole recording
(src/model.rs:313-365).  A session must give exactly that call's logits when the
same audio arrives in pieces, emitting each chunk's rows once the chunk's samples
are complete, with the final centred chunk at close; the RunOutput totals at close
are run_streaming's.  Checked on the tiny 2-layer model in every streaming mode,
against run_streaming (same kernels: < 1e-6) and against the CPU oracle
(frame_check gates).
"""

import numpy as np
import pytest

import n3d
import synth
from conftest import frame_check

pytestmark = pytest.mark.gpu

MODES = ["low_latency", "very_low_latency", "ultra_low_latency"]


def _gates_ok(r):
    return r["maxdiff"] < 2e-2 and r["flips"] == 0 and r["segments_identical"]


def _pieces(a, rng, max_piece):
    out, i = [], 0
    while i < a.size:
        k = int(rng.integers(1, max_piece))
        out.append(a[i:i + k])
        i += k
    return out


@pytest.mark.parametrize("mode", MODES)
def test_session_in_pieces_equals_run_streaming(tiny_gpu_model, tiny_oracle, mode):
    a = synth.clip(11, 12.0, 4, overlap=0.3)
    want = tiny_gpu_model.run_streaming(a, mode)
    ss = tiny_gpu_model.open_session(mode)
    rows = []
    for p in _pieces(a, np.random.default_rng(5), 9000):  # random piece sizes, up to 0.56 s
        rows.append(ss.push(p).logits)
    last = ss.close()
    rows.append(last.logits)
    ss.free()
    got = np.concatenate(rows)
    assert got.shape == want.logits.shape
    assert np.abs(got - want.logits).max() < 1e-6
    assert (last.num_chunks, last.cache_compressed, last.cache_frames, last.fifo_frames) == \
        (want.num_chunks, want.cache_compressed, want.cache_frames, want.fifo_frames)
    r = frame_check(got, tiny_oracle.run_streaming(a, mode)["logits"])
    assert _gates_ok(r), r


def test_rows_arrive_before_close(tiny_gpu_model):
    a = synth.clip(12, 6.0, 3)
    want = tiny_gpu_model.run_streaming(a, "ultra_low_latency")
    ss = tiny_gpu_model.open_session("ultra_low_latency")
    first = ss.push(a[:8000])  # half a second: chunk 0 (4 encoder frames = 0.32 s + window) is complete
    assert first.num_chunks == 1 and first.num_frames > 0
    rest = ss.push(a[8000:])   # every later full chunk runs now
    assert rest.num_chunks == want.num_chunks - 1
    end = ss.close()           # the final centred chunk
    assert end.num_chunks == want.num_chunks
    assert first.num_frames + rest.num_frames + end.num_frames == want.num_frames
    ss.free()


def test_batched_sessions_equal_single_runs(tiny_gpu_model):
    clips = [synth.clip(30 + i, d, 3) for i, d in enumerate([5.0, 8.0, 3.5])]
    want = [tiny_gpu_model.run_streaming(c, "very_low_latency") for c in clips]
    ss = [tiny_gpu_model.open_session("very_low_latency") for _ in clips]
    rows = [[] for _ in clips]
    step = 4000  # 250 ms per push, like a live feed; shorter sessions get empty pieces at the end
    for t in range(0, max(c.size for c in clips), step):
        for r, o in zip(rows, tiny_gpu_model.sessions_push(ss, [c[t:t + step] for c in clips])):
            r.append(o.logits)
    ends = tiny_gpu_model.sessions_push(ss, [np.zeros(0, np.float32)] * len(clips), close=True)
    for r, o, w in zip(rows, ends, want):
        r.append(o.logits)
        got = np.concatenate(r)
        assert got.shape == w.logits.shape
        assert np.abs(got - w.logits).max() < 1e-6
        assert o.num_chunks == w.num_chunks
    for s in ss:
        s.free()


def test_too_short_session_is_unsupported_audio_then_unusable(tiny_gpu_model):
    ss = tiny_gpu_model.open_session("low_latency")
    assert ss.push(np.zeros(100, np.float32)).num_frames == 0  # nothing is complete yet
    with pytest.raises(n3d.DiarizationError) as e:
        ss.close()
    assert e.value.kind == "UnsupportedAudio"  # as run_streaming on the same 100 samples
    with pytest.raises(n3d.DiarizationError) as e:
        ss.push(np.zeros(10, np.float32))
    assert e.value.kind == "InvalidArgument"
    ss.free()


def test_push_after_close_is_rejected(tiny_gpu_model):
    ss = tiny_gpu_model.open_session("ultra_low_latency")
    ss.push(synth.clip(14, 2.0, 2))
    ss.close()
    with pytest.raises(n3d.DiarizationError) as e:
        ss.push(np.zeros(160, np.float32))
    assert e.value.kind == "InvalidArgument"
    ss.free()


def test_offline_is_not_a_session_mode(tiny_gpu_model):
    with pytest.raises(n3d.DiarizationError) as e:
        tiny_gpu_model.open_session("offline")
    assert e.value.kind == "InvalidArgument"

"""The reference's own known-answer tests, run against the CPU oracle.

Each test restates one `#[test]` of the reference crate with the same inputs
and the same expected values, so the oracle is pinned to the reference's
published behaviour before it is trusted as the parity checker:
src/tensor.rs:151-201, src/mel.rs:253-329, src/streaming.rs:506-610,
src/segments.rs:153-221.
"""

import math

import numpy as np
import pytest

import oracle as O

FE = {"feature_size": 128, "n_fft": 512, "hop_length": 160, "win_length": 400, "sampling_rate": 16000,
      "preemphasis": 0.97}


# ------------------------------------------------------------- src/tensor.rs

def test_matmul_matches_hand_computation():  # src/tensor.rs:151-158
    c = O.matmul([1, 2, 3, 4, 5, 6], 2, 3, [1, 0, 0, 1, 0, 0], 2)
    assert c.tolist() == [1.0, 2.0, 4.0, 5.0]


def test_linear_matches_hand_computation():  # src/tensor.rs:160-168
    y = O.linear([1, 2, 3, 4, 5, 6], 2, 3, [1, 0, 0, 0, 1, 0], 2)
    assert y[0:2].tolist() == [1.0, 2.0]
    assert y[2:4].tolist() == [4.0, 5.0]


def test_layer_norm_normalises():  # src/tensor.rs:170-180
    y = O.layer_norm([1, 2, 3, 4], 1, 4, [1, 1, 1, 1], [0, 0, 0, 0])
    assert abs(np.float32(y.sum()) / 4) < 1e-5
    assert abs(np.float32((y * y).sum()) / 4 - 1.0) < 1e-3


def test_gelu_matches_known_values():  # src/tensor.rs:182-192
    g = O.gelu([0.0, 1.0, -1.0])
    assert abs(g[0]) < 1e-6
    assert abs(g[1] - 0.8413447) < 1e-6
    assert abs(g[2] + 0.1586553) < 1e-6


def test_softmax_sums_to_one_and_is_stable():  # src/tensor.rs:194-201
    x = O.softmax_last([1000.0, 1000.0, 1000.0, -1e30], 1, 4)
    assert abs(float(x.sum()) - 1.0) < 1e-5
    assert x[3] < 1e-6


# ---------------------------------------------------------------- src/mel.rs

def test_log_guard_is_the_expected_floor():  # src/mel.rs:255-262
    assert abs(math.log(np.float32(5.9604645e-8)) - (-16.635532)) < 1e-4


def test_periodic_false_hann_is_symmetric_and_zero_at_both_ends():  # src/mel.rs:264-281
    w = O.hann_periodic_false(400)
    assert abs(w[0]) < 1e-6
    assert abs(w[399]) < 1e-6
    for i in range(200):
        assert abs(w[i] - w[399 - i]) < 1e-6
    assert 0.999 < w[199] < 1.001


def test_mel_filterbank_shape_and_coverage():  # src/mel.rs:283-306
    f = O.slaney_mel_filterbank(128, 512, 16000, 0.0, 8000.0)
    assert f.size == 128 * 257
    f = f.reshape(128, 257)
    assert all((f[m] > 0).any() for m in range(128))
    top = f[127]
    assert 244 <= int(np.argmax(top)) <= 256
    assert abs(top[256]) < 1e-12
    assert f[0, 1] > 0.0


def test_frame_counts_match_the_processor():  # src/mel.rs:308-317
    assert O.frame_count(16_680, FE, True) == 104
    assert O.frame_count(17_040, FE, False) == 104
    assert O.frame_count(16_000, FE, True) == 100


def test_features_are_finite_and_bounded_below():  # src/mel.rs:319-330
    filters = O.slaney_mel_filterbank(128, 512, 16000, 0.0, 8000.0)
    samples = (np.sin(np.arange(16_000, dtype=np.float32) * np.float32(0.01)) * np.float32(0.1)).astype(np.float32)
    f = O.log_mel(samples, FE, True, filters)
    assert f.size == 100 * 128
    assert np.isfinite(f).all()
    assert (f >= math.log(np.float32(5.9604645e-8)) - 1e-3).all()


# ---------------------------------------------------------- src/streaming.rs

def _cfg(**kw):  # src/streaming.rs:489-503
    base = dict(fifo_length=4, speaker_cache_length=8, update_period=3, num_silence_frames=1, score_threshold=0.25,
                latest_frames_score_boost=0.05, num_speakers=2, subsampling_factor=2, min_positive_scores=1,
                num_strong_boosted_frames=2, num_weak_boosted_frames=4)
    base.update(kw)
    return O.cache_cfg(**base)


def test_pool_probs_truncates_and_masks_per_group():  # src/streaming.rs:505-527
    c = _cfg()
    logits = [10.0 if (i // 2) % 2 == 0 else -10.0 for i in range(2 * 5 * 2)]
    mask = [1, 1, 0, 1, 1]
    p = O.pool_probs(c, logits, 10, mask)
    assert p.size == 5 * 2
    hi = np.float32(1) / (np.float32(1) + np.exp(np.float32(-10.0)))
    lo = np.float32(1) / (np.float32(1) + np.exp(np.float32(10.0)))
    assert abs(p[0] - (hi + lo) / 2) < 1e-6
    assert p[4] == 0.0 and p[5] == 0.0
    assert O.pool_probs(c, logits, 9, mask).size == 4 * 2


def test_num_popped_follows_the_reference_rule():  # src/streaming.rs:529-538
    c = _cfg()
    assert O.num_popped(c, 4) == 0
    assert O.num_popped(c, 5) == 3
    assert O.num_popped(c, 20) == 16
    assert O.num_popped(c, 2) == 0


def test_compress_keeps_one_silence_slot_per_speaker():  # src/streaming.rs:540-568
    c = _cfg()
    ns, hidden, nf = 2, 2, 9
    embeds = np.arange(nf * hidden, dtype=np.float32)
    probs = np.zeros(nf * ns, np.float32)
    for f in range(nf):
        probs[f * ns] = 0.9 if f < 5 else 0.01
        probs[f * ns + 1] = 0.01 if f < 5 else 0.9
    e, p = O.compress(c, hidden, embeds, probs, nf, [7.0, 8.0])
    assert e.size == 8 * hidden and p.size == 8 * ns
    sil = [i for i in range(8) if e[i * hidden] == 7.0 and e[i * hidden + 1] == 8.0]
    assert len(sil) == 2
    for i in sil:
        assert p[i * ns:(i + 1) * ns].tolist() == [0.0, 0.0]
    kept = [i for i in range(8) if i not in sil]
    assert all(b > a for a, b in zip(kept, kept[1:]))


def test_boost_top_is_per_speaker():  # src/streaming.rs:570-587
    c = _cfg(num_strong_boosted_frames=1, num_weak_boosted_frames=0)
    scores = np.zeros(8, np.float32)
    for f in range(4):
        scores[f * 2] = [10.0, 1.0, 2.0, 3.0][f]
        scores[f * 2 + 1] = [0.0, 0.0, 0.0, 9.0][f]
    s = O.boost_top(c, scores, 4, 1, 1.0)
    assert s[0] == 11.0
    assert s[7] == 10.0
    assert s[1] == 0.0


def test_frame_scores_uses_neg_log_half():  # src/streaming.rs:589-610
    c = _cfg(min_positive_scores=2, score_threshold=0.01)
    probs = np.full(8, 0.01, np.float32)
    for f in range(3):
        probs[f * 2] = 0.95
    s = O.frame_scores(c, probs, 4)
    assert s[0] > 0.0
    lp = math.log(np.float32(0.95))
    lc0 = math.log(np.float32(1.0) - np.float32(0.95))
    lc1 = math.log(max(np.float32(1.0) - np.float32(0.01), 0.01))
    want = lp - lc0 + (lc0 + lc1) + math.log(2)
    assert abs(s[0] - want) < 1e-5
    assert math.isinf(s[1]) and s[1] < 0


# ----------------------------------------------------------- src/segments.rs

def _logit(active):
    return 2.0 if active else -2.0


def test_runs_become_segments_in_arrival_order():  # src/segments.rs:153-174
    acts = [[0, 0, 1, 1, 0, 0], [0, 1, 0, 0, 1, 1]]
    logits = [_logit(acts[s][t]) for t in range(6) for s in range(2)]
    segs = O.extract_speaker_dict(logits, 6, 2, 0.01, None, 0.5)
    want = [(0.01, 0.02, 1), (0.02, 0.04, 0), (0.04, 0.06, 1)]
    assert [(round(a, 6), round(b, 6), s) for a, b, s in segs] == \
        [(float(np.float32(a)).__round__(6), float(np.float32(b)).__round__(6), s) for a, b, s in want]
    assert [(np.float32(a), np.float32(b), s) for a, b, s in segs] == \
        [(np.float32(a), np.float32(b), s) for a, b, s in want]


def test_a_run_open_at_the_end_is_still_closed():  # src/segments.rs:176-184
    logits = [_logit(False), _logit(False), _logit(True), _logit(False)]
    segs = O.extract_speaker_dict(logits, 2, 2, 0.01, None, 0.5)
    assert [(np.float32(a), np.float32(b), s) for a, b, s in segs] == [(np.float32(0.01), np.float32(0.02), 0)]


def test_the_mask_removes_frames_from_both_sides():  # src/segments.rs:186-205
    logits = [_logit(t % 2 == 0) for t in range(6)]
    segs = O.extract_speaker_dict(logits, 6, 1, 0.01, [0, 1, 1, 1, 1, 0], 0.5)
    assert [(np.float32(a), np.float32(b), s) for a, b, s in segs] == \
        [(np.float32(0.02), np.float32(0.03), 0), (np.float32(0.04), np.float32(0.05), 0)]


def test_round2_matches_pythons_half_to_even():  # src/segments.rs:207-213
    assert O.round2(0.125) == np.float32(0.12)
    assert O.round2(0.135) == np.float32(0.14)
    assert O.round2(1.005) == np.float32(1.0)
    assert O.round2(28.1) == np.float32(28.1)


def test_stats_count_frames_not_segments():  # src/segments.rs:215-221
    logits = [v for t in range(4) for v in (_logit(t < 2), _logit(t == 3))]
    pct, per = O.activity_stats(logits, 4, 2, None, 0.5)
    assert per == [2, 1]
    assert pct == 75.0

"""The oracle's speaker-cache compression against an independent numpy restatement of
the reference's code (src/streaming.rs:294-482), on random inputs full of ties.

The reference's own known-answer tests pin the oracle on a few hand cases.  Here every
stage is restated and checked on thousands of frames:
* frame_scores: the log-odds score, the -inf mask for frames at or below 0.5, and the
  per-speaker "enough positives" rule.  Values are compared to within a few ulps,
  because numpy's float32 log need not round like libm's logf; the -inf pattern must
  be identical;
* the ranking, from the oracle's own scores:
  * the latest-frames boost, then the strong and weak per-speaker top-k boosts (stable
    descending sorts);
  * the flat speaker-major layout with +inf silence slots and a stable descending sort
    truncated to the cache length;
  * the -inf -> sentinel remap and the final index sort.
  The picks must equal the oracle's bit for bit;
* the gather of embeddings and probabilities (silence rows with zero probabilities),
  bit for bit.
This is integer and index work on fp32 keys, so the bar is exact."""

import numpy as np
import pytest

import oracle

F32 = np.float32
LN2 = F32(np.log(2.0))


def _cfg(cache_len, ns, n_sil, thr, latest, min_pos, k_strong, k_weak):
    return oracle.cache_cfg(fifo_length=0, speaker_cache_length=cache_len, update_period=0, num_silence_frames=n_sil,
                            score_threshold=thr, latest_frames_score_boost=latest, num_speakers=ns,
                            subsampling_factor=8, min_positive_scores=min_pos, num_strong_boosted_frames=k_strong,
                            num_weak_boosted_frames=k_weak)


def _frame_scores(cc, probs, nf):
    ns = cc.num_speakers
    p = probs.reshape(nf, ns)
    thr = F32(cc.score_threshold)
    lp = np.log(np.maximum(p, thr).astype(np.float64)).astype(F32)
    lc = np.log(np.maximum((F32(1.0) - p).astype(F32), thr).astype(np.float64)).astype(F32)
    s = np.zeros(nf, F32)
    for j in range(ns):  # sequential fp32 sum, as iter().sum()
        s = (s + lc[:, j]).astype(F32)
    v = ((((lp - lc).astype(F32) + s[:, None]).astype(F32)) + LN2).astype(F32)
    scores = np.where(p > 0.5, v, F32(-np.inf)).astype(F32)
    pos = (scores > 0).sum(axis=0)
    for j in range(ns):
        if pos[j] >= cc.min_positive_scores:
            kill = (scores[:, j] <= 0) & (p[:, j] > 0.5)
            scores[kill, j] = F32(-np.inf)
    return scores


def _boost_top(scores, k, boost):
    out = scores.copy()
    nf, ns = out.shape
    for j in range(ns):
        order = sorted(range(nf), key=lambda i: -float(out[i, j]))  # stable, descending
        for i in order[:min(k, nf)]:
            out[i, j] = F32(out[i, j] + boost)
    return out


def _picked(cc, scores):
    nf, ns = scores.shape
    sc = scores.copy()
    sc[cc.speaker_cache_length:] = (sc[cc.speaker_cache_length:] + F32(cc.latest_frames_score_boost)).astype(F32)
    sc = _boost_top(sc, cc.num_strong_boosted_frames, F32(2.0) * LN2)
    sc = _boost_top(sc, cc.num_weak_boosted_frames, LN2)
    n_scored = nf + cc.num_silence_frames
    flat = np.full(ns * n_scored, F32(np.inf), F32)
    for j in range(ns):
        flat[j * n_scored:j * n_scored + nf] = sc[:, j]
    sentinel = n_scored * ns
    order = sorted(range(flat.size), key=lambda i: -float(flat[i]))[:cc.speaker_cache_length]
    picked = sorted(sentinel if flat[i] == -np.inf else i for i in order)
    return np.array(picked, np.int64), sentinel, n_scored


def _probs(rng, nf, ns, ties):
    if ties == "rows":  # a few prototype rows repeated: exact ties in every speaker's ranking
        proto = (rng.integers(0, 17, (5, ns)) / 16.0).astype(F32)
        return proto[rng.integers(0, 5, nf)].reshape(-1)
    if ties:  # quantised probabilities
        return (rng.integers(0, 17, (nf, ns)) / 16.0).astype(F32).reshape(-1)
    return rng.random((nf, ns)).astype(F32).reshape(-1)


CASES = [  # cache_len, ns, n_sil, thr, latest, min_pos, k_strong, k_weak, frames
    (264, 8, 1, 0.25, 0.05, 25, 24, 49, 564),
    (264, 8, 1, 0.25, 0.05, 25, 24, 49, 300),
    (32, 8, 1, 0.25, 0.05, 1, 2, 4, 42),
    (32, 4, 2, 0.1, 0.5, 3, 1, 6, 40),
    (16, 2, 0, 0.3, 0.0, 0, 3, 3, 16),
    (64, 8, 3, 0.25, 0.05, 200, 0, 0, 70),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("ties", [False, True, "rows"])
def test_compression_matches_a_restatement(case, ties):
    cache_len, ns, n_sil, thr, latest, min_pos, ks, kw, nf = CASES[case]
    cc = _cfg(cache_len, ns, n_sil, thr, latest, min_pos, ks, kw)
    rng = np.random.default_rng(case * 3 + [False, True, "rows"].index(ties))
    for _ in range(5):
        probs = _probs(rng, nf, ns, ties)
        # stage 1: scores
        got = oracle.frame_scores(cc, probs, nf).reshape(nf, ns)
        want = _frame_scores(cc, probs, nf)
        assert np.array_equal(np.isneginf(got), np.isneginf(want))
        fin = np.isfinite(want)
        assert np.allclose(got[fin], want[fin], rtol=0, atol=4e-6)
        # stage 2: ranking from the oracle's scores, exact
        picked, sentinel = oracle.compress_picked(cc, probs, nf)
        mine, my_sentinel, n_scored = _picked(cc, got)
        assert sentinel == my_sentinel
        assert np.array_equal(picked, mine)
        # stage 3: gather, exact
        hidden = 16
        embeds = rng.standard_normal((nf, hidden)).astype(F32)
        silence = rng.standard_normal(hidden).astype(F32)
        oe, op = oracle.compress(cc, hidden, embeds.reshape(-1), probs, nf, silence)
        frames = [nf if i == sentinel else min(i % n_scored, nf) for i in mine]
        we = np.stack([silence if f == nf else embeds[f] for f in frames])
        wp = np.stack([np.zeros(ns, F32) if f == nf else probs.reshape(nf, ns)[f] for f in frames])
        assert np.array_equal(oe.reshape(cache_len, hidden), we)
        assert np.array_equal(op.reshape(cache_len, ns), wp)

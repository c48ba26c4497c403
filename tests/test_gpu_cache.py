"""The device speaker-cache ranking against the oracle, bit for bit.

The chunk loop's cache kernel ranks compression candidates by radix selection
with index tie-breaks (csrc/cache.cu), where the reference sorts stably
(SpeakerCache::compress, src/streaming.rs:410-482).  A swapped pick moves a frame
in or out of the cache and still gives plausible logits, so end-to-end gates can
miss it.  n3d_cache_compress runs the same selection and gather code on given
probabilities; here its picks, sentinel and gathered rows must equal the oracle's
`compress_picked` / `compress` exactly, on inputs built to tie at every top-k
boundary: quantised probabilities, repeated prototype rows, and exact 0, -0, 0.5,
the score threshold and 1."""

import numpy as np
import pytest

import n3d
import oracle
import synth
from test_oracle_cache_policy import CASES, _cfg, _probs

pytestmark = pytest.mark.gpu

F32 = np.float32


def _device_cfg(cc) -> n3d.CacheConfig:
    d = n3d.CacheConfig()
    for name, _ in n3d.CacheConfig._fields_:
        setattr(d, name, getattr(cc, name))
    return d


def _edge_probs(rng, nf, ns, thr):
    """Exact boundary values: the 0.5 decision edge, the score clamp, -0, 0 and 1."""
    vals = np.array([0.0, -0.0, thr, 0.5, np.nextafter(F32(0.5), F32(1)), 1.0 - thr, 0.75, 1.0, 0.9999999],
                    F32)
    p = vals[rng.integers(0, vals.size, (nf, ns))]
    mix = rng.random((nf, ns)) < 0.2
    p[mix] = rng.random(int(mix.sum())).astype(F32)
    return p.reshape(-1)


def _check(cc, probs, nf, rng, hidden=16):
    want, sentinel = oracle.compress_picked(cc, probs, nf)
    got, got_sentinel = n3d.cache_compress(0, _device_cfg(cc), probs, nf)
    assert got_sentinel == sentinel
    assert np.array_equal(got, want), np.nonzero(got != want)
    embeds = rng.standard_normal((nf, hidden)).astype(F32)
    silence = rng.standard_normal(hidden).astype(F32)
    oe, op = oracle.compress(cc, hidden, embeds.reshape(-1), probs, nf, silence)
    got2, _, ge, gp = n3d.cache_compress(0, _device_cfg(cc), probs, nf, embeds, hidden, silence)
    assert np.array_equal(got2, want)
    assert np.array_equal(ge, oe.reshape(-1, hidden))
    assert np.array_equal(gp, op.reshape(-1, cc.num_speakers))
    return want


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("ties", [False, True, "rows", "edges"])
def test_device_compression_picks_equal_the_oracle(case, ties):
    cache_len, ns, n_sil, thr, latest, min_pos, ks, kw, nf = CASES[case]
    cc = _cfg(cache_len, ns, n_sil, thr, latest, min_pos, ks, kw)
    rng = np.random.default_rng(1000 + case * 7 + [False, True, "rows", "edges"].index(ties))
    for _ in range(4):
        probs = _edge_probs(rng, nf, ns, thr) if ties == "edges" else _probs(rng, nf, ns, ties)
        _check(cc, probs, nf, rng)


@pytest.mark.parametrize("offline", [False, True])
def test_device_compression_on_the_model_cache_geometry(offline):
    """The synthetic checkpoint's own cache policy (264 frames, 8 speakers, one silence
    slot per speaker), at the candidate counts the chunk loop produces."""
    cc = oracle.cache_cfg_from_model(synth.MODEL_CONFIG, offline=offline)
    rng = np.random.default_rng(77 + offline)
    for nf in (265, 300, 364, 564, 640):
        for kind in (False, True, "rows", "edges"):
            probs = _edge_probs(rng, nf, 8, cc.score_threshold) if kind == "edges" else _probs(rng, nf, 8, kind)
            _check(cc, probs, nf, rng, hidden=512)


def test_all_silent_candidates_give_sentinels_and_silence_rows():
    """No probability above 0.5: every frame scores -inf, so only the +inf silence
    slots survive and the rest of the cache is sentinels."""
    cc = _cfg(32, 8, 1, 0.25, 0.05, 1, 2, 4)
    rng = np.random.default_rng(5)
    probs = (rng.random((40, 8)) * 0.5).astype(F32).reshape(-1)
    want = _check(cc, probs, 40, rng)
    assert (want == 8 * 41).sum() == 32 - 8

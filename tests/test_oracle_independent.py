"""The oracle's front end against an independent float64 restatement (CPU only).

The reference transforms with rustfft 6.4.1, whose summation order cannot be reproduced
here, so the oracle's own radix-2 FFT is not pinned bit for bit.  These tests bound what
that can cost: the oracle's FFT equals numpy's float64 DFT to fp32 rounding, and its
whole log-mel (src/mel.rs:160-225: preemphasis, centre padding, the Hann window centred
in the 512-point frame, power spectrum, filterbank, log guard) stays within 2e-4 of the
same steps computed in float64 with numpy.fft.  An fp32 FFT in any other order lands in
the same band, far inside the reference's 1e-2 front-end tolerance
(src/bin/front_end_check.rs:21)."""

import numpy as np
import pytest

import oracle
import synth

FE = synth.PROCESSOR_CONFIG["feature_extractor"]


@pytest.mark.parametrize("n", [2, 4, 8, 16, 64, 256, 512])
def test_fft_equals_the_float64_dft(n):
    rng = np.random.default_rng(n)
    cases = [rng.standard_normal((2, n)), np.stack([np.ones(n), np.zeros(n)]),  # DC
             np.stack([(-1.0) ** np.arange(n), np.zeros(n)]),                  # Nyquist
             np.stack([np.eye(1, n, n // 3)[0], np.zeros(n)])]                  # impulse
    for x in cases:
        re, im = x.astype(np.float32)
        got_re, got_im = oracle.fft(re, im)
        want = np.fft.fft(re.astype(np.float64) + 1j * im.astype(np.float64))
        err = np.abs((got_re + 1j * got_im.astype(np.float64)) - want).max()
        assert err <= 4e-7 * max(np.abs(want).max(), 1.0), (n, err)


def _log_mel64(s, centered, filters):
    """src/mel.rs:160-225 in float64, with numpy's FFT."""
    n_fft, hop, wl, nm = FE["n_fft"], FE["hop_length"], FE["win_length"], FE["feature_size"]
    nfr = len(s) // hop if centered else (0 if len(s) < n_fft else (len(s) - n_fft) // hop + 1)
    x = s.astype(np.float64)
    x[1:] = x[1:] - FE["preemphasis"] * x[:-1]  # preemphasis before the padding
    if centered:
        x = np.concatenate([np.zeros(n_fft // 2), x, np.zeros(n_fft // 2)])
    w = np.zeros(n_fft)
    left = (n_fft - wl) // 2
    w[left:left + wl] = oracle.hann_periodic_false(wl)
    frames = np.stack([x[t * hop:t * hop + n_fft] * w for t in range(nfr)])
    power = np.abs(np.fft.rfft(frames, axis=1)) ** 2
    return np.log(power @ filters.reshape(nm, n_fft // 2 + 1).astype(np.float64).T + 2.0 ** -24)


@pytest.mark.parametrize("seed,seconds,centered", [(1, 3.0, True), (2, 3.0, False), (3, 0.37, True)])
def test_log_mel_within_2e4_of_float64(seed, seconds, centered):
    filters = oracle.slaney_mel_filterbank(FE["feature_size"], FE["n_fft"], FE["sampling_rate"], 0.0,
                                           FE["sampling_rate"] / 2.0)
    a = synth.clip(seed, seconds, 3)
    got = oracle.log_mel(a, FE, centered, filters)
    want = _log_mel64(a, centered, filters)
    assert got.shape == want.shape
    assert np.abs(got - want).max() < 2e-4


def test_log_mel_of_near_silence():
    filters = oracle.slaney_mel_filterbank(128, 512, 16000, 0.0, 8000.0)
    a = np.zeros(16000, np.float32)
    a[8000:8100] = 1e-4
    assert np.abs(oracle.log_mel(a, FE, True, filters) - _log_mel64(a, True, filters)).max() < 2e-4


def test_gelu_with_a_correctly_rounded_erff():
    """The oracle's GELU uses glibc's erff; the reference uses libm 0.2.16's (neither is
    available to compare directly).  Against the reference's fp32 formula
    0.5 * v * (1 + erff(v / sqrt 2)) (src/tensor.rs:113-120) evaluated with a correctly
    rounded erff, the oracle differs by at most one ulp of erf carried through the
    formula: one ulp of erf can move the rounded 1 + erf by one of its own ulps, so
    |diff| <= 0.5 |v| (ulp(erf) + ulp(1 + erf)) + ulp(result).  Any faithful erff,
    libm's included, stays within twice that of the oracle."""
    from scipy.special import erf

    f = np.float32
    v = np.concatenate([np.linspace(-10, 10, 400_001, dtype=np.float32),
                        np.array([0.0, -0.0, 1e-30, -1e-30, 3.9, -3.9, 5.0, -5.0], np.float32)])
    got = oracle.gelu(v)
    t = (v * f(1.0 / np.sqrt(2.0))).astype(np.float32)  # v * FRAC_1_SQRT_2 in fp32
    e = erf(t.astype(np.float64)).astype(np.float32)      # correctly rounded erff
    one_e = (f(1.0) + e).astype(np.float32)
    want = (f(0.5) * v).astype(np.float32) * one_e
    ulp = lambda a: np.spacing(np.abs(a)).astype(np.float64)
    bound = 0.5 * np.abs(v.astype(np.float64)) * (ulp(e) + ulp(one_e)) + ulp(want)
    diff = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert (diff <= bound).all(), float((diff - bound).max())
    assert np.mean(got == want) > 0.99  # bit-equal almost everywhere

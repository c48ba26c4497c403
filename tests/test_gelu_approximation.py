"""The branch-free GELU of the GEMM epilogue (csrc/gemm.cu, gelu1/gelu2) on the CPU.

Its coefficients come from nemotron3-diarization-wgpu_b200/fit_gelu.py (a fitted
erfc form, evaluated as t * 2^(Q(t) - x^2 log2(e)/2), t = 1/(1 + C1 |x|)).  These
tests check that the fit still reproduces the constants in the kernel source, and
emulate the kernel's fp32 evaluation (each operation rounded to fp32; the GPU's
approximate reciprocal and exp2 taken as correctly rounded) against the reference
formula 0.5 x (1 + erf(x / sqrt 2)) in fp32 (src/tensor.rs:113-120)."""

import os
import re

import numpy as np
import pytest
from scipy.special import erf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GEMM_CU = os.path.join(ROOT, "nemotron3-diarization-wgpu_b200", "csrc", "gemm.cu")
f32 = np.float32


def kernel_constants():
    src = open(GEMM_CU).read()
    c1 = float(re.search(r"GELU_C1 = ([-0-9.e]+)f", src).group(1))
    kx = float(re.search(r"GELU_KX = ([-0-9.e]+)f", src).group(1))
    body = re.search(r"constexpr float gelu_q\(int i\) \{(.*?)\n\}", src, re.S).group(1)
    q = [float(v) for v in re.findall(r"(-?[0-9]+\.[0-9]+)f", body)]
    assert len(q) == 9
    return f32(c1), f32(kx), np.array(q, np.float32)


def gelu_kernel_emulation(x):
    c1, kx, q = kernel_constants()
    x = x.astype(np.float32)
    xd = x.astype(np.float64)

    def fma(a, b, c):
        return (a.astype(np.float64) * b + c).astype(np.float32)

    t = (1.0 / fma(np.full_like(x, c1), np.abs(x), f32(1)).astype(np.float64)).astype(np.float32)
    acc = fma(t, q[8], q[7])
    for i in range(6, -1, -1):
        acc = fma(acc, t, q[i])
    xl = (x * kx).astype(np.float32)
    with np.errstate(over="ignore"):  # x^2 past fp32 range -> -inf, as on the GPU
        y = (acc.astype(np.float64) + xl.astype(np.float64) * xd).astype(np.float32)
    h = (t * np.exp2(y.astype(np.float64)).astype(np.float32)).astype(np.float32)
    d = fma(h, np.full_like(h, -1.0), f32(0.5))
    phi = (f32(0.5) + np.copysign(d, x)).astype(np.float32)
    return (x * phi).astype(np.float32)


def test_fit_reproduces_the_kernel_constants():
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "fit_gelu", os.path.join(ROOT, "nemotron3-diarization-wgpu_b200", "fit_gelu.py"))
    fg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fg)
    coef, err = fg.fit()
    assert err < 5e-8
    q = coef * np.log2(np.e)
    q[0] -= 1.0
    c1, kx, qk = kernel_constants()
    assert np.array_equal(q.astype(np.float32), qk)
    assert c1 == f32(fg.P_SHIFT / np.sqrt(2.0))
    assert kx == f32(-np.log2(np.e) / 2)


@pytest.mark.parametrize("lo,hi", [(-12.0, 12.0), (-4.0, 4.0)])
def test_gelu_emulation_against_the_reference_formula(lo, hi):
    x = np.concatenate([np.linspace(lo, hi, 400_001), np.random.default_rng(0).normal(0, 0.5, 200_000)])
    x = x[(x >= lo) & (x <= hi)].astype(np.float32)
    got = gelu_kernel_emulation(x)
    er = erf((x * f32(0.70710678118654752)).astype(np.float64)).astype(np.float32)
    want = (f32(0.5) * x * (f32(1) + er)).astype(np.float32)
    diff = np.abs(got.astype(np.float64) - want)
    # absolute: the reference's own 1 + erf cancellation for negative x is ~5e-7
    assert diff.max() < 1e-6
    core = np.abs(want) > 1e-3
    ulps = diff[core] / np.spacing(np.abs(want[core])).astype(np.float64)
    assert ulps.mean() < 2.0
    assert np.isfinite(got).all()


def test_gelu_emulation_special_values():
    x = np.array([0.0, -0.0, np.inf, 1e30, -1e30, -40.0, 40.0], np.float32)
    g = gelu_kernel_emulation(x)
    assert g[0] == 0.0 and g[1] == 0.0
    assert g[2] == np.inf and g[3] == np.float32(1e30)
    assert g[4] == 0.0 and g[5] == 0.0 and g[6] == np.float32(40.0)

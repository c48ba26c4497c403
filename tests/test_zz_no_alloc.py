"""The allocation-free linear entry point (n3d_linear_noalloc).

It exists for callers that cannot allocate device memory when they call (a
real-time audio thread that must not block in the driver's allocator, a host
framework that owns all GPU memory through its own pool): its operand split
lives in a fixed 16 MiB array inside the library instead of cudaMalloc'd
scratch.  These tests call it through the C ABI twice in a row and check each
result against the allocating entry point n3d_linear, within the kernel tests'
1e-3 gate; the array keeps the previous call's contents, so the second call
also shows that stale scratch does not leak into a result.  This file is named
to run last, and it passes both alone in a fresh process and after the others.
"""

import numpy as np
import pytest

import n3d

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _run(fn, x, w, b, rows, cols, out):
    import torch

    dx = torch.from_numpy(x).cuda()
    dw = torch.from_numpy(w).cuda()
    db = torch.from_numpy(b).cuda() if b is not None else None
    dy = torch.full((rows * out,), float("nan"), dtype=torch.float32, device="cuda")
    fn(0, dx.data_ptr(), rows, cols, dw.data_ptr(), out, db.data_ptr() if db is not None else None, dy.data_ptr())
    torch.cuda.synchronize()
    return dy.cpu().numpy()


def test_noalloc_linear_matches_the_allocating_entry_point_on_two_calls():
    rng = np.random.default_rng(7)
    cases = [(684, 512, 1536, True), (380, 2048, 512, False)]
    for rows, cols, out, with_bias in cases:
        x = rng.standard_normal(rows * cols).astype(np.float32)
        w = (rng.standard_normal(out * cols) * 0.02).astype(np.float32)
        b = rng.standard_normal(out).astype(np.float32) if with_bias else None
        got = _run(n3d.linear_noalloc, x, w, b, rows, cols, out)
        want = _run(n3d.linear, x, w, b, rows, cols, out)
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() < TOL


def test_noalloc_linear_rejects_requests_beyond_its_scratch():
    import torch

    rows, cols, out = 4096, 1024, 1024  # needs 2 * (4 Mi + 1 Mi) floats > 4 Mi
    d = torch.zeros(16, dtype=torch.float32, device="cuda")
    with pytest.raises(n3d.DiarizationError) as e:
        n3d.linear_noalloc(0, d.data_ptr(), rows, cols, d.data_ptr(), out, None, d.data_ptr())
    assert e.value.kind == "InvalidArgument"
    assert "scratch" in str(e.value)

"""The allocation-free linear entry point (n3d_linear_noalloc).

It exists for callers that cannot allocate device memory when they call (a
real-time audio thread that must not block in the driver's allocator, a host
framework that owns all GPU memory through its own pool): its operand split
lives in a fixed 16 MiB array inside the library instead of cudaMalloc'd
scratch.  These tests call it through the C ABI twice in a row and check each
result against the CPU oracle's tensor::linear within the kernel sweep's gate
(1e-3 absolute, and 3e-5 relative to the largest output), and against the
allocating entry point n3d_linear, which runs the same dot products in the same
order.  The array keeps the previous call's contents, so the second call also
shows that stale scratch does not leak into a result.  This file is named to run
last, and it passes both alone in a fresh process and after the others.
"""

import numpy as np
import pytest

import n3d
import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-3
CAPACITY = 4 << 20  # 4-byte words in the fixed scratch


def _run(fn, x, w, b, rows, cols, out, **kw):
    import torch

    dx = torch.from_numpy(x).cuda()
    dw = torch.from_numpy(w).cuda()
    db = torch.from_numpy(b).cuda() if b is not None else None
    dy = torch.full((rows * out,), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    fn(0, dx.data_ptr(), rows, cols, dw.data_ptr(), out, db.data_ptr() if db is not None else None, dy.data_ptr(),
       **kw)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


def _operands(rng, rows, cols, out, with_bias):
    x = rng.standard_normal(rows * cols).astype(np.float32)
    w = (rng.standard_normal(out * cols) * 0.02).astype(np.float32)
    b = rng.standard_normal(out).astype(np.float32) if with_bias else None
    return x, w, b


def _need(rows, cols, out):
    """Scratch words a call takes: 64 for the two operands' maxima, then each operand's
    fp16 split (n fp16 twice = n words, rounded up to 64)."""
    r64 = lambda n: (n + 63) // 64 * 64
    return 64 + r64(rows * cols) + r64(out * cols)


def _check(x, w, b, rows, cols, out, **kw):
    got = _run(n3d.linear_noalloc, x, w, b, rows, cols, out, **kw)
    assert np.isfinite(got).all()
    ref = _run(n3d.linear, x, w, b, rows, cols, out)
    assert np.array_equal(got, ref)
    want = oracle.linear(x, rows, cols, w, out, b)
    err = np.abs(got - want).max()
    assert err < TOL and err <= 3e-5 * max(1.0, np.abs(want).max()), err


CASES = [  # rows, cols, out, bias
    (684, 512, 1536, True),   # the QKV projection of a steady-state window
    (380, 2048, 512, False),  # FC2 of an offline window
    (33, 32, 37, True),       # rows*cols and out*cols not multiples of 64: padded parts
]


def test_noalloc_linear_matches_the_oracle_on_two_calls_in_a_row():
    rng = np.random.default_rng(7)
    for rows, cols, out, with_bias in CASES:
        for _ in range(2):
            _check(*_operands(rng, rows, cols, out, with_bias), rows, cols, out)


def test_noalloc_linear_at_exactly_its_capacity():
    rows, cols, out = 65471, 64, 64
    assert _need(rows, cols, out) == CAPACITY
    rng = np.random.default_rng(8)
    _check(*_operands(rng, rows, cols, out, True), rows, cols, out)


def test_noalloc_linear_on_a_caller_stream():
    import torch

    s = torch.cuda.Stream()
    rng = np.random.default_rng(9)
    _check(*_operands(rng, 300, 512, 192, True), 300, 512, 192, stream=s.cuda_stream)


def test_noalloc_linear_rejects_requests_beyond_its_scratch():
    import torch

    d = torch.zeros(16, dtype=torch.float32, device="cuda")
    for rows, cols, out in [(4096, 1024, 1024), (65472, 64, 64)]:  # the second is one row past capacity
        assert _need(rows, cols, out) > CAPACITY
        with pytest.raises(n3d.DiarizationError) as e:
            n3d.linear_noalloc(0, d.data_ptr(), rows, cols, d.data_ptr(), out, None, d.data_ptr())
        assert e.value.kind == "InvalidArgument"
        assert "scratch" in str(e.value)
    # the call after a rejection still works
    rng = np.random.default_rng(10)
    _check(*_operands(rng, 64, 64, 64, False), 64, 64, 64)

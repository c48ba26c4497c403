"""Failure detection on the GPU, without a fault.

Every wait in the library's kernels is bounded: when it gives up it records its
site in a device status word, the kernel frees its TMEM and returns, and the host
reports N3D_ERR_TIMEOUT (the reference only reports wgpu errors,
src/gpu_engine.rs:1345-1349).  n3d_selftest_wait_timeout runs that path on a flag
that nothing sets, with a short limit.  These tests check the status, the message,
the time the wait took, and that the device computes correctly right afterwards."""

import numpy as np
import pytest

import n3d
import oracle

pytestmark = pytest.mark.gpu


def _linear_ok():
    import torch

    rng = np.random.default_rng(3)
    m, k, n = 300, 512, 192
    x = rng.standard_normal(m * k).astype(np.float32)
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    dy = torch.empty(m * n, dtype=torch.float32, device="cuda")
    n3d.linear(0, dx.data_ptr(), m, k, dw.data_ptr(), n, db.data_ptr(), dy.data_ptr())
    return np.abs(dy.cpu().numpy() - oracle.linear(x, m, k, w, n, b)).max() < 1e-3


@pytest.mark.parametrize("limit_ms", [1.0, 20.0])
def test_an_expired_device_wait_reports_timeout_and_leaves_the_device_usable(limit_ms):
    st, msg, waited = n3d.selftest_wait_timeout(0, limit_ms)
    assert n3d.STATUS[st] == "Timeout", msg
    assert "timed out" in msg and "site 6" in msg
    assert limit_ms <= waited < limit_ms + 500.0, waited
    assert _linear_ok()
    # the status word was cleared: a second expired wait reports itself again, and the
    # work after it still succeeds
    st, msg, _ = n3d.selftest_wait_timeout(0, limit_ms)
    assert n3d.STATUS[st] == "Timeout"
    assert _linear_ok()


def test_a_model_run_after_an_expired_wait_is_unaffected(tiny_gpu_model, tiny_oracle):
    import synth
    from conftest import frame_check

    a = synth.clip(12, 4.0, 3)
    before = tiny_gpu_model.run_offline(a)
    st, _, _ = n3d.selftest_wait_timeout(0, 2.0)
    assert n3d.STATUS[st] == "Timeout"
    after = tiny_gpu_model.run_offline(a)
    assert np.array_equal(before.logits, after.logits)
    r = frame_check(after.logits, tiny_oracle.run_offline(a)["logits"])
    assert r["maxdiff"] < 2e-2 and r["flips"] == 0 and r["segments_identical"]

"""Kernel-level parity on a B200 through the C ABI: the tcgen05 GEMM (fp16 split:
h*h + h*l + l*h with per-operand power-of-two scales),
LayerNorm and RoPE+attention against the CPU oracle's restatement of
src/tensor.rs and src/encoder.rs.

Shapes: the reference's own GPU probe lists (src/bin/gpu_check.rs:78-130) and
the kernel-sweep configuration (GEMM M in {1024, 4096, 16384} x K, N in
{512..4096}, A ~ N(0,1), B ~ N(0,1/K) + bias; attention 8 heads, head_dim
64/128, seq 512/1024/4096 with RoPE and a key mask; LayerNorm [16384 x 1024]).
Tolerance: the sweep's 1e-3 max-abs gate (and the probes' 1e-3).  The GEMM
lands orders of magnitude inside it (~2^-22 relative per product), which the tighter
relative bound also checks; attention runs on the same fp16 split (Q, K, V and P
scaled by powers of two), ~2^-22 per product.
"""

import numpy as np
import pytest

import n3d
import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _cuda(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _gemm(x, w, b, rows, cols, out):
    import torch

    dx, dw = _cuda(x), _cuda(w)
    db = _cuda(b) if b is not None else None
    dy = torch.empty(rows * out, dtype=torch.float32, device="cuda")
    n3d.linear(0, dx.data_ptr(), rows, cols, dw.data_ptr(), out, db.data_ptr() if db is not None else None,
               dy.data_ptr())
    torch.cuda.synchronize()
    return dy.cpu().numpy()


# GEMM_CHECK shapes, src/bin/gpu_check.rs:111-120 (M, N, K)
PROBE_SHAPES = [(128, 128, 512), (380, 512, 512), (380, 2048, 512), (684, 512, 512), (505, 512, 512),
                (380, 100, 512), (380, 8, 512), (17, 24, 512), (684, 1536, 512), (376, 512, 2048),
                (3008, 192, 576), (8, 192, 192)]


@pytest.mark.parametrize("m,n,k", PROBE_SHAPES)
def test_linear_matches_oracle_on_probe_shapes(m, n, k):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    x = rng.standard_normal(m * k).astype(np.float32)
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    got = _gemm(x, w, b, m, k, n)
    want = oracle.linear(x, m, k, w, n, b)
    err = np.abs(got - want).max()
    assert err < TOL
    # fp32-grade: well inside the gate
    assert err <= 1e-5 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("m", [1024, 4096, 16384])
@pytest.mark.parametrize("k", [512, 1024, 2048, 4096])
@pytest.mark.parametrize("n", [512, 1024, 2048, 4096])
def test_linear_kernel_sweep(m, k, n):
    """Kernel sweep; the oracle checks 48 sampled rows (each output row is an
    independent dot-product chain, so a row subset is an exact check of it)."""
    rng = np.random.default_rng(2)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = (rng.standard_normal((n, k), dtype=np.float32) / np.float32(np.sqrt(k))).astype(np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    got = _gemm(x, w, b, m, k, n).reshape(m, n)
    rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, 46)]))
    want = oracle.linear(x[rows], len(rows), k, w, n, b).reshape(len(rows), n)
    assert np.abs(got[rows] - want).max() < TOL
    assert np.isfinite(got).all()


@pytest.mark.parametrize("m,n", [(10240, 512), (49152, 512), (16384, 1024)])
def test_linear_pair_tiles_with_a_partial_last_wave_match_oracle(m, n):
    """CTA-pair shapes (256 x 256 tiles) whose last wave is partial (10240 x 512: 80
    tiles on 74 pairs); every row of the last 1024 and a sample of the others against
    the oracle."""
    k = 512
    rng = np.random.default_rng(5)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    got = _gemm(x, w, b, m, k, n).reshape(m, n)
    rows = np.unique(np.concatenate([np.arange(m - 1024, m), rng.integers(0, m - 1024, 64)]))
    want = oracle.linear(x[rows], len(rows), k, w, n, b).reshape(len(rows), n)
    err = np.abs(got[rows] - want).max()
    assert err < TOL
    assert err <= 1e-5 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("rows,cols", [(17, 512), (684, 512), (16384, 1024)])
def test_layer_norm_matches_oracle(rows, cols):
    import torch

    rng = np.random.default_rng(rows)
    x = (rng.standard_normal(rows * cols) * 3 + 0.5).astype(np.float32)
    w = rng.standard_normal(cols).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    dx, dw, db = _cuda(x), _cuda(w), _cuda(b)
    dy = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    n3d.layer_norm(0, dx.data_ptr(), rows, cols, dw.data_ptr(), db.data_ptr(), dy.data_ptr())
    got = dy.cpu().numpy()
    want = oracle.layer_norm(x, rows, cols, w, b)
    assert np.abs(got - want).max() < 1e-5


# ATTN_GEMM_CHECK seqs (src/bin/gpu_check.rs:84) and the sweep's (512, 1024, 4096)
@pytest.mark.parametrize("seq,hd,valid", [(8, 64, 5), (17, 64, 17), (130, 64, 101), (380, 64, 380), (684, 64, 683),
                                          (512, 64, 512), (512, 128, 400), (1024, 64, 1000), (1024, 128, 1024),
                                          (4096, 64, 4000), (4096, 128, 4096), (8, 128, 5), (17, 128, 17),
                                          (130, 128, 101), (684, 128, 683)])
def test_rope_attention_matches_oracle(seq, hd, valid):
    import torch

    heads = 8
    rng = np.random.default_rng(seq + hd)
    q, k, v = (rng.standard_normal(seq * heads * hd).astype(np.float32) for _ in range(3))
    dq, dk, dv = _cuda(q), _cuda(k), _cuda(v)
    do = torch.empty(seq * heads * hd, dtype=torch.float32, device="cuda")
    n3d.attention(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), seq, heads, hd, valid, do.data_ptr())
    got = do.cpu().numpy()
    cs, sn = oracle.rope_tables(seq, hd)
    qr = oracle.apply_rope(q, seq, heads, hd, cs, sn)
    kr = oracle.apply_rope(k, seq, heads, hd, cs, sn)
    want = oracle.attention(qr, kr, v, seq, heads, hd, valid)
    assert np.abs(got - want).max() < TOL


@pytest.mark.parametrize("hd", [64, 128])
def test_attention_with_no_valid_keys_is_zero(hd):
    import torch

    seq, heads = 8, 8
    q = np.ones(seq * heads * hd, np.float32)
    dq = _cuda(q)
    do = torch.full((seq * heads * hd,), 7.0, dtype=torch.float32, device="cuda")
    n3d.attention(0, dq.data_ptr(), dq.data_ptr(), dq.data_ptr(), seq, heads, hd, 0, do.data_ptr())
    assert (do.cpu().numpy() == 0).all()

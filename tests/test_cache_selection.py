"""The selection rule of the speaker-cache kernel (csrc/cache.cu), restated in numpy.

The kernel picks "the first k of a stable descending sort" (Rust's stable `sort_by`
then a truncation: src/streaming.rs:333-346, 436-463) without sorting: it finds the
k-th largest order key by an MSB-first radix select, keeps every element above it,
and among the elements equal to it keeps the lowest indices.  This checks that rule
against a stable sort on adversarial data (heavy ties, -inf, +inf)."""

import numpy as np
import pytest


def order_key(v):
    v = np.asarray(v, np.float32) + np.float32(0.0)  # -0 -> +0, as the kernel does
    u = v.view(np.uint32).astype(np.uint64)
    return np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)


def radix_select_first_k(v, k):
    """Flags of the first k elements in (value desc, index asc) order."""
    key = order_key(v)
    n = len(key)
    k = min(k, n)
    flags = np.zeros(n, bool)
    if k == 0:
        return flags
    prefix, mask, need = 0, 0, k
    for bit in range(31, -1, -1):
        b = 1 << bit
        c = int(np.count_nonzero(((key & mask) == prefix) & ((key & b) != 0)))
        if c >= need:
            prefix |= b
        else:
            need -= c
        mask |= b
    eq = key == prefix
    tie_rank = np.cumsum(eq) - eq
    return (key > prefix) | (eq & (tie_rank < need))


def stable_first_k(v, k):
    order = sorted(range(len(v)), key=lambda i: (-float(v[i]), i))
    flags = np.zeros(len(v), bool)
    flags[order[:k]] = True
    return flags


@pytest.mark.parametrize("seed", range(12))
def test_radix_selection_equals_stable_sort_prefix(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 700))
    pool = np.array([-np.inf, np.inf, 0.0, -0.0, 1.5, -2.25, 3.0, 1e-30, -1e30], np.float32)
    v = np.where(rng.random(n) < 0.5, rng.choice(pool, n), rng.standard_normal(n)).astype(np.float32)
    for k in (0, 1, 24, 48, n // 2, n, n + 5):
        assert np.array_equal(radix_select_first_k(v, k), stable_first_k(v, min(k, n))), (seed, k)


def test_signed_zeros_tie_like_the_reference():
    v = np.array([-0.0, 0.0, -0.0, 1.0, 0.0], np.float32)
    assert np.array_equal(np.flatnonzero(radix_select_first_k(v, 3)), [0, 1, 3])


def test_all_equal_values_keep_the_lowest_indices():
    v = np.full(100, -np.inf, np.float32)
    assert np.array_equal(np.flatnonzero(radix_select_first_k(v, 7)), np.arange(7))

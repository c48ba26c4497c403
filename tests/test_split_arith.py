"""Integer identities the kernels' fp16 splits rely on, checked on the host.

The attention kernel (csrc/attention_tc.cu, split_p2) forms the fp16 bits of
h = round11(x), x = P * 2^7 in [2^-14, 2^15], as the high half of
bits(x) * 8 + 0x40008000 (modulo 2^32) instead of (bits(x) + 2^12 - (112 << 23)) >> 13,
and l = x - h in fp32.  These tests check, over every float bit pattern of that range
(strided) and its edges, that both give the same 16 bits, that the result is the
round-half-up 11-bit rounding of x as an fp16, and that h + l reproduces x exactly
before l's own rounding to fp16.
"""

import numpy as np

LO = np.float32(2.0**-14).view(np.uint32)
HI = np.float32(2.0**15).view(np.uint32)


def _bits(stride):
    b = np.arange(int(LO), int(HI) + 1, stride, dtype=np.uint64)
    edges = np.array([LO, LO + 1, HI - 1, HI, 0x3F7FFFFF, 0x3F800000, 0x46FFF000, 0x46FFF001], dtype=np.uint64)
    return np.unique(np.concatenate([b, edges])).astype(np.uint32)


def _h_reference(bits):
    return ((bits.astype(np.uint64) + 0x1000 - 0x38000000) >> 13).astype(np.uint16)


def _h_kernel(bits):
    return (((bits.astype(np.uint64) * 8 + 0x40008000) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def test_high_half_form_equals_the_shifted_rebias():
    bits = _bits(3)
    assert np.array_equal(_h_kernel(bits), _h_reference(bits))


def test_h_is_x_rounded_to_11_bits_and_h_plus_l_is_x():
    bits = _bits(101)
    x = bits.view(np.float32)
    h16 = _h_kernel(bits).view(np.float16).astype(np.float32)
    # round half up (away from zero) to 11 significant bits
    rounded = ((bits.astype(np.uint64) + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)
    assert np.array_equal(h16, rounded)
    l = (x - h16).astype(np.float32)
    assert np.array_equal((h16.astype(np.float64) + l.astype(np.float64)).astype(np.float32), x)
    # |l| <= half an 11-bit ulp of x: l's fp16 rounding then costs at most 2^-23 relative
    assert np.all(np.abs(l) <= np.ldexp(np.abs(x), -11))

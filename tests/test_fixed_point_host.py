"""Host-side checks of the fixed-point sums the radix aggregation pass keeps for f32 values
(winrapids_b200/csrc/radix.cu, rx_agg_kernel): a value v with 2^-13 <= |v| < 2^E is added as the
integer q = v * 2^36, held in two u32 words per group; the low word's atomic add returns the old
low word, from which the adding thread knows the carry into the high word.  These tests restate
that arithmetic in Python and check the three facts the kernel depends on:

  * every f32 with |v| >= 2^-13 is an exact multiple of 2^-36 (so q is an integer);
  * the two-word sum with carries taken from the returned low words equals the exact sum modulo
    2^64, whatever order the adds arrive in;
  * with E = 63 - 36 - bits(cap), a bucket of at most `cap` rows cannot leave the signed 63-bit range.
"""
import math

import numpy as np

FX_SHIFT = 36
FX_MIN = 2.0 ** -13


def fx_lim(cap):
    cap_bits = (cap | 1).bit_length()  # 64 - clz(cap | 1)
    return 2.0 ** (63 - FX_SHIFT - cap_bits)


def two_word_sum(qs):
    """The kernel's update: lo += xl (returns old), hi += xh + carry, all modulo 2^32."""
    lo = hi = 0
    for q in qs:
        u = q & (2**64 - 1)
        xl, xh = u & 0xFFFFFFFF, u >> 32
        old = lo
        lo = (lo + xl) & 0xFFFFFFFF
        carry = 1 if lo < old else 0  # (old + xl) wrapped
        hi = (hi + xh + carry) & 0xFFFFFFFF
    total = (hi << 32) | lo
    return total - 2**64 if total >= 2**63 else total


def test_f32_at_or_above_the_threshold_is_a_multiple_of_2_pow_minus_36():
    rng = np.random.default_rng(1)
    for e in range(-13, 40):
        mant = rng.integers(1 << 23, 1 << 24, 2000, dtype=np.int64)
        v = (mant.astype(np.float64) * 2.0 ** (e - 23)).astype(np.float32)
        q = v.astype(np.float64) * 2.0**FX_SHIFT
        assert np.all(q == np.round(q)), e
    # just below the threshold the f32 grid is finer than 2^-36
    below = np.nextafter(np.float32(FX_MIN), np.float32(0.0))
    q = float(below) * 2.0**FX_SHIFT
    assert q != round(q)


def test_two_word_sum_is_exact_in_any_order():
    rng = np.random.default_rng(2)
    for trial in range(200):
        n = int(rng.integers(1, 60))
        mag = 2.0 ** rng.integers(-13, 12, n)
        v = (rng.uniform(1.0, 2.0, n) * mag * rng.choice([-1.0, 1.0], n)).astype(np.float32)
        qs = [int(x) for x in (v.astype(np.float64) * 2.0**FX_SHIFT)]
        exact = sum(qs)
        for _ in range(3):
            order = rng.permutation(n)
            assert two_word_sum([qs[i] for i in order]) == exact, trial
        # the kernel's output: the exact integer rounded once to f64, scaled back
        got = math.ldexp(float(two_word_sum(qs)), -FX_SHIFT)
        want = math.fsum(float(x) for x in v.astype(np.float64))
        assert abs(got - want) <= 2.0**-52 * abs(want) + 1e-300


def test_range_bound_keeps_a_full_bucket_inside_63_bits():
    for cap in (1, 2, 100, 7_629, 11_392, 1 << 14, (1 << 14) + 1, 40_000, 1 << 20):
        lim = fx_lim(cap)
        largest = np.nextafter(np.float32(lim), np.float32(0.0))  # the largest f32 below the limit
        q = int(float(largest) * 2.0**FX_SHIFT)
        assert cap * q < 2**63, cap
        assert -cap * q > -(2**63), cap
        # the carries stay exact at the bound
        assert two_word_sum([q] * min(cap, 64)) == q * min(cap, 64)

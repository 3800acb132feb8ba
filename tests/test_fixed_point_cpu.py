"""The int64 fixed-point histogram sums against the exactness known answers
of the reference's own integer summation (src/backend/exact_sum.rs tests
`domain_boundary`, `in_domain_sums_match_the_cpu_chain`,
`the_cpu_chain_rounds_just_past_the_bound`), restated for the fixed-point
form the CUDA path sums in: q = rint(v * 2^s), s = 53 - ceil(log2 n) - e with
max|v| < 2^e, so that every sum of n such values is an integer below 2^53,
held exactly by an f64 (the C ABI's GradStats).

Checked on the CPU oracle, whose fixed-point histograms the GPU kernels
equal bit for bit (tests/test_gpu_parity.py)."""

import math

import numpy as np
import pytest

import oracle_lib as O


def _one_feature(n, n_bins):
    """A complete single-feature matrix whose value i % n_bins lands in bin
    i % n_bins, with its cuts."""
    x = (np.arange(n) % n_bins).astype(np.float32).reshape(-1, 1)
    off, cuts = O.cuts_dense(x[:n_bins], 256)
    assert off[1] - off[0] == n_bins
    return x, off, cuts


def _xorshift(seed):
    state = seed
    mask = (1 << 64) - 1
    while True:
        state ^= (state << 13) & mask
        state ^= state >> 7
        state ^= (state << 17) & mask
        yield state


def test_scale_keeps_every_sum_inside_int64():
    # `domain_boundary` in fixed-point terms: n values of magnitude up to
    # max|v| < 2^e sum to at most n * max|v| * 2^s <= 2^53 once scaled
    for max_abs in (1.0, float(np.nextafter(np.float32(1.0), np.float32(0.0))), 4.0, 2.0**-10, 2.0**60):
        for n in (1, 2, 3, 4096, 1 << 24, 1 << 41):
            s = O.fixed_scale(max_abs, n)
            q = round(float(np.float32(max_abs)) * 2.0**s)
            assert q * n <= 1 << 53, (max_abs, n, s)
            # and it wastes at most one bit each to rounding n and max|v|
            # up to powers of two
            assert 4 * q * (1 << (n - 1).bit_length()) > 1 << 53, (max_abs, n, s)
    # zeros take the identity scale; the smallest subnormal scales up past 2^53
    assert O.fixed_scale(0.0, 1 << 60) == 0
    assert O.fixed_scale(float(np.uint32(1).view(np.float32)), 1) == 53 + 148


@pytest.mark.parametrize("case", range(40))
def test_in_domain_fixed_sums_match_the_f64_chain(case):
    # `in_domain_sums_match_the_cpu_chain`: mostly-positive values with full
    # 24-bit significands near the top of the exact range, mixed with odd
    # small ones. Where the f64 sums are exact the fixed-point sums equal
    # them bit for bit, whatever the row grouping. The scale keeps
    # max|v| < 2^e strictly, so the largest value is one bit below the f64
    # domain's 2^(53 - ceil(log2 n)) to keep a grain of 1.
    rnd = _xorshift(0x9E3779B97F4A7C15 + case)
    n = 4096 + next(rnd) % 4096
    top = 52 - math.ceil(math.log2(n))
    vals = []
    for _ in range(n):
        r = next(rnd)
        sign = -1.0 if (r >> 40) % 8 == 0 else 1.0
        kind = (r >> 1) % 4
        if kind < 2:
            v = float((r >> 8) % (1 << 24)) * 2.0 ** (top - 24)
        elif kind == 2:
            v = float((r >> 8) % 1000 * 2 + 1)
        else:
            v = 2.0**top
        vals.append(sign * v)
    g = np.array(vals, np.float32)
    assert np.array_equal(g.astype(np.float64), np.array(vals))  # every value is an f32
    x, off, cuts = _one_feature(n, 8)
    gp = np.stack([g, np.ones(n, np.float32)], 1)
    sg = O.fixed_scale(float(np.max(np.abs(g))), n)
    sh = O.fixed_scale(1.0, n)
    assert sg >= 0, "the grain of these values is 2^0 or coarser"
    rows = np.arange(n, dtype=np.uint32)
    f64 = O.hist(x, off, cuts, rows, gp)
    fixed = O.hist(x, off, cuts, rows, gp, fixed_point=True, sg=sg, sh=sh)
    exact = [sum(int(vals[i]) for i in range(b, n, 8)) for b in range(8)]
    for b in range(8):
        assert int(fixed[b, 0]) == exact[b] << sg
        assert int(fixed[b, 1]) == len(range(b, n, 8)) << sh
        assert float(exact[b]) == f64[b, 0]
        assert math.ldexp(float(int(fixed[b, 0])), -sg) == f64[b, 0]
    # any row subset and order: the integer sums are order-free
    perm = np.array(list(reversed(range(n))), np.uint32)[::3]
    a = O.hist(x, off, cuts, perm, gp, fixed_point=True, sg=sg, sh=sh)
    b = O.hist(x, off, cuts, np.sort(perm), gp, fixed_point=True, sg=sg, sh=sh)
    np.testing.assert_array_equal(a, b)


def test_fixed_sums_stay_exact_past_the_f64_chain_bound():
    # `the_cpu_chain_rounds_just_past_the_bound`: 1 + k * 2^30 with
    # k = 2^23 + 1 is 2^53 + 2^30 + 1, which no f64 holds, and the f64 chain
    # rounds it in an order-dependent way. The fixed-point scale puts the
    # grain where the n-row sum stays within 2^53: here 4, so the 1 rounds to
    # 0 once, at quantisation, and the integer sum is exact in an f64.
    k = (1 << 23) + 1
    n = k + 1
    g = np.full(n, 2.0**30, np.float32)
    g[0] = 1.0
    x = np.zeros((n, 1), np.float32)
    off, cuts = O.cuts_dense(x[:1], 256)
    gp = np.stack([g, np.ones(n, np.float32)], 1)
    rows = np.arange(n, dtype=np.uint32)
    sg = O.fixed_scale(2.0**30, n)
    assert sg == -2
    want = sum(int(np.rint(np.float64(v) * 2.0**sg)) for v in (1.0, 2.0**30)) + (k - 1) * (1 << 28)
    fixed = O.hist(x, off, cuts, rows, gp, fixed_point=True, sg=sg, sh=0)
    assert int(fixed[0, 0]) == want and want < 1 << 53
    assert float(int(fixed[0, 0])) == int(fixed[0, 0])  # the f64 ABI carries it exactly
    chain = np.cumsum(g.astype(np.float64))[-1]  # sequential f64 adds in row order
    assert int(chain) == 1 + k * (1 << 30) - 1

"""hb_build_noalloc (the node histogram on caller-owned device buffers, with
static scratch) against hb_build, the entry point it varies, and against the
CPU oracle's fixed-point histogram of the same rows.

Some callers cannot allocate device memory while they run: a host framework
that hands all of HBM to its own pool allocator, or one that forbids
cudaMalloc once training has started. This entry point serves them, and the
tests below check both its results and that it allocates nothing.

Tolerance: none. Both entry points sum the same int64 fixed-point values
with the same kernel and dequantise once, so their f64 outputs are equal
bit for bit; the comparison uses rtol=0, atol=0.

This file is collected last on purpose: it must pass both alone in a fresh
process (the first call on the device does the scratch set-up) and after
every other test of the suite.
"""

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
from hessboost_b200 import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TOL = dict(rtol=0.0, atol=0.0)


def _device(a, dtype):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda:0", dtype=dtype)
    torch.cuda.synchronize()
    return t


def _noalloc(e, rows_np, total_bins):
    rows = _device(rows_np.astype(np.int32), torch.int32)
    out = torch.full((total_bins, 2), float("nan"), dtype=torch.float64, device="cuda:0")
    torch.cuda.synchronize()
    e.build_noalloc(rows.data_ptr(), rows.numel(), out.data_ptr())
    return out.cpu().numpy()


@pytest.fixture(scope="module")
def staged():
    x, y = synth.logistic_c2(200_003, 28, seed=31)
    m = H.BinnedMatrix.from_dense(x)
    e = H.Engine()
    e.upload(m)
    rng = np.random.default_rng(5)
    e.load_margins((rng.standard_normal(m.n_rows) * 0.5).astype(np.float32))
    assert e.gradients(H.HB_LOSS_LOGISTIC, y)
    e.x = x
    yield e, m
    e.close()


def test_matches_oracle_fixed_point(staged):
    """The no-allocation histogram equals the oracle's int64 fixed-point sums
    of the same rows, dequantised with the engine's scales."""
    e, m = staged
    gp, sg, sh = e.read_gradients()
    rows = np.arange(1, m.n_rows, 7, dtype=np.uint32)
    q = O.hist(e.x, m.feature_offset, m.cut_values, rows, gp, fixed_point=True, sg=sg, sh=sh)
    want = np.stack([q[:, 0].astype(np.float64) * 2.0 ** -sg, q[:, 1].astype(np.float64) * 2.0 ** -sh], 1)
    np.testing.assert_array_equal(_noalloc(e, rows, m.total_bins), want)


def test_allocates_no_device_memory(staged):
    """After the first call (which only looks up the static array's address),
    further calls leave the device's free memory unchanged."""
    e, m = staged
    rows_a = _device(np.arange(0, m.n_rows, 2).astype(np.int32), torch.int32)
    rows_b = _device(np.arange(1, m.n_rows, 5).astype(np.int32), torch.int32)
    out = torch.zeros((m.total_bins, 2), dtype=torch.float64, device="cuda:0")
    torch.cuda.synchronize()
    e.build_noalloc(rows_a.data_ptr(), rows_a.numel(), out.data_ptr())
    free0 = torch.cuda.mem_get_info(0)[0]
    for r in (rows_b, rows_a, rows_b):
        e.build_noalloc(r.data_ptr(), r.numel(), out.data_ptr())
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0


def test_invalid_arguments_record_a_reason(staged):
    e, m = staged
    rows = torch.arange(10, dtype=torch.int32, device="cuda:0")
    out = torch.zeros((m.total_bins, 2), dtype=torch.float64, device="cuda:0")
    torch.cuda.synchronize()
    cases = [(rows.data_ptr(), m.n_rows + 1, out.data_ptr(), "more row ids"),
             (rows.data_ptr(), 10, 0, "NULL"),
             (rows.data_ptr() + 2, 4, out.data_ptr(), "aligned")]
    for rp, n, op, why in cases:
        with pytest.raises(H.HbError, match=why) as ex:
            e.build_noalloc(rp, n, op)
        assert ex.value.status == H.HB_INVALID_ARGUMENT
    # still usable
    np.testing.assert_allclose(_noalloc(e, np.arange(0, m.n_rows, 3, dtype=np.uint32), m.total_bins),
                               e.build(np.arange(0, m.n_rows, 3, dtype=np.uint32)), **TOL)


def test_two_calls_in_a_row_match_build(staged):
    e, m = staged
    n = m.n_rows
    rng = np.random.default_rng(7)
    rows_a = np.sort(rng.choice(n, size=n * 2 // 5, replace=False)).astype(np.uint32)
    rows_b = np.arange(n // 3, n, dtype=np.uint32)
    got_a = _noalloc(e, rows_a, m.total_bins)
    got_b = _noalloc(e, rows_b, m.total_bins)
    np.testing.assert_allclose(got_a, e.build(rows_a), **TOL)
    np.testing.assert_allclose(got_b, e.build(rows_b), **TOL)
    # and the same rows again: the scratch starts from zero every call
    np.testing.assert_allclose(_noalloc(e, rows_a, m.total_bins), got_a, **TOL)


def test_empty_rows_give_zero_histogram(staged):
    e, m = staged
    rows = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    out = torch.full((m.total_bins, 2), float("nan"), dtype=torch.float64, device="cuda:0")
    torch.cuda.synchronize()
    e.build_noalloc(rows.data_ptr(), 0, out.data_ptr())
    np.testing.assert_array_equal(out.cpu().numpy(), 0.0)


def test_bad_rows_refused_without_reading(staged):
    e, m = staged
    n = m.n_rows
    for bad in (np.array([5, 3, 9], np.uint32), np.array([0, 1, n], np.uint32),
                np.array([2, 2], np.uint32)):
        rows = _device(bad.astype(np.int32), torch.int32)
        out = torch.full((m.total_bins, 2), float("nan"), dtype=torch.float64, device="cuda:0")
        torch.cuda.synchronize()
        with pytest.raises(H.HbError) as ex:
            e.build_noalloc(rows.data_ptr(), rows.numel(), out.data_ptr())
        assert ex.value.status == H.HB_REFUSED
        np.testing.assert_array_equal(out.cpu().numpy(), 0.0)
    # the engine stays usable
    rows = np.arange(0, n, 3, dtype=np.uint32)
    np.testing.assert_allclose(_noalloc(e, rows, m.total_bins), e.build(rows), **TOL)


def test_host_buffers_refused(staged):
    e, m = staged
    rows = np.arange(10, dtype=np.uint32)
    out = np.zeros((m.total_bins, 2), np.float64)
    with pytest.raises(H.HbError) as ex:
        e.build_noalloc(rows.ctypes.data, rows.size, out.ctypes.data)
    assert ex.value.status == H.HB_REFUSED


def test_index_beyond_scratch_refused():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3000, 200)).astype(np.float32)
    m = H.BinnedMatrix.from_dense(x)
    assert 32768 < m.total_bins
    e = H.Engine()
    try:
        e.upload(m)
        e.load_margins(np.zeros(m.n_rows, np.float32))
        assert e.gradients(H.HB_LOSS_SQUARED_ERROR, rng.standard_normal(m.n_rows).astype(np.float32))
        rows = torch.arange(100, dtype=torch.int32, device="cuda:0")
        out = torch.zeros((m.total_bins, 2), dtype=torch.float64, device="cuda:0")
        torch.cuda.synchronize()
        with pytest.raises(H.HbError, match="32768 bins") as ex:
            e.build_noalloc(rows.data_ptr(), 100, out.data_ptr())
        assert ex.value.status == H.HB_REFUSED
    finally:
        e.close()

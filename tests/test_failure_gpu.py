"""Failure handling with a host-side fault injector (no GPU fault).

The reference's contract (src/tree/hist/mod.rs:209-212,
src/backend/cuda/driver.rs:26-44): a backend call that did not run answers
`None` and the caller keeps its host path; a device error poisons the
backend for the rest of the process. hb_engine_inject_fault makes one of the
engine's checked CUDA calls fail on the host, before it reaches CUDA and
outside any stream capture, exactly as a device error would be reported.
Checked here: that call answers HB_DEVICE_FAILED, every later call on the
engine HB_REFUSED (destroy still works), and a fresh engine on the same GPU
trains bit-exact as before.
"""

import numpy as np
import pytest

import hessboost_b200 as H
from hessboost_b200 import synth

pytestmark = pytest.mark.gpu


def _forest_bits(m):
    return m.nodes.tobytes(), np.asarray(m.tree_ptr).tobytes()


@pytest.fixture(scope="module")
def data():
    x, y = synth.logistic_c2(20_011, 12, seed=7)
    p = H.TrainingParams(objective="binary:logistic", max_depth=6, eta=0.3)
    m = H.BinnedMatrix.from_dense(x)
    want = H.train(p, y=y, rounds=3, matrix=m)
    return x, y, p, m, want


def _until_failure(fn, limit=60):
    for _ in range(limit):
        try:
            fn()
        except H.HbError as err:
            return err
    raise AssertionError("the armed fault never fired")


@pytest.mark.parametrize("after", [0, 1, 5, 25])
def test_fault_in_training_is_sticky(data, after):
    x, y, p, m, want = data
    e = H.Engine()
    try:
        e.upload(m)
        e.train_begin(y, H.base_margin(p, y))
        e.train_rounds(p, 1)
        e.inject_fault(after)
        err = _until_failure(lambda: e.train_rounds(p, 1))
        assert err.status == H.HB_DEVICE_FAILED and "injected fault" in str(err)
        # every later call is refused: training, the RowEngine seam, reads
        for call in (lambda: e.train_rounds(p, 1), lambda: e.read_margins(),
                     lambda: e.build(np.arange(10, dtype=np.uint32)),
                     lambda: e.train_begin(y, 0.0), lambda: e.upload(m)):
            with pytest.raises(H.HbError) as ex:
                call()
            assert ex.value.status == H.HB_REFUSED
    finally:
        e.close()


def test_fault_in_upload_and_in_row_engine_calls(data):
    x, y, p, m, want = data
    e = H.Engine()
    try:
        e.inject_fault(2)
        with pytest.raises(H.HbError) as ex:
            e.upload(m)
        assert ex.value.status == H.HB_DEVICE_FAILED
        with pytest.raises(H.HbError) as ex:
            e.upload(m)
        assert ex.value.status == H.HB_REFUSED
    finally:
        e.close()
    e = H.Engine()
    try:
        e.upload(m)
        e.load_margins(np.zeros(m.n_rows, np.float32))
        assert e.gradients(H.HB_LOSS_LOGISTIC, y)
        seg = e.begin_tree(np.arange(m.n_rows))
        e.inject_fault(0)
        with pytest.raises(H.HbError) as ex:
            e.histograms([seg])
        assert ex.value.status == H.HB_DEVICE_FAILED
        with pytest.raises(H.HbError) as ex:
            e.root_total(seg)
        assert ex.value.status == H.HB_REFUSED
    finally:
        e.close()


def test_disarmed_fault_never_fires(data):
    x, y, p, m, want = data
    e = H.Engine()
    try:
        e.inject_fault(3)
        e.inject_fault(-1)
        e.upload(m)
        nodes, ptr = e.train(p, y, 3, H.base_margin(p, y))
        assert nodes.tobytes() == want.nodes.tobytes()
    finally:
        e.close()


def test_fresh_engine_after_failures_trains_bit_exact(data):
    x, y, p, m, want = data
    got = H.train(p, y=y, rounds=3, matrix=m)
    assert _forest_bits(got) == _forest_bits(want)


def test_peer_exchange_wait_gives_up():
    """The peer-memory histogram exchange bounds every wait on another
    rank's flag by the GPU's global timer: a wait on a flag that nothing
    raises returns after the limit with the status word set (the engine
    then fails with HB_DEVICE_FAILED), and the GPU stays usable."""
    import ctypes

    st, ms = ctypes.c_uint64(), ctypes.c_double()
    assert H.lib().hb_peer_wait_probe(0, 200, ctypes.byref(st), ctypes.byref(ms)) == H.HB_OK
    assert st.value == 1
    assert 190.0 <= ms.value < 2000.0, ms.value
    x, y = synth.logistic_c2(5_003, 6, seed=3)
    H.train(H.TrainingParams(objective="binary:logistic", max_depth=3), x, y, 1)

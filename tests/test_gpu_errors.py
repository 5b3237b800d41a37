"""Error status of the kernels' bounded waits, on the GPU, without a fault.

The warp kernels stage each chain's record into shared memory with a bulk copy that completes on an
mbarrier, and wait for it at most 2^wait_log2 SM cycles.  With the test-only flag TSA_DEBUG_ARM_ONLY the
barrier is armed for the record's bytes but no copy is issued: the wait runs out with nothing in flight,
the kernel records the error and returns, and the call must return TSA_ERR_TIMEOUT (6).  The same process
then runs a normal session, which must be correct: the context stays usable."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from tests import _util
from treesa_gpu_b200 import _abi, engine

pytestmark = pytest.mark.gpu

TSA_ERR_TIMEOUT = 6
TSA_DEBUG_ARM_ONLY = 1


def _session_run_rc(net, **opts):
    L = _abi.lib()
    keep = _abi.Packed()
    o = _abi.make_options(keep, **opts)
    h = C.c_void_p()
    err = C.create_string_buffer(512)
    rc = L.tsa_session_create(C.byref(net.inst), C.byref(o), C.byref(h), err, 512)
    assert rc == 0, err.value
    try:
        rc = L.tsa_session_run(h, err, 512)
        return rc, err.value.decode()
    finally:
        L.tsa_session_destroy(h)


@pytest.mark.parametrize("kernel", ["warp", "pair"])
def test_bounded_wait_runs_out_and_the_device_stays_usable(kernel):
    rec = _util.instance("sat100")
    net = engine.Network(rec["ixs"], rec["iy"], rec["nlab"])
    onet = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
    trees = _util.start_trees(rec, 64, seed=3)
    betas = np.array([0.5, 2.0], np.float32)
    base = dict(betas=betas, niters=2, nchains=64, sc_target=24.0, order="par", seed=3, init_trees=trees,
                kernel_hint=kernel, device=0)
    rc, msg = _session_run_rc(net, wait_log2=20, debug_flags=TSA_DEBUG_ARM_ONLY, **base)
    assert rc == TSA_ERR_TIMEOUT and "timed out" in msg, (rc, msg)
    # tsa_run reports it the same way
    L = _abi.lib()
    keep = _abi.Packed()
    o = _abi.make_options(keep, wait_log2=20, debug_flags=TSA_DEBUG_ARM_ONLY, **base)
    r = _abi.Result()
    err = C.create_string_buffer(512)
    assert L.tsa_run(C.byref(net.inst), C.byref(o), C.byref(r), err, 512) == TSA_ERR_TIMEOUT
    L.tsa_result_free(C.byref(r))
    # a normal session afterwards, in the same process: bit-exact with the oracle
    s = engine.Session(net, **base)
    s.run()
    t, lab = s.chains()
    st = s.stats()
    s.close()
    ot, olab, ocnt = O.sweeps(onet, trees, betas, 2, order="par", seed=3, sc_target=24.0)
    assert (t == ot).all() and (lab[:, :, :onet.nw] == olab).all()
    assert st["proposals"] == ocnt[0] and st["accepts"] == ocnt[1]

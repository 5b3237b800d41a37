"""tsa_session_timing: where a run's time goes, as the bench's step_split reports it."""
import numpy as np
import pytest

from tests import _util
from treesa_gpu_b200 import engine

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scheme", ["indep", "pa", "trunc"])
def test_run_timing_is_consistent(scheme):
    rec = _util.instance("grid24")
    net = engine.Network(rec["ixs"], rec["iy"], rec["nlab"])
    s = engine.Session(net, betas=_util.julia_betas(0.5, 0.5, 5.0), niters=2, nchains=64, sc_target=30.0,
                       scheme=scheme, seed=4, init_trees=_util.start_trees(rec, 64, seed=4))
    s.run()
    t = s.timing()
    st = s.stats()
    rc, d = s.result()
    s.close()
    assert rc == 0 and d["valid"]
    assert t["kernel_s"] == pytest.approx(st["kernel_s"]) and t["kernel_s"] > 0
    assert t["run_s"] >= t["kernel_s"]
    assert min(t["gather_s"], t["resample_s"], t["select_s"], t["fetch_s"]) >= 0
    assert t["sent_bytes"] == 0 and t["recv_bytes"] == 0  # one GPU: no record crosses to another rank
    if scheme == "indep":
        assert t["resample_s"] == 0
    else:  # every level but the last resamples the population
        assert t["resample_s"] > 0 and t["gather_s"] > 0 and d["nresample"] == 9

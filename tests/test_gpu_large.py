"""Full-size checks of the CTA-per-chain kernel on the reference's large-lattice benchmark
(bench/results/large_compare_gpu_par.jsonl): L x L lattice, row-major path start, par order, 72 chains x 20
sweeps, betas 5:0.05:15, seed 1, pure tc (sc_target 10000).  The reference's GPU binary logged
tc 44.209 / sc 33 (L=32), 61.685 / 49 (L=48) and 78.643 / 65 (L=64), identical on RTX 6000 and H100; with the device expf
(the binary's Metropolis) this build reproduces them.  Also size-independent properties at the BASELINE
sizes: the final labels equal the labels recomputed from the final topology for every chain."""
import numpy as np
import pytest

import workloads as _instances
from tests import _util
from treesa_gpu_b200 import engine

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("L", [32, 48, 64])
def test_lattice_row_major_logged_result(L, golden):
    exp = [e for e in golden[1]["large"] if e["instance"] == f"sq{L}"][0]
    ixs, iy = _instances.sq(L)
    net = engine.Network(ixs, iy)
    tree = _instances.path_words(list(range(L * L)), L * L)[None, :]
    rc, d = engine.run(net, betas=_util.julia_betas(5.0, 0.05, 15.0), niters=20, nchains=72, sc_target=10000.0,
                       order="par", seed=1, init_trees=tree, exp_mode="device")
    assert rc == 0 and d["valid"] and d["labels_ok"]
    assert round(d["tc"], 3) == exp["tc"] and d["sc"] == exp["sc"], (d["tc"], d["sc"])


@pytest.mark.parametrize("cfg", ["c3", "c4", "c5"])
def test_baseline_configs_keep_labels_consistent(cfg):
    """Short schedules at the BASELINE sizes: every chain's labels equal the topology's."""
    import oracle as O
    if cfg == "c3":
        ixs, iy = _instances.reg3_dual(2000, 1)
        kw = dict(nchains=64, scheme="pa")
    elif cfg == "c4":
        ixs, iy = _instances.sq(64)
        kw = dict(nchains=16, scheme="indep")
    else:
        ixs, iy = _instances.grid_ksat(24, 4.26, 3, 1, seed=1)
        kw = dict(nchains=64, scheme="trunc", slicing=True, sc_target=30.0)
    net = engine.Network(ixs, iy)
    onet = O.Net(ixs, iy)
    s = engine.Session(net, betas=np.array([0.5, 2.0, 6.0], np.float32), niters=2, seed=2, **kw)
    s.run()
    t, lab = s.chains()
    rc, d = s.result()
    s.close()
    assert rc == 0 and d["valid"] and d["labels_ok"]
    for c in range(0, t.shape[0], max(1, t.shape[0] // 8)):
        assert (O.labels(onet, t[c]) == lab[c, :, :onet.nw]).all()

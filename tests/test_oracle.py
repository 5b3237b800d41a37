"""CPU pins of the oracle (oracle/tsa_oracle.cpp), the checker of the CUDA path.

* against the reference's own csrc/cpu_ref.h compiled from its sources (oracle/_ref): bit-identical final
  trees and labels, live when the harness is built, else through the SHA-256 digests recorded from it in
  tests/golden/expected.json;
* against the reference's logged end-to-end results (tests/test_python_results*.txt): every
  best-of-N (indep) row, both orders and both starts, tc to the log's 4 decimals and sc exact.
  Population annealing and truncation select on float energies that the reference computes with the
  device's log2f/exp2f; those rows are pinned on the GPU (tests/test_gpu_parity.py), here only the
  rows whose selections the host's libm reproduces are asserted (the known exceptions are listed).
"""
import os

import numpy as np
import pytest

import oracle as O
from tests import _util

CHECK_BETAS = np.array([0.2 + 0.7 * i for i in range(10)], np.float32)
NAMES = ["sat40", "sat60", "sat100", "reg3_100", "reg3_250", "lat10", "lat14", "grid24"]


def _onet(name):
    rec = _util.instance(name)
    return rec, O.Net(rec["ixs"], rec["iy"], rec["nlab"])


@pytest.mark.parametrize("order", ["par", "preorder"])
@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_cpu_ref_digest(name, order, golden):
    exp = [e for e in golden[1]["cpuref"] if e["instance"] == name and e["order"] == order][0]
    rec, net = _onet(name)
    trees = _util.start_trees(rec, 8, seed=7)
    t, lab, cnt = O.sweeps(net, trees, CHECK_BETAS, 4, order=order, seed=7, sc_target=24.0)
    assert _util.digest(t, lab) == exp["sha256"]
    assert cnt[0] == exp["proposals"] and cnt[1] == exp["accepts"]


@pytest.mark.skipif(not os.path.exists(O.CPUREF_SO), reason="reference harness not built (no reference sources)")
@pytest.mark.parametrize("order", ["par", "preorder"])
@pytest.mark.parametrize("name", ["sat60", "reg3_250", "lat14"])
def test_oracle_matches_cpu_ref_live(name, order):
    """More chains, another seed and fixed random slice sets (masking), against the live cpu_ref.h."""
    rec, net = _onet(name)
    trees = _util.start_trees(rec, 24, seed=11)
    rng = np.random.default_rng(5)
    S = np.zeros((24, net.nw), np.uint64)
    for c in range(12, 24):  # half of the chains with 6 sliced labels
        for l in rng.choice(net.nlab, 6, replace=False):
            S[c, l >> 6] |= np.uint64(1) << np.uint64(l & 63)
    betas = np.array([0.5 + 0.9 * i for i in range(8)], np.float32)
    a = O.sweeps(net, trees, betas, 3, order=order, seed=11, sc_target=18.0, S=S)
    b = O.ref_sweeps(net, trees, betas, 3, order=order, seed=11, sc_target=18.0, S=S)
    assert (a[0] == b[0]).all() and (a[1] == b[1]).all()
    assert a[2][0] == b[2][0] and a[2][1] == b[2][1]


@pytest.mark.parametrize("name", list(_util.EDGE))
def test_oracle_matches_cpu_ref_on_edge_networks(name, golden):
    """Small and degenerate networks (three tensors, an empty tensor, disconnected parts, open legs, a
    star, rings at the packed-word boundaries): the reference's own digests, both orders."""
    ixs, iy = _util.EDGE[name]
    nlab = 1 + max(l for ix in ixs for l in ix)
    net = O.Net(ixs, iy, nlab)
    trees = np.stack([O.random_tree(net.m, 3, c) for c in range(16)])
    for order in ("par", "preorder"):
        exp = [e for e in golden[1]["edge"] if e["instance"] == name and e["order"] == order][0]
        t, lab, cnt = O.sweeps(net, trees, np.array(exp["betas"], np.float32), exp["niters"], order=order,
                               seed=exp["seed"], sc_target=exp["sc_target"])
        assert _util.digest(t, lab) == exp["sha256"], order
        assert cnt[0] == exp["proposals"] and cnt[1] == exp["accepts"], order


def test_oracle_matches_cpu_ref_par_variants(golden):
    """--par-band L and --par-follow (cpu_ref.h:140-175): the reference's own digests."""
    for e in golden[1]["variants"]:
        rec, net = _onet(e["instance"])
        trees = _util.start_trees(rec, 8, seed=7)
        t, lab, cnt = O.sweeps(net, trees, CHECK_BETAS, 4, order="par", seed=7, sc_target=24.0,
                               par_band=e["par_band"], par_follow=bool(e["par_follow"]))
        assert _util.digest(t, lab) == e["sha256"], e
        assert cnt[0] == e["proposals"] and cnt[1] == e["accepts"], e


def test_oracle_matches_cpu_ref_energy_modes(golden):
    """--mode gpu / h100 (cpu_ref.h:42-80, common.h:128-162): the reference's own digests."""
    for e in golden[1]["modes"]:
        rec, net = _onet(e["instance"])
        trees = _util.start_trees(rec, 8, seed=7)
        t, lab, cnt = O.sweeps(net, trees, CHECK_BETAS, 4, order=e["order"], seed=7, sc_target=24.0, mode=e["mode"])
        assert _util.digest(t, lab) == e["sha256"], e
        assert cnt[0] == e["proposals"] and cnt[1] == e["accepts"], e


@pytest.mark.skipif(not os.path.exists(O.CPUREF_SO), reason="reference harness not built (no reference sources)")
@pytest.mark.parametrize("band,follow", [(3, True), (8, False), (0, True)])
def test_oracle_matches_cpu_ref_live_variants(band, follow):
    rec, net = _onet("reg3_100")
    trees = _util.start_trees(rec, 16, seed=3)
    betas = np.array([0.5 + 1.1 * i for i in range(6)], np.float32)
    a = O.sweeps(net, trees, betas, 3, order="par", seed=3, sc_target=16.0, par_band=band, par_follow=follow)
    b = O.ref_sweeps(net, trees, betas, 3, order="par", seed=3, sc_target=16.0, par_band=band, par_follow=follow)
    assert (a[0] == b[0]).all() and (a[1] == b[1]).all()
    assert a[2][0] == b[2][0] and a[2][1] == b[2][1]


# PA rows whose float-energy selections the host libm does not reproduce (pinned on the GPU instead)
PA_HOST_EXCEPTIONS = {("lat10", "par", "greedy"), ("lat10", "preorder", "random")}


def _rows(golden, scheme):
    return [r for r in golden[1]["e2e"] if r["scheme"] == scheme]


@pytest.mark.parametrize("scheme", ["indep", "pa"])
def test_oracle_reproduces_logged_results(scheme, golden):
    bad = []
    for r in _rows(golden, scheme):
        if scheme == "pa" and (r["instance"], r["order"], r["init"]) in PA_HOST_EXCEPTIONS:
            continue
        rec, net = _onet(r["instance"])
        kw = dict(betas=_util.julia_betas(), niters=4, nchains=128, sc_target=30.0, scheme=scheme, order=r["order"],
                  seed=1)
        if r["init"] == "greedy":
            kw["init_trees"] = _util.words(rec["tree"])[None, :]
        rc, d = O.run(net, **kw)
        if rc != 0 or d["sc"] != r["sc"] or abs(d["tc"] - r["tc"]) >= 5e-5:
            bad.append((r, d["tc"], d["sc"]))
    assert not bad, bad


def test_random_tree_and_labels_valid():
    rec, net = _onet("sat60")
    for c in range(5):
        t = O.random_tree(net.m, 1, c)
        lab = O.labels(net, t)
        assert lab.shape == (net.m - 1, net.nw)
        # the root's output labels are the open labels (none here)
        assert not lab[-1].any()
    bad = O.random_tree(net.m, 1, 0).copy()
    bad[0] = bad[1]
    with pytest.raises(ValueError):
        O.labels(net, bad)

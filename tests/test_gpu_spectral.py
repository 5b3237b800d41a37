"""The spectral start trees' GPU parts (tsa_laplacian_vectors: cuSOLVER; tsa_path_costs: own kernel) against
the host implementation in treesa_gpu_b200/spectral.py (the reference's spectral.py semantics)."""
import numpy as np
import pytest

import workloads as _instances
from tests import _util
from treesa_gpu_b200 import engine, spectral

pytestmark = pytest.mark.gpu


def _mapped(ixs, iy):
    lmap = {}
    for ix in ixs:
        for l in ix:
            lmap.setdefault(l, len(lmap))
    for l in iy:
        lmap.setdefault(l, len(lmap))
    return engine.Network([[lmap[l] for l in ix] for ix in ixs], [lmap[l] for l in iy], max(1, len(lmap)))


def _cases():
    out = []
    for name in ("sat60", "reg3_100", "lat14", "grid24"):
        rec = _util.instance(name)
        out.append((name, rec["ixs"], rec["iy"]))
    ixs, iy = _instances.sq(12)
    out.append(("sq12_open", ixs, [ixs[0][0], ixs[5][1]]))  # two open labels
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_path_costs_equal_host(case):
    name, ixs, iy = case
    net = _mapped(ixs, iy)
    rng = np.random.default_rng(1)
    m = len(ixs)
    orders = [rng.permutation(m) for _ in range(40)] + [np.arange(m), np.arange(m)[::-1]]
    tc, sc = engine.path_costs(net, np.stack(orders))
    for o, a, b in zip(orders, tc, sc):
        t0, s0 = spectral.path_cost(o.tolist(), ixs, iy)
        assert abs(a - t0) < 1e-9 and b == s0


@pytest.mark.parametrize("name", ["reg3_250", "lat14", "grid24"])
def test_laplacian_vectors_are_the_low_eigenvectors(name):
    rec = _util.instance(name)
    n, rows, cols, w = spectral.tensor_graph(rec["ixs"])
    V = engine.laplacian_vectors(n, rows, cols, w, k=3)
    L = np.zeros((n, n))
    L[rows, cols] -= w
    L[cols, rows] -= w
    L[np.arange(n), np.arange(n)] -= L.sum(1)
    lam = np.linalg.eigvalsh(L)[1:4]
    got = np.einsum("ik,ij,jk->k", V, L, V)
    assert np.allclose(V.T @ V, np.eye(3), atol=1e-8)
    assert np.allclose(got, lam, rtol=1e-7, atol=1e-9)
    assert np.linalg.norm(L @ V - V * got) < 1e-6 * max(1.0, np.abs(lam).max()) * np.sqrt(n)


@pytest.mark.parametrize("name", ["sat100", "reg3_250", "grid24"])
def test_gpu_spectral_orders_match_host(name):
    """The same search; the eigensolvers may order a degenerate eigenspace differently, so the best path
    costs are compared within a tolerance and every returned tc is the exact cost of its ordering."""
    rec = _util.instance(name)
    host = spectral.spectral_orders(rec["ixs"], rec["iy"], k=4, seed=1)
    gpu = spectral.spectral_orders(rec["ixs"], rec["iy"], k=4, seed=1, device=0)
    assert len(gpu) == len(host)
    assert gpu[0][0] <= host[0][0] + 1.0
    for tc, sc, o in gpu:
        t0, s0 = spectral.path_cost(o, rec["ixs"], rec["iy"])
        assert abs(tc - t0) < 1e-9 and sc == s0

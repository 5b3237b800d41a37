"""The public Python API on the GPU (the reference's tests/test_python.py checks, without omeco): valid
trees, tc / sc / modeled times reported by the library equal treesa_gpu_b200.trees on the returned dict,
for every scheme and start; slicing returns the tree of the sliced network; select="sc"."""
import math

import pytest

from tests import _util
import treesa_gpu_b200 as tg
from treesa_gpu_b200 import spectral, trees as tu

pytestmark = pytest.mark.gpu


def _check(tree, info, ixs, iy, m, sliced=()):
    sl = set(sliced)
    ixs_s = [[l for l in ix if l not in sl] for ix in ixs]
    assert sorted(tu.leaf_ids(tree)) == list(range(m)) and info["valid"] and info["labels_ok"]
    assert tu.recompute_outputs(tree, ixs_s, [l for l in iy if l not in sl]) == tree
    assert abs(info["tc"] - info["tc_py"]) < 1e-4 and info["sc"] == info["sc_py"]
    assert abs(math.log(info["gpu_time"]) - math.log(info["gpu_time_py"])) < 1e-5
    assert abs(math.log(info["h100_time"]) - math.log(info["h100_time_py"])) < 1e-5


@pytest.mark.parametrize("scheme", ["indep", "pa", "trunc"])
@pytest.mark.parametrize("init", ["greedy", "random", "spectral"])
@pytest.mark.parametrize("name", ["sat40", "lat10", "reg3_100"])
def test_optimize_schemes_and_starts(name, init, scheme):
    rec = _util.instance(name)
    tree, info = tg.optimize(rec["ixs"], rec["iy"], nchains=128, niters=4, sc_target=30, scheme=scheme, init=init)
    _check(tree, info, rec["ixs"], rec["iy"], rec["m"])
    assert info["scheme"] == scheme and info["init"] == init


@pytest.mark.parametrize("name,T", [("sat60", 30), ("reg3_250", 24), ("grid24", 34)])
def test_optimize_slicing(name, T):
    rec = _util.instance(name)
    tree, info = tg.optimize(rec["ixs"], rec["iy"], nchains=128, niters=3, sc_target=T, scheme="pa", slicing=True)
    _check(tree, info, rec["ixs"], rec["iy"], rec["m"], info["sliced"])
    assert info["sc"] <= T and info["nsliced"] == len(info["sliced"])
    assert abs(info["h100_time_total_py"] - info["h100_time_py"] * 2.0 ** len(info["sliced"])) < 1e-9 * info[
        "h100_time_total_py"]
    rj = tg.runner_json(tree, info)
    assert rj["sliced"] == info["sliced"] and rj["tree"] == tree


def test_optimize_tree_list_and_spectral_tcs():
    rec = _util.instance("lat14")
    so = spectral.spectral_orders(rec["ixs"], rec["iy"], k=3)
    tree, info = tg.optimize(rec["ixs"], rec["iy"], nchains=96, niters=3, sc_target=30, init="tree",
                             init_tree=[spectral.path_tree(o) for _, _, o in so] + [tg.greedy_tree(rec["ixs"], rec["iy"])])
    _check(tree, info, rec["ixs"], rec["iy"], rec["m"])
    tree2, info2 = tg.optimize(rec["ixs"], rec["iy"], nchains=96, niters=3, sc_target=30, init="spectral", spectral_k=3)
    _check(tree2, info2, rec["ixs"], rec["iy"], rec["m"])
    assert len(info2["init_tcs"]) == 3


@pytest.mark.parametrize("name,T", [("sat60", 14), ("reg3_250", 20)])
def test_select_sc(name, T):
    """indep: the selection rule changes only which snapshot is reported, so the sc-first pick has sc <= the
    default pick's; with sc_target above every sc both rules report the same tc."""
    rec = _util.instance(name)
    r = {}
    for sel in ("score", "sc"):
        tree, info = tg.optimize(rec["ixs"], rec["iy"], nchains=192, niters=3, sc_target=T, sc_weight=4.0, seed=3,
                                 select=sel)
        r[sel] = info
    assert r["sc"]["sc_py"] <= r["score"]["sc_py"]
    hi = [tg.optimize(rec["ixs"], rec["iy"], nchains=96, niters=2, sc_target=1000, seed=5, select=sel)[1]["tc_py"]
          for sel in ("score", "sc")]
    assert abs(hi[0] - hi[1]) < 1e-9


def test_optimize_multi_on_one_gpu():
    """optimize_multi with the same device several times (reference tests/test_multi.py)."""
    import random
    rng = random.Random(1)
    ixs = [rng.sample(range(80), 3) for _ in range(340)]
    tree, best, infos = tg.optimize_multi(ixs, [], gpus=[0, 0, 0], nchains=256, niters=4, sc_target=30)
    tcs = [i["tc_total_py"] for i in infos]
    assert all(i["valid"] for i in infos) and best["tc_total_py"] == min(tcs) and len(set(tcs)) > 1


def test_block_cache_reuse_keeps_results():
    """tsa_run reuses a finished call's device and pinned blocks (stale contents included): repeated calls,
    calls of another size in between and a call after tsa_release_cached_memory return the same tree."""
    from treesa_gpu_b200 import _abi
    rec = _util.instance("sat40")
    kw = dict(nchains=96, niters=3, sc_target=30, init="random", seed=5)
    t0, i0 = tg.optimize(rec["ixs"], rec["iy"], **kw)
    tg.optimize(rec["ixs"], rec["iy"], **dict(kw, nchains=200, seed=9))
    t1, i1 = tg.optimize(rec["ixs"], rec["iy"], **kw)
    assert _abi.lib().tsa_release_cached_memory() == 0
    t2, i2 = tg.optimize(rec["ixs"], rec["iy"], **kw)
    assert t0 == t1 == t2
    assert (i0["tc"], i0["sc"], i0["proposals"]) == (i1["tc"], i1["sc"], i1["proposals"]) == \
        (i2["tc"], i2["sc"], i2["proposals"])


@pytest.mark.parametrize("name", ["triangle", "empty_tensor", "disconnected", "open_legs", "star", "ring65"])
def test_optimize_edge_networks(name):
    """Small and degenerate networks end to end: a valid tree whose reported costs match trees.py."""
    ixs, iy = _util.EDGE[name]
    tree, info = tg.optimize(ixs, iy, nchains=64, niters=3, sc_target=10, init="random")
    _check(tree, info, ixs, iy, len(ixs))


def test_timeout_stops_the_run_like_the_reference_subprocess():
    """optimize(timeout=...) stops between levels and raises subprocess.TimeoutExpired, as the reference's
    subprocess.run(timeout=...) does (treesa_gpu/driver.py:305); the device stays usable."""
    import subprocess
    rec = _util.instance("sat100")
    kw = dict(nchains=512, niters=10, sc_target=20, init="random", betas=[0.01 + 0.05 * i for i in range(300)])
    with pytest.raises(subprocess.TimeoutExpired):
        tg.optimize(rec["ixs"], rec["iy"], timeout=1e-4, **kw)
    tree, info = tg.optimize(rec["ixs"], rec["iy"], timeout=600, **dict(kw, betas=kw["betas"][:20]))
    assert info["valid"] and info["nlevels"] == 20


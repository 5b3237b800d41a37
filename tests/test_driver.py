"""CPU tests of the Python side of the drop-in: tree conversions, topology-derived labels, tc / sc, spectral
start trees and the greedy start, against independent computations (the C oracle, brute force)."""
import random

import numpy as np
import pytest

import oracle as O
from tests import _util
from treesa_gpu_b200 import driver, spectral, trees


def _random_tree_dict(m, seed):
    w = O.random_tree(m, seed, 0)
    return [(int(x & 0xFFFF), int(x >> 16)) for x in w]


def test_label_map_and_betas():
    assert driver.label_map([["a", "b"], ["b", "c"]], ["d"]) == {"a": 0, "b": 1, "c": 2, "d": 3}
    b = driver.julia_betas()
    assert len(b) == 300 and b[0] == 0.01 and abs(b[-1] - 14.96) < 1e-9
    assert len(driver.julia_betas(1.0, 0.05, 15.0)) == 281
    assert len(driver.julia_betas(0.2, 0.7, 7.0)) == 10


@pytest.mark.parametrize("m", [3, 17, 300, 3000])
def test_children_dict_round_trip(m):
    rng = random.Random(m)
    ixs = [[rng.randrange(2 * m) for _ in range(2)] for _ in range(m)]
    ixs = [sorted(set(ix)) for ix in ixs]
    for seed in (3, 4):
        tree = _random_tree_dict(m, seed)
        d = driver.children_to_dict(tree, m, ixs, [])
        assert driver.check_tree(d, m)
        ch = driver.dict_to_children(d, m)
        d2 = driver.children_to_dict(ch, m, ixs, [])
        assert trees.complexity(d, ixs) == trees.complexity(d2, ixs)
    # a path tree (depth m) round-trips without recursion limits
    d = spectral.path_tree(list(range(m)))
    ch = driver.dict_to_children(d, m)
    assert ch[0] == (0, 1) and ch[-1] == (2 * m - 3, m - 1)
    assert driver.dict_to_children(driver.children_to_dict(ch, m, ixs, []), m) == ch


@pytest.mark.parametrize("name", ["sat60", "lat14", "reg3_250", "grid24"])
def test_topology_labels_and_complexity_agree_with_oracle(name):
    rec = _util.instance(name)
    net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
    for c in range(3):
        w = O.random_tree(net.m, 9, c)
        ch = [(int(x & 0xFFFF), int(x >> 16)) for x in w]
        d = driver.children_to_dict(ch, net.m, rec["ixs"], rec["iy"])
        lab = O.labels(net, w)
        # iy of internal node m+i in the dict (post-order walk of the dict == node ids of ch? no: map by walk)
        outs = {}
        st = [(2 * net.m - 2, d)]
        while st:
            v, t = st.pop()
            outs[v] = set(t["eins"]["iy"])
            l, r = ch[v - net.m]
            if l >= net.m:
                st.append((l, t["args"][0]))
            if r >= net.m:
                st.append((r, t["args"][1]))
        for v, s in outs.items():
            bits = {w_ * 64 + b for w_ in range(net.nw) for b in range(64) if int(lab[v - net.m, w_]) >> b & 1}
            assert s == bits
        tc, sc = trees.complexity(d, rec["ixs"])
        _, _, _, tch, sch = O.energy(net, w)
        assert abs(tc - tch) < 1e-9 and sc == sch


def test_path_cost_equals_complexity():
    rec = _util.instance("lat14")
    ixs, iy = rec["ixs"], [rec["ixs"][0][0]]  # one open label
    for s in range(4):
        o = list(range(len(ixs)))
        random.Random(s).shuffle(o)
        a = spectral.path_cost(o, ixs, iy)
        b = trees.complexity(trees.recompute_outputs(spectral.path_tree(o), ixs, iy), ixs)
        assert abs(a[0] - b[0]) < 1e-9 and a[1] == b[1]


@pytest.mark.parametrize("name", ["sat60", "lat14"])
def test_spectral_orders_are_exact_permutations(name):
    rec = _util.instance(name)
    so = spectral.spectral_orders(rec["ixs"], rec["iy"], k=3)
    assert len(so) == 3
    for tc, sc, o in so:
        assert sorted(o) == list(range(rec["m"]))
        d = trees.recompute_outputs(spectral.path_tree(o), rec["ixs"], rec["iy"])
        assert abs(trees.complexity(d, rec["ixs"])[0] - tc) < 1e-9
    assert [t for t, _, _ in so] == sorted(t for t, _, _ in so)


def test_spectral_sparse_solver_on_a_large_lattice():
    """Above dense_max the sparse shift-invert solver runs (64x64 lattice needs it in the benchmarks)."""
    L = 30
    lab, ixs = {}, [[] for _ in range(L * L)]
    for x in range(L):
        for y in range(L):
            v = x * L + y
            for u in ((x + 1) * L + y if x + 1 < L else None, x * L + y + 1 if y + 1 < L else None):
                if u is not None:
                    e = len(lab)
                    lab[(v, u)] = e
                    ixs[v].append(e)
                    ixs[u].append(e)
    so = spectral.spectral_orders(ixs, [], k=2, dense_max=100)
    # a good lattice ordering cuts ~L labels: far below a random order's cut
    assert so[0][1] <= 2 * L + 2


def test_greedy_tree_is_valid_and_deterministic():
    rec = _util.instance("sat60")
    d1 = driver.greedy_tree(rec["ixs"], rec["iy"])
    d2 = driver.greedy_tree(rec["ixs"], rec["iy"])
    assert driver.check_tree(d1, rec["m"]) and d1 == d2
    tc, sc = trees.complexity(d1, rec["ixs"])
    assert 40 < tc < 70


def test_time_models_match_reference_formulas():
    # spot values of the reference's model formulas (treesa_gpu/trees.py:95-140)
    g = trees.gpu_time(2, 3, 4, 5)
    ops = 2.0 ** (1 + 2 + 6 + 6 + 8)
    bits = 2.0 ** 10 + 2.0 ** 11 + 2.0 ** 9
    assert g == max(ops / 11.9e15, bits / 1.6e13) + 4e-6
    h = trees.h100_time(5, 6, 7, 8)
    a, b, c = 2.0 ** 19, 2.0 ** 20, 2.0 ** 18
    M = trees.H100_MODEL
    cc = M["cc_bit"] * (a + b + c) + M["cc_cell"] * 2.0 ** 26
    tcv = M["tc_bit"] * (a + b + c) + M["tc_pad_cell"] * 2.0 ** (5 + 6 + 7 + 8) + M["tc_out_bit"] * c
    assert abs(h - (3 * M["launch"] + 2 * (a + b) / M["perm_bw_bits"] + min(cc, tcv))) < 1e-18


def _subtrees(ch, m):
    under, out = {}, set()
    for i, (l, r) in enumerate(ch):
        s = (frozenset([l]) if l < m else under[l]) | (frozenset([r]) if r < m else under[r])
        under[m + i] = s
        out.add(s)
    return out


@pytest.mark.parametrize("name", ["sat40", "sat60", "sat100", "reg3_100", "reg3_250", "lat10", "lat14", "grid24",
                                  "grid28"])
def test_greedy_tree_equals_omeco_greedy_fixture(name):
    """The reference's tests/data/<inst>.tree files hold omeco's GreedyMethod trees (driver.py:117-122,
    the reference's greedy start); the restatement in driver._greedy_children builds the same tree: the
    same set of contracted tensor groups (child order aside)."""
    rec = _util.instance(name)
    m = rec["m"]
    ch = driver._greedy_children([list(ix) for ix in rec["ixs"]], list(rec["iy"]))
    assert _subtrees(ch, m) == _subtrees([tuple(x) for x in rec["tree"]], m)


def test_sq46_fixture_is_the_row_major_path():
    """sq46.tree is not a greedy tree: the reference's checks start sq46 from the row-major path
    (tests/run_checks.sh names those runs "sweep")."""
    import workloads as WL
    rec = _util.instance("sq46")
    assert (_util.words(rec["tree"]) == WL.path_words(list(range(rec["m"])), rec["m"])).all()

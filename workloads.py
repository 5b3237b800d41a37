"""The BASELINE workloads of bench.py, shared with the tests: seeded instances, beta schedules, start trees.

Instances (all dimension-2 labels, seeded, generated here; no dataset is read):
  sat(n, seed)            random 3-SAT with round(4.26 n) clauses, the reference's generator
                          (bench/instances.py:10-17 random_ksat with Python's random.Random, one clause
                          = rng.sample of k variables, then k sign draws), labels renumbered in order of
                          first appearance as in the reference's tests/data files; sat(60, 1) and
                          sat(100, 1) are its tests/data/sat60.txt and sat100.txt (C1, C2)
  grid_ksat(L, alpha, k, radius, seed)
                          lattice-local k-SAT, the reference's generator (bench/instances.py:19-29): a
                          clause picks a uniform site and k distinct sites of its clipped neighbourhood;
                          label = site x*L + y (C5: grid_ksat(24, 4.26, 3, 1, seed=1), 2454 clauses)
  sq(L)                   L x L open square lattice, one tensor per vertex, one label per edge
                          (bench/large_compare.py:25-36; C4: L = 64, 4096 tensors, 8064 labels)
  reg3_dual(n, seed)      random 3-regular graph by the configuration model, redrawn until it has no
                          loop or multi-edge; 3n/2 rank-2 edge tensors over vertex labels, then n rank-1
                          vertex tensors (C3: n = 2000; the reference names no generator for it)
"""
import random

import numpy as np

CONFIGS = {
    "c1": "C1: random 3-SAT n=60 m=256 (sat60), path start in clause order, order preorder, sc_target 20, "
          "64 chains, betas 0.01:0.05:15 x 10 sweeps",
    "c2": "C2: random 3-SAT n=100 m=426 (sat100), spectral start, order par, tc/sc sc_target 20, best-of-N, "
          "{n} chains per GPU, betas 0.01:0.05:15 x 10 sweeps",
    "c3": "C3: random 3-regular n=2000 (configuration model, seed 1), 3000 edge + 2000 vertex tensors, "
          "spectral start, order par, population annealing (resampling every beta), {n} chains per GPU, "
          "betas 0.01:0.05:15 x 10 sweeps",
    "c4": "C4: 64x64 open lattice (4096 tensors, 8064 labels), row-major path start, order par, best-of-N, "
          "{n} chains per GPU x 20 sweeps, betas 0.01:0.05:15",
    "c5": "C5: grid 3-SAT L=24 alpha 4.26 (2454 clauses, 576 vars, seed 1), slicing sc_target 30, greedy start, "
          "truncation selection, {n} chains per GPU, betas 0.01:0.05:15 x 10 sweeps",
}
DEFAULT_CHAINS = {"c1": 64, "c2": 4096, "c3": 1024, "c4": 72, "c5": 576}


def julia_betas(a=0.01, st=0.05, e=15.0):
    """Julia range a:st:e as float32 (the driver's expansion, then the library's float conversion)."""
    n = int(np.floor((e - a) / st + 1e-9)) + 1
    return np.array([a + i * st for i in range(n)], np.float32)


def _first_appearance(ixs):
    ids = {}
    return [[ids.setdefault(l, len(ids)) for l in ix] for ix in ixs]


def sat(n, seed=1, alpha=4.26, k=3):
    """Random k-SAT tensor network: (ixs, iy) with labels numbered by first appearance."""
    rng = random.Random(seed)
    clauses = []
    for _ in range(round(alpha * n)):
        vs = rng.sample(range(1, n + 1), k)
        for _v in vs:  # the sign draws of the clause's literals (signs do not enter the network)
            rng.random()
        clauses.append([v - 1 for v in vs])
    return _first_appearance(clauses), []


def grid_ksat(L=24, alpha=4.26, k=3, radius=1, seed=1):
    """Lattice-local k-SAT on an L x L grid of variables: (ixs, iy), label = site index."""
    rng = random.Random(seed)
    ixs = []
    for _ in range(round(alpha * L * L)):
        cx, cy = rng.randrange(L), rng.randrange(L)
        sites = [(x, y) for x in range(max(0, cx - radius), min(L, cx + radius + 1))
                 for y in range(max(0, cy - radius), min(L, cy + radius + 1))]
        pick = rng.sample(sites, k)
        for _p in pick:
            rng.random()
        ixs.append([x * L + y for x, y in pick])
    return ixs, []


def sq(L):
    """L x L open square lattice: tensor x*L+y carries the labels of its (up to 4) edges."""
    ixs = [[] for _ in range(L * L)]
    e = 0
    for x in range(L):
        for y in range(L):
            v = x * L + y
            for u in (v + L if x + 1 < L else -1, v + 1 if y + 1 < L else -1):
                if u >= 0:
                    ixs[v].append(e)
                    ixs[u].append(e)
                    e += 1
    return ixs, []


def reg3_dual(n=2000, seed=1):
    rng = np.random.default_rng(seed)
    while True:
        stubs = np.repeat(np.arange(n), 3)
        rng.shuffle(stubs)
        e = stubs.reshape(-1, 2)
        if (e[:, 0] == e[:, 1]).any():
            continue
        key = np.sort(e, axis=1)
        if len(np.unique(key[:, 0] * n + key[:, 1])) != len(key):
            continue
        break
    return [[int(a), int(b)] for a, b in e] + [[v] for v in range(n)], []


def path_words(order, m):
    """Children words of the left-deep path tree over ``order``: internal node m+i-1 joins the prefix
    with order[i]."""
    w, prev = [], int(order[0])
    for i in range(1, m):
        w.append(prev | (int(order[i]) << 16))
        prev = m + i - 1
    return np.array(w, np.uint32)


def instance(config):
    """(ixs, iy, nlab) of a BASELINE config."""
    ixs, iy = {"c1": lambda: sat(60, 1), "c2": lambda: sat(100, 1), "c3": lambda: reg3_dual(2000, 1),
               "c4": lambda: sq(64), "c5": lambda: grid_ksat(24, 4.26, 3, 1, seed=1)}[config]()
    return ixs, iy, 1 + max(l for ix in ixs for l in ix)


def workload(nchains, config="c2"):
    """The BASELINE configuration as a dict: instance record, schedule and options."""
    ixs, iy, nlab = instance(config)
    W = dict(config=config, nchains=nchains, betas=julia_betas(0.01, 0.05, 15.0), niters=10, sc_target=20.0,
             order="par", scheme="indep", seed=1, slicing=False, rec=dict(ixs=ixs, iy=iy, m=len(ixs), nlab=nlab))
    if config == "c1":
        W.update(order="preorder")
    elif config == "c3":
        W.update(scheme="pa")
    elif config == "c4":
        W.update(niters=20)
    elif config == "c5":
        W.update(scheme="trunc", slicing=True, sc_target=30.0)
    return W


def start_trees(rec, config="c2", seed=1):
    """C1: path in clause order; C4: row-major path; C5: the greedy tree; C2/C3: the 4 best spectral path
    trees.  Children words, one row per distinct start tree (chain c starts from row c % rows)."""
    from treesa_gpu_b200 import driver, engine, spectral
    m = rec["m"]
    if config in ("c1", "c4"):
        return path_words(list(range(m)), m)[None, :]
    if config == "c5":
        return engine.tree_words(driver.dict_to_children(driver.greedy_tree(rec["ixs"], rec["iy"]), m))[None, :]
    so = spectral.spectral_orders(rec["ixs"], rec["iy"], k=4, seed=seed)
    return np.stack([engine.tree_words(driver.dict_to_children(spectral.path_tree(o), m)) for _, _, o in so])

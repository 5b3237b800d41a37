"""Seeded synthetic instances of the BASELINE configurations (shared by bench.py and the tests).

C1/C2 use the reference's own sat60/sat100 instances (tests/golden, from its tests/data).  The others are
generated here with the shapes, sizes and distributions the BASELINE describes:
  sq(L)              L x L open square lattice: one tensor per vertex, one dim-2 label per edge
                     (C4: L = 64, 4096 tensors of rank 2-4, 8064 labels)
  reg3_dual(n, seed) random 3-regular graph by the configuration model, resampled until it has no loops
                     or multi-edges; each edge is a rank-2 tensor over its two vertex labels and each
                     vertex a rank-1 tensor (C3: n = 2000, 5000 tensors, 2000 labels)
  grid_ksat(L, alpha, seed)  L x L variables, round(alpha L^2) clauses; a clause picks a uniform site and
                     3 distinct variables of its 3 x 3 neighbourhood clipped at the border
                     (C5: L = 24, alpha = 4.26: 2454 clauses over 576 labels)
"""
import numpy as np


def sq(L):
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
    ixs = [[int(a), int(b)] for a, b in e] + [[v] for v in range(n)]
    return ixs, []


def grid_ksat(L=24, alpha=4.26, seed=1, k=3):
    rng = np.random.default_rng(seed)
    ixs = []
    for _ in range(int(round(alpha * L * L))):
        cx, cy = int(rng.integers(L)), int(rng.integers(L))
        cand = [x * L + y for x in range(max(0, cx - 1), min(L, cx + 2)) for y in range(max(0, cy - 1), min(L, cy + 2))]
        ixs.append(sorted(int(v) for v in rng.choice(cand, k, replace=False)))
    return ixs, []


def path_words(order, m):
    """Children words of the left-deep path tree over ``order`` (internal node m+i joins the prefix with
    order[i+1])."""
    w, prev = [], int(order[0])
    for i in range(1, m):
        w.append(prev | (int(order[i]) << 16))
        prev = m + i - 1
    return np.array(w, np.uint32)

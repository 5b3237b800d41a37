"""Spectral start trees: linear orderings of the tensors from Laplacian eigenvectors, as path trees.

The annealer's local rotations rarely change a tree's global structure, so large networks need a good start.
An ordering along a low-frequency Laplacian eigenvector of the tensor graph (spectral seriation; Fiedler)
keeps cuts small without knowing the geometry.  Same role and interface as the reference's
treesa_gpu/spectral.py (tensor_graph, laplacian_vectors, path_cost, path_tree, spectral_orders):

* tensor graph: one vertex per tensor; a label shared by k tensors adds 1/(k-1) to each of its k(k-1)/2
  pairs (weighted clique expansion of the hyperedge);
* eigenvectors 1..3 of the graph Laplacian: dense ``numpy.linalg.eigh`` up to ``dense_max`` tensors, else
  ``scipy.sparse.linalg.eigsh`` in shift-invert mode around 0;
* candidate orderings sort the tensors by a direction in the span of the eigenvectors (a sweep of angles in
  the (v1, v2) plane, refined around the best ones, plus random unit directions in (v1, v2, v3)), each in
  both directions; every candidate path tree is scored exactly by ``path_cost``; the ``k`` best distinct
  orderings are returned so that different chains can start from different trees.

The orderings depend on the eigensolver, so they are compared on tc, not as exact permutations.

With a ``device``, both numerical parts run on that GPU through libtreesa_b200.so: the eigenvectors by
cuSOLVER on the dense Laplacian (tsa_laplacian_vectors) and every batch of candidate orderings scored by
one kernel launch (tsa_path_costs); the search itself is the same.
"""
import math

import numpy as np


def tensor_graph(ixs):
    """Weighted clique expansion as (n, rows, cols, w), every unordered pair once (rows < cols)."""
    n = len(ixs)
    occ = {}
    for t, ix in enumerate(ixs):
        for l in set(ix):
            occ.setdefault(l, []).append(t)
    acc = {}
    for ts in occ.values():
        k = len(ts)
        if k < 2:
            continue
        w = 1.0 / (k - 1)
        for a in range(k):
            for b in range(a + 1, k):
                key = (ts[a], ts[b]) if ts[a] < ts[b] else (ts[b], ts[a])
                acc[key] = acc.get(key, 0.0) + w
    if not acc:
        return n, np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros(0)
    keys = np.array(list(acc.keys()), np.int64)
    return n, keys[:, 0], keys[:, 1], np.array(list(acc.values()), np.float64)


def laplacian_vectors(n, rows, cols, w, k=3, dense_max=3000, seed=0, device=None):
    """Eigenvectors 1..k (the lowest skipped) of the graph Laplacian, as the columns of an (n, k) array."""
    k = max(1, min(k, n - 2))
    if device is not None:
        from . import engine
        return engine.laplacian_vectors(n, rows, cols, w, k=k, device=device)
    deg = np.zeros(n)
    np.add.at(deg, rows, w)
    np.add.at(deg, cols, w)
    if n <= dense_max:
        L = np.zeros((n, n))
        L[rows, cols] -= w
        L[cols, rows] -= w
        L[np.arange(n), np.arange(n)] += deg
        _, V = np.linalg.eigh(L)
        return V[:, 1:k + 1]
    import scipy.sparse as sp
    import scipy.sparse.linalg as sla
    L = sp.coo_matrix((np.concatenate([-w, -w, deg]),
                       (np.concatenate([rows, cols, np.arange(n)]), np.concatenate([cols, rows, np.arange(n)]))),
                      shape=(n, n)).tocsc()
    rng = np.random.default_rng(seed)
    vals, V = sla.eigsh(L, k=k + 1, sigma=-1e-3, which="LM", v0=rng.standard_normal(n))
    o = np.argsort(vals)
    return V[:, o[1:k + 1]]


def path_cost(order, ixs, iy=()):
    """(tc, sc) in log2 of the path tree contracting the tensors in ``order`` left to right.

    Step i >= 1 contracts the prefix order[0..i-1] with tensor order[i]; its cost is the number of distinct
    labels involved: the labels alive across the cut (first occurrence before i, last at or after i) plus
    those first seen at i (step 1: the union of the first two tensors).  Output of step i: the labels
    alive across the cut after position i (open labels stay alive to the end)."""
    m = len(order)
    if m < 2:
        return 0.0, max((len(set(ix)) for ix in ixs), default=0)
    pos = np.empty(m, np.int64)
    pos[np.asarray(order, np.int64)] = np.arange(m)
    first, last = {}, {}
    for t, ix in enumerate(ixs):
        p = int(pos[t])
        for l in ix:
            if l not in first or p < first[l]:
                first[l] = p
            if l not in last or p > last[l]:
                last[l] = p
    opened = set(iy)
    labs = list(first)
    f = np.array([first[l] for l in labs], np.int64)
    la = np.array([m if l in opened else last[l] for l in labs], np.int64)
    # alive[c]: labels with first < c <= last  (crossing the cut between positions c-1 and c)
    diff = np.zeros(m + 2, np.int64)
    np.add.at(diff, f + 1, 1)
    np.add.at(diff, la + 1, -1)
    alive = np.cumsum(diff)[:m + 1]
    newc = np.bincount(f, minlength=m)
    cost = alive[1:m] + newc[1:m]
    cost[0] = len(set(ixs[order[0]]) | set(ixs[order[1]]))
    outs = alive[2:m + 1]
    sc = int(max(int(outs.max()), max(len(set(ix)) for ix in ixs)))
    cm = int(cost.max())
    tc = cm + math.log2(float(np.sum(np.exp2(cost - cm))))
    return tc, sc


def path_tree(order):
    """Left-deep tree dict contracting the tensors in ``order``."""
    t = {"tensor_index": int(order[0])}
    for i in order[1:]:
        t = {"args": [t, {"tensor_index": int(i)}]}
    return t


def _gpu_scorer(ixs, iy, device):
    """score(list of orderings) -> list of (tc, sc), one kernel launch per call."""
    from . import engine
    lmap = {}
    for ix in ixs:
        for l in ix:
            lmap.setdefault(l, len(lmap))
    for l in iy:
        lmap.setdefault(l, len(lmap))
    net = engine.Network([[lmap[l] for l in ix] for ix in ixs], [lmap[l] for l in iy], max(1, len(lmap)))

    def score(orders):
        tc, sc = engine.path_costs(net, np.array(orders, np.int32), device=device)
        return [(float(a), int(b)) for a, b in zip(tc, sc)]
    return score


def spectral_orders(ixs, iy=(), k=8, nangles=24, nrandom=24, seed=0, dense_max=3000, device=None):
    """The ``k`` best distinct spectral orderings: list of (tc, sc, order), best first.  With a ``device``
    the eigenvectors and the path costs are computed on that GPU."""
    n = len(ixs)
    if n < 3:
        return [(0.0, 0, list(range(n)))]
    n_, rows, cols, w = tensor_graph(ixs)
    V = laplacian_vectors(n, rows, cols, w, k=3, dense_max=dense_max, seed=seed, device=device)
    d = V.shape[1]
    rng = np.random.default_rng(seed)
    cands, seen = [], set()
    if device is not None:
        score = _gpu_scorer(ixs, iy, device)
    else:
        def score(orders):
            return [path_cost(o, ixs, iy) for o in orders]

    def try_dirs(vs):
        """Candidates of the directions vs (both senses each), scored together; best tc per direction."""
        todo, owner = [], []
        for j, v in enumerate(vs):
            o = np.argsort(V @ v, kind="stable")
            for oo in (o, o[::-1]):
                key = oo.tobytes()
                if key in seen:
                    continue
                seen.add(key)
                todo.append(oo.tolist())
                owner.append(j)
        best = [None] * len(vs)
        for (tc, sc), oo, j in zip(score(todo) if todo else [], todo, owner):
            cands.append((tc, sc, oo, np.array(vs[j], float)))
            best[j] = tc if best[j] is None else min(best[j], tc)
        return best

    def try_dir(v):
        return try_dirs([v])[0]

    def plane(th):
        v = np.zeros(d)
        v[0], v[1] = math.cos(th), math.sin(th)
        return v

    first = [plane(math.pi * a / nangles) for a in range(nangles)] if d >= 2 else [np.ones(1)]
    for _ in range(nrandom if d >= 3 else 0):
        v = rng.standard_normal(d)
        first.append(v / np.linalg.norm(v))
    try_dirs(first)
    if d >= 2:
        # local refinement of the angle around the three best plane directions (a small tilt orders the
        # sites inside a wavefront on lattices)
        plane_c = sorted([c for c in cands if np.count_nonzero(c[3][2:]) == 0], key=lambda c: (c[0], c[1]))
        starts = []
        for c in plane_c:
            th = math.atan2(c[3][1], c[3][0])
            if all(abs(th - t0) > 1e-9 for t0 in starts):
                starts.append(th)
            if len(starts) == 3:
                break
        for th0 in starts:
            th, step = th0, math.pi / nangles / 2
            cur = min(c[0] for c in plane_c if abs(math.atan2(c[3][1], c[3][0]) - th0) < 1e-9)
            for _ in range(8):
                moved = False
                for dth in (-step, step):
                    t = try_dir(plane(th + dth))
                    if t is not None and t < cur - 1e-9:
                        cur, th, moved = t, th + dth, True
                        break
                if not moved:
                    step /= 2
    cands.sort(key=lambda c: (c[0], c[1]))
    return [(c[0], c[1], c[2]) for c in cands[:k]]

"""Spectral start trees: tensor orderings from a low-frequency spectral embedding, as left-deep path trees.

The annealer's local rotations rarely change a tree's global structure, so large networks need a start
whose cuts are already small.  The reference draws such starts from Laplacian eigenvectors of the tensor
graph (treesa_gpu/spectral.py, called from treesa_gpu/driver.py:123-128 as ``spectral_orders(ixs, iy,
k=spectral_k)``); this module keeps that interface -- a list of ``(tc, sc, order)``, best first, whose
orders become path trees through ``path_tree`` -- and finds the orderings with its own search:

* graph: the hypergraph of the network (tensors = vertices, labels = hyperedges) expanded into cliques
  through the sparse incidence matrix H, A = H diag(w) H^T off the diagonal, with w = 2/k for a label on k
  tensors (a hyperedge adds the weight of one spanning tree, k - 1, spread over its k(k-1)/2 pairs);
* embedding: the ``nvec`` lowest non-constant Laplacian eigenvectors; each coordinate is scaled by
  1/sqrt(lambda), so that directions near the Fiedler vector dominate random draws.  Dense solver
  (``scipy.linalg.eigh`` restricted to the wanted indices) up to ``dense_max`` tensors, sparse shift-invert
  ``eigsh`` above, cuSOLVER on a device;
* search: a small evolution strategy over unit directions u of the embedding.  A direction orders the
  tensors by their projection, in both senses; generation 0 holds the coordinate axes and random
  directions, each later generation perturbs the best directions found so far with a shrinking step.
  Every generation is scored as one batch: one kernel launch on a device (``tsa_path_costs``), one
  vectorised numpy pass otherwise (``path_costs``).

Orderings depend on the eigensolver's rounding, so results are compared on tc, not as permutations.
"""
import functools
import math

import numpy as np


# ------------------------------------------------------------------------------------------------
# graph and embedding
# ------------------------------------------------------------------------------------------------
def _incidence(ixs):
    """(tensor ids, label ids) of every distinct (tensor, label) pair, and the labels (sorted) whose ids
    those are."""
    ts, ls = [], []
    for t, ix in enumerate(ixs):
        for l in sorted(set(ix)):
            ts.append(t)
            ls.append(l)
    ls = np.asarray(ls, np.int64)
    uniq, lid = np.unique(ls, return_inverse=True) if len(ls) else (np.zeros(0, np.int64), ls)
    return np.asarray(ts, np.int64), lid.astype(np.int64), uniq


def tensor_graph(ixs):
    """Weighted clique expansion of the network's hypergraph as (n, rows, cols, w), each pair once with
    rows < cols; a label shared by k >= 2 tensors adds 2/k to each of its pairs."""
    import scipy.sparse as sp
    n = len(ixs)
    ts, lid, labels = _incidence(ixs)
    nl = len(labels)
    if nl == 0:
        return n, np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros(0)
    H = sp.csr_matrix((np.ones(len(ts)), (ts, lid)), shape=(n, nl))
    k = np.asarray(H.sum(0)).ravel()
    lw = np.where(k >= 2, 2.0 / np.maximum(k, 1.0), 0.0)
    A = sp.triu(H @ sp.diags(lw) @ H.T, k=1).tocoo()
    keep = A.data > 0
    return n, A.row[keep].astype(np.int64), A.col[keep].astype(np.int64), A.data[keep].astype(np.float64)


def laplacian_vectors(n, rows, cols, w, k=3, dense_max=3000, seed=0, device=None):
    """The eigenvectors of eigenvalues 2..k+1 (ascending; the constant one skipped) of the graph
    Laplacian as the columns of an (n, k) array."""
    k = max(1, min(k, n - 2))
    if device is not None:
        from . import engine
        return engine.laplacian_vectors(n, rows, cols, w, k=k, device=device)
    import scipy.sparse as sp
    A = sp.coo_matrix((w, (rows, cols)), shape=(n, n))
    A = (A + A.T).tocsr()
    Lap = sp.diags(np.asarray(A.sum(1)).ravel()) - A
    if n <= dense_max:
        import scipy.linalg as la
        _, V = la.eigh(Lap.toarray(), subset_by_index=[1, k])
        return V
    import scipy.sparse.linalg as sla
    v0 = np.random.default_rng(seed).standard_normal(n)
    vals, V = sla.eigsh(Lap.tocsc(), k=k + 1, sigma=-1e-3, which="LM", v0=v0)
    return V[:, np.argsort(vals)[1:k + 1]]


def _rayleigh(V, rows, cols, w):
    """lambda_j = v_j^T L v_j = sum over edges of w (v_j[r] - v_j[c])^2, for each column."""
    d = V[rows] - V[cols]
    return (w[:, None] * d * d).sum(0)


# ------------------------------------------------------------------------------------------------
# path trees and their cost
# ------------------------------------------------------------------------------------------------
def path_tree(order):
    """Left-deep tree dict contracting the tensors in ``order`` left to right."""
    leaves = [{"tensor_index": int(t)} for t in order]
    return functools.reduce(lambda acc, leaf: {"args": [acc, leaf]}, leaves[1:], leaves[0])


class _PathScorer:
    """Vectorised exact (tc, sc) of the path trees of a batch of orderings on the host.

    Contraction step i (1 <= i < m) joins the prefix order[0..i-1] with tensor order[i].  With f and e a
    label's first position and its end (last position, or m when the label is open), the prefix carries
    the labels with f <= i-1 < e (at step 1 the prefix is the leaf order[0], which carries every label
    with f == 0), the tensor brings the labels with f == i in addition, and the step's output keeps the
    labels with f <= i < e.  tc = log2 sum_i 2^|step i|; sc = max(outputs, every input tensor)."""

    def __init__(self, ixs, iy=()):
        self.m = len(ixs)
        self.ts, self.lid, labels = _incidence(ixs)
        self.nl = len(labels)
        order = np.lexsort((self.ts, self.lid))
        self.occ_t = self.ts[order]
        lsorted = self.lid[order]
        self.starts = np.flatnonzero(np.r_[True, lsorted[1:] != lsorted[:-1]]) if len(lsorted) else np.zeros(0, int)
        opened = set(int(l) for l in iy)
        self.open = np.array([int(l) in opened for l in labels], bool)
        self.max_in = max((len(set(ix)) for ix in ixs), default=0)

    def __call__(self, orders):
        orders = np.atleast_2d(np.asarray(orders, np.int64))
        B, m = orders.shape
        if m < 2:
            return [(0.0, self.max_in)] * B
        if self.nl == 0:
            return [(math.log2(m - 1), self.max_in)] * B
        pos = np.empty_like(orders)
        pos[np.arange(B)[:, None], orders] = np.arange(m)[None, :]
        P = pos[:, self.occ_t]
        f = np.minimum.reduceat(P, self.starts, axis=1)
        e = np.where(self.open[None, :], m, np.maximum.reduceat(P, self.starts, axis=1))
        # live[b, c] = #{labels: f <= c < e}, by +1 at f and -1 at e, summed along the positions
        row = (np.arange(B) * (m + 1))[:, None]
        delta = np.zeros(B * (m + 1), np.int64)
        np.add.at(delta, (row + f).ravel(), 1)
        np.add.at(delta, (row + e).ravel(), -1)
        live = np.cumsum(delta.reshape(B, m + 1), axis=1)[:, :m]
        born = np.zeros(B * m, np.int64)
        np.add.at(born, (np.arange(B)[:, None] * m + f).ravel(), 1)
        born = born.reshape(B, m)
        left = live[:, :m - 1].copy()
        left[:, 0] = born[:, 0]
        step = left + born[:, 1:]
        hi = step.max(1)
        tc = hi + np.log2(np.exp2(step - hi[:, None]).sum(1))
        sc = np.maximum(live[:, 1:].max(1), self.max_in)
        return [(float(a), int(b)) for a, b in zip(tc, sc)]


def path_costs(orders, ixs, iy=()):
    """[(tc, sc)] in log2 of the path trees of a batch of orderings (host, vectorised)."""
    return _PathScorer(ixs, iy)(orders)


def path_cost(order, ixs, iy=()):
    """(tc, sc) in log2 of the path tree contracting the tensors in ``order`` left to right."""
    return _PathScorer(ixs, iy)([list(order)])[0]


def _device_scorer(ixs, iy, device):
    """score(batch of orderings) -> [(tc, sc)] by one tsa_path_costs launch."""
    from . import engine
    ids = {}
    for l in [l for ix in ixs for l in ix] + list(iy):
        ids.setdefault(l, len(ids))
    net = engine.Network([[ids[l] for l in ix] for ix in ixs], [ids[l] for l in iy], max(1, len(ids)))

    def score(orders):
        tc, sc = engine.path_costs(net, np.asarray(orders, np.int32), device=device)
        return [(float(a), int(b)) for a, b in zip(tc, sc)]
    return score


# ------------------------------------------------------------------------------------------------
# the search
# ------------------------------------------------------------------------------------------------
def spectral_orders(ixs, iy=(), k=4, nvec=6, batch=64, generations=16, nelite=6, step=0.35, seed=0,
                    dense_max=3000, device=None):
    """The ``k`` best distinct orderings found, as a list of (tc, sc, order), best first.

    nvec        eigenvectors spanning the embedding
    batch       directions per generation (each scored in both senses)
    generations rounds of the evolution strategy after generation 0
    nelite      directions kept as parents of the next generation
    step        initial perturbation size (relative to a unit direction), halved every two generations
    With a ``device`` the eigenvectors and every generation's path costs are computed on that GPU."""
    n = len(ixs)
    if n < 3:
        return [(0.0, max((len(set(ix)) for ix in ixs), default=0), list(range(n)))]
    n_, rows, cols, w = tensor_graph(ixs)
    V = laplacian_vectors(n, rows, cols, w, k=nvec, dense_max=dense_max, seed=seed, device=device)
    d = V.shape[1]
    lam = _rayleigh(V, rows, cols, w) if len(w) else np.ones(d)
    E = V / np.sqrt(np.maximum(lam, 1e-12 * max(1.0, float(lam.max()))))[None, :]
    score = _device_scorer(ixs, iy, device) if device is not None else _PathScorer(ixs, iy)
    rng = np.random.default_rng(seed)
    found = {}  # ordering bytes -> (tc, sc, serial, order, direction)

    def evaluate(dirs):
        todo, src = [], []
        for u in dirs:
            o = np.argsort(E @ u, kind="stable")
            for oo in (o, o[::-1]):
                key = oo.tobytes()
                if key not in found:
                    found[key] = None
                    todo.append(oo)
                    src.append(u)
        if not todo:
            return
        for (tc, sc), oo, u in zip(score(np.stack(todo)), todo, src):
            found[oo.tobytes()] = (tc, sc, len(found), oo, u)

    def ranked():
        return sorted((v for v in found.values() if v is not None), key=lambda c: (c[0], c[1], c[2]))

    unit = lambda x: x / max(np.linalg.norm(x), 1e-300)  # noqa: E731
    gen0 = [np.eye(d)[j] for j in range(d)]
    gen0 += [unit(rng.standard_normal(d)) for _ in range(max(0, batch - d))]
    evaluate(gen0)
    sigma = step
    for g in range(generations):
        parents = []
        for c in ranked():
            if not any(np.allclose(c[4], p) for p in parents):
                parents.append(c[4])
            if len(parents) == nelite:
                break
        kids = [unit(parents[i % len(parents)] + sigma * rng.standard_normal(d)) for i in range(batch)]
        evaluate(kids)
        if g % 2 == 1:
            sigma *= 0.5
    return [(c[0], c[1], c[3].tolist()) for c in ranked()[:k]]

"""Shared helpers of the test suite: golden fixtures and instance packing."""
import functools
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


@functools.lru_cache(None)
def golden():
    with open(os.path.join(GOLDEN, "instances.json")) as f:
        inst = json.load(f)
    with open(os.path.join(GOLDEN, "expected.json")) as f:
        exp = json.load(f)
    return inst, exp


def instance(name):
    return golden()[0][name]


def words(tree):
    t = np.asarray(tree, np.int64).reshape(-1, 2)
    return (t[:, 0] | (t[:, 1] << 16)).astype(np.uint32)


from workloads import julia_betas  # noqa: E402,F401  (Julia range a:st:e as float32)


def start_trees(rec, nchains, seed):
    """Chains 0..nchains/2-1 from the greedy tree, the rest random (the host's random_tree stream)."""
    import oracle as O
    m = rec["m"]
    g = words(rec["tree"])
    half = nchains // 2
    return np.stack([g] * half + [O.random_tree(m, seed, c) for c in range(half, nchains)])


def digest(trees, labels):
    import hashlib
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(trees, np.uint32).tobytes())
    h.update(np.ascontiguousarray(labels, np.uint64).tobytes())
    return h.hexdigest()


def ring(n):
    return [[i, (i + 1) % n] for i in range(n)], []


# small and degenerate networks, and label counts at the packed-word boundaries (1, 2, 3->4, 8 and 9->10
# words): three tensors, an empty tensor, disconnected parts (outer products), open legs, a star
EDGE = {
    "triangle": ([[0, 1], [1, 2], [2, 0]], []),
    "empty_tensor": ([[0, 1], [], [1, 2], [2, 0]], []),
    "disconnected": ([[0], [0], [1], [1], [2, 3], [3]], []),
    "open_legs": ([[0, 5], [0, 1, 6], [1, 7], [7, 5]], [5, 6]),
    "star": ([[0, 1, 2, 3], [0], [1], [2], [3]], []),
    "ring64": ring(64),
    "ring65": ring(65),
    "ring129": ring(129),
    "ring512": ring(512),
    "ring513": ring(513),
}

"""Python API of the B200 TreeSA annealer: a drop-in for the reference's ``treesa_gpu.driver``.

    from treesa_gpu_b200 import optimize
    tree, info = optimize(ixs, iy, nchains=4096, niters=10, sc_target=20, init="spectral")

``optimize`` keeps the reference's signature, defaults and output (treesa_gpu/driver.py:133-332): ``tree`` is
an omeco-format dict with internal ``iy`` recomputed from the topology, ``info`` holds every key of the
binary's JSON result plus the Python recomputations (tc_py, sc_py, gpu_time_py, h100_time_py, totals over
slices, wall, init).  Where the reference wrote temp files and spawned its CLI binary
(driver.py:215-314), this calls ``tsa_run`` of libtreesa_b200.so through ctypes; there is no fallback path.
Kernel-tuning keywords of the reference (wpb, block, lpc, coop_*, wpc, chunk_sums, wide) are accepted; they
never change a result, here or in the reference, and are ignored.  ``kernel`` keeps its meaning (anything
but "auto"/"par" selects the pre-order sweep), and the par-order variants ``par_follow`` and ``par_band``
(the CLI's --par-follow / --par-band, csrc/treesa_gpu.cu:1388-1389) run as in the reference.
"""
import heapq
import math
import subprocess
import sys
import time

import numpy as np

from . import _abi, engine, trees

DEFAULT_GPU_MODEL = dict(trees.GPU_MODEL)
DEFAULT_H100_MODEL = dict(trees.H100_MODEL)
MODE_ALIASES = {"gpu2": "h100", "tc+gpu2": "tc+h100"}
H100_KEYS = ("launch", "perm_bw_bits", "cc_bit", "cc_cell", "tc_bit", "tc_pad_cell", "tc_out_bit", "small_rank",
             "small_cell")
GPU_KEYS = ("peak_ops", "bw_bits", "m0", "n0", "k0", "launch")


# ---------------------------------------------------------------------------------------------
# instance / tree conversion (same conventions as the reference, driver.py:60-122)
# ---------------------------------------------------------------------------------------------
def label_map(ixs, iy):
    """Map arbitrary hashable labels to 0..L-1 in order of first appearance (ixs, then iy)."""
    mp = {}
    for ix in list(ixs) + [iy]:
        for l in ix:
            if l not in mp:
                mp[l] = len(mp)
    return mp


def dict_to_children(d, m):
    """omeco dict -> list of (left, right) for internal nodes m..2m-2 (post-order ids, root last)."""
    ch = []
    st = [(d, False)]
    ids = []
    while st:
        t, done = st.pop()
        if "tensor_index" in t:
            ids.append(t["tensor_index"])
            continue
        if done:
            b = ids.pop()
            a = ids.pop()
            ch.append((a, b))
            ids.append(m + len(ch) - 1)
            continue
        st.append((t, True))
        st.append((t["args"][1], False))
        st.append((t["args"][0], False))
    root = ids.pop()
    assert root == 2 * m - 2 and len(ch) == m - 1, "tree must be binary over all m tensors"
    return ch


def children_to_dict(ch, m, ixs, iy):
    """Children list (node ids, root = 2m-2) -> omeco dict with topology-derived internal iy.  Node ids
    of an annealed tree are not in post-order any more, so the dict is built by a walk from the root."""
    def node(v):
        return {"tensor_index": int(v)} if v < m else {"args": [None, None], "eins": {"ixs": [[], []], "iy": []}}
    root = node(2 * m - 2)
    st = [(2 * m - 2, root)]
    while st:
        v, d = st.pop()
        l, r = ch[v - m]
        a, b = node(l), node(r)
        d["args"] = [a, b]
        if r >= m:
            st.append((r, b))
        if l >= m:
            st.append((l, a))
    return trees.recompute_outputs(root, ixs, iy)


def check_tree(d, m):
    """Every leaf exactly once, binary."""
    return sorted(trees.leaf_ids(d)) == list(range(m))


def _greedy_children(ixs, iy):
    """Greedy pairwise contraction order (the GreedyMethod rule with alpha = 0, temperature 0): repeatedly
    contract the two tensors, among those sharing a label, whose result has the fewest labels; ties go to
    the pair of lowest (smaller id, larger id); disconnected parts are joined smallest first at the end.
    Returns (left, right) children in post-order ids."""
    m = len(ixs)
    sets = [set(ix) for ix in ixs]
    count = {}
    for s in sets:
        for l in s:
            count[l] = count.get(l, 0) + 1
    opened = set(iy)
    alive = {i: i for i in range(m)}  # tensor slot -> node id
    holders = {}
    for i, s in enumerate(sets):
        for l in s:
            holders.setdefault(l, set()).add(i)

    def out_of(a, b):
        sa, sb = sets[a], sets[b]
        o = set()
        for l in sa | sb:
            inside = (l in sa) + (l in sb)
            if l in opened or count[l] > inside:
                o.add(l)
        return o

    heap = []
    version = [0] * (2 * m)

    def push_pairs(a):
        seen = set()
        for l in sets[a]:
            for b in holders.get(l, ()):
                if b != a and b not in seen and b in alive:
                    seen.add(b)
                    x, y = (a, b) if a < b else (b, a)
                    heapq.heappush(heap, (len(out_of(x, y)), x, y, version[x], version[y]))

    for a in range(m):
        push_pairs(a)
    ch = []
    slot_next = m
    while len(alive) > 1:
        while heap:
            loss, x, y, vx, vy = heap[0]
            if x in alive and y in alive and version[x] == vx and version[y] == vy:
                break
            heapq.heappop(heap)
        if not heap:  # disconnected: join the two smallest tensors
            order = sorted(alive, key=lambda s_: (len(sets[s_]), s_))
            x, y = sorted(order[:2])
        else:
            _, x, y, _, _ = heapq.heappop(heap)
        o = out_of(x, y)
        for l in sets[x] | sets[y]:
            count[l] -= (l in sets[x]) + (l in sets[y])
            holders[l].discard(x)
            holders[l].discard(y)
        ch.append((alive.pop(x), alive.pop(y)))
        z = slot_next
        slot_next += 1
        sets.append(o)
        version.append(0)
        for l in o:
            count[l] = count.get(l, 0) + 1
            holders.setdefault(l, set()).add(z)
        alive[z] = m + len(ch) - 1
        push_pairs(z)
    return ch


def greedy_tree(ixs, iy):
    """Greedy start tree as an omeco dict.  Uses omeco's GreedyMethod when omeco is importable (the
    reference's own choice, driver.py:117-122), else the restatement in _greedy_children."""
    try:
        import omeco  # noqa: F401
    except ImportError:
        omeco = None
    if omeco is not None:
        sizes = {l: 2 for ix in ixs for l in ix}
        for l in iy:
            sizes[l] = 2
        return omeco.optimize_code(ixs, iy, sizes, omeco.GreedyMethod()).to_dict()
    m = len(ixs)
    return children_to_dict(_greedy_children([list(ix) for ix in ixs], list(iy)), m, ixs, iy)


def julia_betas(start=0.01, step=0.05, stop=15.0):
    """Julia range start:step:stop (inclusive)."""
    n = int(math.floor((stop - start) / step + 1e-9)) + 1
    return [start + i * step for i in range(n)]


def _betas32(betas):
    """The reference passes betas as text (repr of the doubles) and its binary reads them as float."""
    return np.array([float(b) for b in betas], np.float64).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# main entry point (driver.py:133-332)
# ---------------------------------------------------------------------------------------------
def optimize(ixs, iy, nchains=1024, betas=None, niters=50, sc_target=20.0, sc_weight=1.0, mode="tc",
             init="auto", seed=1, scheme="indep", order="par", kernel="auto", trunc_frac=0.25, eval_every=1,
             gpu_model=None, h100_model=None, wpb=0, block=0, lpc=32, init_tree=None, stage2_betas=None,
             stage2_niters=None, slicing=False, slice_moves=1, slice_every=1, max_slices=0, init_slices=None,
             wide=False, verbose=False, timeout=3600, device=None, coop_max=0, coop_min_units=0, coop_min=1,
             coop_full=0, coop_chunks=0, spectral_k=4, par_follow=False, par_band=0, chunk_sums=None, wpc=0,
             select="score", **old_names):
    """Run TreeSA on the GPU.  Returns (tree_dict, info); see the module docstring and the reference's
    documentation of every keyword (treesa_gpu/driver.py:138-197).

    Distributed runs (one process per GPU, chains sharded over ranks, NCCL selection) go through
    ``treesa_gpu_b200.distributed.optimize_distributed``, which calls this function with the hidden
    keywords ``_rank``, ``_world_size`` and ``_nccl_id``."""
    rank = old_names.pop("_rank", 0)
    world = old_names.pop("_world_size", 1)
    nccl_id = old_names.pop("_nccl_id", None)
    stream = old_names.pop("_stream", None)
    if old_names:
        unknown = set(old_names) - {"gpu_model2"}
        if unknown:
            raise TypeError(f"unexpected keyword arguments {sorted(unknown)}")
        h100_model = h100_model or old_names["gpu_model2"]
    mode = MODE_ALIASES.get(mode, mode)
    if mode not in ("tc", "gpu", "h100", "tc+gpu", "tc+h100"):
        raise ValueError(f"unknown mode {mode!r}")
    if select not in ("score", "sc"):
        raise ValueError(f"select must be 'score' or 'sc', got {select!r}")
    if scheme not in ("indep", "pa", "trunc"):
        raise ValueError(f"unknown scheme {scheme!r}")
    if order not in ("par", "preorder"):
        raise ValueError("order must be 'par' or 'preorder'")
    if kernel not in ("auto", "par") and order == "par":
        order = "preorder"  # reference: an explicit non-par kernel means the pre-order sweep
    if init == "auto":
        init = "greedy" if slicing else "spectral"
    if betas is None:
        betas = julia_betas(1.0, 0.05, 15.0) if init == "spectral" else julia_betas()
    gm = dict(DEFAULT_GPU_MODEL)
    if gpu_model:
        gm.update(gpu_model)
    h100m = dict(DEFAULT_H100_MODEL)
    if h100_model:
        h100m.update(h100_model)
    m = len(ixs)
    lmap = label_map(ixs, iy)
    inv = {v: k for k, v in lmap.items()}
    net = engine.Network([[lmap[l] for l in ix] for ix in ixs], [lmap[l] for l in iy], len(lmap))
    t_greedy = 0.0
    spectral_tcs = None
    init_trees = None
    if init in ("greedy", "tree", "spectral"):
        t0 = time.time()
        if init == "greedy":
            d0s = [greedy_tree(ixs, iy)]
        elif init == "spectral":
            from . import spectral as _sp
            so = _sp.spectral_orders(ixs, iy, k=spectral_k, seed=seed, device=0 if device is None else int(device))
            d0s = [_sp.path_tree(o) for _, _, o in so]
            spectral_tcs = [round(t, 4) for t, _, _ in so]
        else:
            if init_tree is None:
                raise ValueError("init='tree' needs init_tree")
            d0s = init_tree if isinstance(init_tree, (list, tuple)) else [init_tree]
        t_greedy = time.time() - t0
        init_trees = np.stack([engine.tree_words(dict_to_children(d0, m)) for d0 in d0s])
    elif init != "random":
        raise ValueError(f"unknown init {init!r}")
    opts = dict(betas=_betas32(betas), niters=niters, nchains=nchains, sc_target=sc_target, sc_weight=sc_weight,
                scheme=scheme, trunc_frac=trunc_frac, order=order, seed=seed, eval_every=eval_every,
                slicing=slicing, slice_moves=slice_moves, slice_every=slice_every, max_slices=max_slices,
                init_slices=[lmap[l] for l in (init_slices or [])], select_sc=(select == "sc"),
                init_trees=init_trees, gpu_model=[float(gm[k]) for k in GPU_KEYS],
                h100_model=[float(h100m[k]) for k in H100_KEYS], device=0 if device is None else int(device),
                verbose=verbose, rank=rank, world_size=world, nccl_id=nccl_id, stream=stream,
                par_follow=bool(par_follow), par_band=int(par_band or 0),
                mode=mode if mode in ("tc", "gpu", "h100") else "tc",
                timeout_s=float(timeout) if timeout else 0.0)
    if mode in ("tc+gpu", "tc+h100"):  # stage 2 continues the population in the model energy (driver.py:245-251)
        opts.update(betas2=_betas32(stage2_betas if stage2_betas is not None else julia_betas(1.0, 0.05, 16.0)),
                    niters2=int(stage2_niters or niters), mode2=mode.split("+")[1])
    t0 = time.time()
    try:
        rc, res = engine.run(net, **opts)
    except _abi.DeadlineError as e:  # the reference's CLI run under subprocess.run(timeout=...)
        raise subprocess.TimeoutExpired("treesa_gpu_b200.tsa_run", timeout) from e
    wall = time.time() - t0
    if rc != 0:
        raise RuntimeError(f"treesa_gpu_b200 failed ({rc}): final tree invalid or labels mismatch")
    sliced = [inv[i] for i in res["sliced"]]
    sl = set(sliced)
    ixs_s = [[l for l in ix if l not in sl] for ix in ixs] if sl else ixs
    iy_s = [l for l in iy if l not in sl]
    tree = children_to_dict(res["tree"], m, ixs_s, iy_s)
    assert check_tree(tree, m), "output tree does not contain every leaf exactly once"
    tc, sc = trees.complexity(tree, ixs_s)
    info = dict(res)
    del info["tree"]
    t1 = trees.tree_gpu_time(tree, ixs_s, gm)
    t2 = trees.tree_h100_time(tree, ixs_s, h100m)
    info.update(sliced=sliced, tc_py=tc, sc_py=sc, gpu_time_py=t1, h100_time_py=t2, tc_total_py=tc + len(sliced),
                h100_time_total_py=t2 * 2.0 ** len(sliced), wall=wall, t_greedy=t_greedy, tmpdir=None,
                init_tcs=spectral_tcs, init=init, par_follow=int(bool(par_follow) and order == "par"),
                par_band=int(par_band or 0) if order == "par" else 0)
    return tree, info


def optimize_multi(ixs, iy, gpus, seeds=None, objective=None, **kw):
    """Independent runs, one per GPU (different seeds), in parallel threads (ctypes releases the GIL);
    returns the best (tree, info) and the list of all infos (reference driver.py:335-348)."""
    import concurrent.futures as cf
    seeds = seeds or list(range(1, len(gpus) + 1))
    mode = MODE_ALIASES.get(kw.get("mode", "tc"), kw.get("mode", "tc"))
    objective = objective or ("h100" if "h100" in mode else "tc")
    key = (lambda i: i["h100_time_total_py"]) if objective == "h100" else (lambda i: i["tc_total_py"])
    with cf.ThreadPoolExecutor(max_workers=len(gpus)) as ex:
        futs = [ex.submit(optimize, ixs, iy, seed=s, device=g, **kw) for g, s in zip(gpus, seeds)]
        res = [f.result() for f in futs]
    best = min(res, key=lambda r: key(r[1]))
    return best[0], best[1], [r[1] for r in res]


def runner_json(tree, info):
    """{"tree": dict with iy on the sliced ixs, "sliced": [original labels]} for the H100 runner."""
    return {"tree": tree, "sliced": list(info.get("sliced", []))}


if __name__ == "__main__":  # smoke test: python -m treesa_gpu_b200.driver [n]  (random 3-SAT, alpha = 4.26)
    import random
    n = int(sys.argv[1]) if len(sys.argv) > 1 else 60
    rng = random.Random(1)
    ixs_, iy_ = [rng.sample(range(n), 3) for _ in range(round(4.26 * n))], []
    tree_, info_ = optimize(ixs_, iy_, nchains=512, niters=10, sc_target=30, verbose=True)
    print({k: v for k, v in info_.items() if k != "trace"})

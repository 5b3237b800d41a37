"""Generate the golden fixtures of the test suite from the reference (run where the reference's source
tree exists; the fixtures are committed and the GPU box never reads the reference).

    python tests/golden/make_golden.py [REFERENCE_ROOT] [--baseline] [--instances]

REFERENCE_ROOT defaults to $TREESA_REFERENCE, else BASELINE.json's "reference_path".  --baseline
(re)computes section (g), --instances section (h); either keeps the rest of expected.json.

Writes
  instances.json  -- instances of the reference's tests/data (binary instance format, read_instance
                     semantics) with their greedy start trees (*.tree, the omeco GreedyMethod trees of
                     the reference's tests) and, where present, the multi-tree start files (*_multi.tree)
  expected.json   -- (a) end-to-end tc/sc of the reference's logged Python test run
                     (tests/test_python_results.txt: order par; tests/test_python_results_preorder.txt:
                     order preorder; nchains 128, niters 4, sc_target 30, seed 1, betas 0.01:0.05:15);
                     (b) SHA-256 of the final trees + labels that the reference's own csrc/cpu_ref.h
                     (compiled from its sources by oracle/Makefile) produces on the run_checks.sh
                     schedule (48 chains, betas 0.2:0.7:7, 4 sweeps, sc_target 24, seed 7), chains
                     0..3 from the greedy tree, 4..7 random;
                     (c) the sq32/sq48 row-major-start results of the reference's large-network
                     benchmark log (bench/results/large_compare_gpu_par.jsonl), par order;
                     (d) as (b) in par order with the CLI's --par-band L and --par-follow variants
                     (csrc/cpu_ref.h:140-175);
                     (e) as (b) with the energy modes gpu and h100 (ref_*<1>, ref_*<2>, default model
                     constants), both orders;
                     (f) small and degenerate networks (tests/_util.EDGE: three tensors, an empty
                     tensor, disconnected parts, open legs, a star, rings at the packed-word
                     boundaries), 16 random start trees, betas 0.5/1/2/4 x 3 sweeps, sc_target 2, seed 3,
                     both orders;
                     (g) the BASELINE workloads (workloads.py) on their own schedules through cpu_ref.h:
                     C1 whole (64 chains x 300 levels x 10 sweeps, pre-order); C2 whole (4096 chains x
                     300 x 10, par, from its 4 spectral start trees, stored here), as one digest per
                     block of 64 chains; C3 / C4 / C5 at full size on a few chains over three levels of
                     the schedule (its first, middle and last beta) x the config's sweeps, C5 with a
                     fixed slice set;
                     (h) SHA-256 of the BASELINE instances that the reference's own generators build
                     (bench/instances.py sat / grid_ksat, bench/large_compare.py sq, imported from its
                     tree): C1 sat(60, 1) and C2 sat(100, 1) with labels numbered by first appearance,
                     C4 sq(64), C5 grid_ksat(24, 4.26, 3, 1, seed=1), labels = abs(literal) - 1.
"""
import hashlib
import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

INSTANCES = ["sat40", "sat60", "sat100", "reg3_100", "reg3_250", "lat10", "lat14", "grid24", "grid28", "sq46"]


def read_instance(path):
    tok = open(path).read().split()
    m, nlab = int(tok[0]), int(tok[1])
    k, ixs = 2, []
    for _ in range(m):
        n = int(tok[k])
        ixs.append([int(x) for x in tok[k + 1:k + 1 + n]])
        k += 1 + n
    ny = int(tok[k]) if k < len(tok) else 0
    iy = [int(x) for x in tok[k + 1:k + 1 + ny]]
    return m, nlab, ixs, iy


def read_trees(path, m):
    v = np.array(open(path).read().split(), np.int64).reshape(-1, 2)
    return v.reshape(-1, m - 1, 2).tolist()


def julia_betas(a, st, e):
    n = int(np.floor((e - a) / st + 1e-9)) + 1
    return [a + i * st for i in range(n)]


def tree_words(t):
    t = np.asarray(t, np.int64)
    return (t[:, 0] | (t[:, 1] << 16)).astype(np.uint32)


def dump_json(obj, path):
    """Indented JSON with every list of numbers on one line (start trees stay compact)."""
    text = json.dumps(obj, indent=1)
    text = re.sub(r"\[\s*([-\d.eE+,\s]+?)\s*\]", lambda mm: "[" + ", ".join(mm.group(1).split()).replace(",,", ",") + "]",
                  text)
    with open(path, "w") as f:
        f.write(text)


def digest(trees, labels):
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(trees, np.uint32).tobytes())
    h.update(np.ascontiguousarray(labels, np.uint64).tobytes())
    return h.hexdigest()


def baseline(ref_unused=None):
    """Section (g): the BASELINE workloads through the reference's cpu_ref.h (all host threads)."""
    import time

    import oracle as O
    import workloads as WL
    out = []
    lv = WL.julia_betas(0.01, 0.05, 15.0)
    three = [float(lv[0]), float(lv[len(lv) // 2]), float(lv[-1])]

    def run(cfg, trees, betas, niters, order, sc_target, c0=0, S=None, block=0):
        ixs, iy, nlab = WL.instance(cfg)
        net = O.Net(ixs, iy, nlab)
        t0 = time.time()
        t, l, cnt, _ = O.ref_sweeps(net, trees, np.asarray(betas, np.float32), niters, order=order, seed=1,
                                    sc_target=sc_target, c0=c0, S=S)
        e = dict(config=cfg, order=order, niters=niters, nbetas=len(betas), seed=1, sc_target=sc_target, c0=c0,
                 nchains=len(trees), proposals=int(cnt[0]), accepts=int(cnt[1]))
        if block:
            e["block"] = block
            e["sha256_blocks"] = [digest(t[b:b + block], l[b:b + block]) for b in range(0, len(trees), block)]
        else:
            e["sha256"] = digest(t, l)
        print(cfg, len(trees), "chains", f"{time.time() - t0:.1f} s", flush=True)
        return e

    # C1 whole: path start in clause order
    W1 = WL.workload(64, "c1")
    t1 = WL.start_trees(W1["rec"], "c1")
    e = run("c1", np.repeat(t1, 64, 0), lv, 10, "preorder", 20.0)
    e.update(betas="0.01:0.05:15")
    out.append(e)
    # C2 whole: 4096 chains, chain c from spectral tree c % 4
    W2 = WL.workload(4096, "c2")
    t2 = WL.start_trees(W2["rec"], "c2")
    e = run("c2", np.stack([t2[c % len(t2)] for c in range(4096)]), lv, 10, "par", 20.0, block=64)
    e.update(betas="0.01:0.05:15", start_trees=[[int(x) for x in t] for t in t2])
    out.append(e)
    # C3 / C4 / C5 at full size: a few chains, first / middle / last beta
    for cfg, nch, niters in (("c3", 8, 10), ("c4", 4, 20), ("c5", 8, 10)):
        W = WL.workload(nch, cfg)
        st = WL.start_trees(W["rec"], cfg)
        trees = np.stack([st[c % len(st)] for c in range(nch)])
        S = None
        sl = None
        if cfg == "c5":
            nlab = W["rec"]["nlab"]
            sl = sorted(int(x) for x in np.random.default_rng(5).choice(nlab, 6, replace=False))
            nw = (nlab + 63) // 64
            S1 = np.zeros(nw, np.uint64)
            for q in sl:
                S1[q >> 6] |= np.uint64(1) << np.uint64(q & 63)
            S = np.tile(S1, (nch, 1))
        e = run(cfg, trees, three, niters, "par", W["sc_target"], S=S)
        e.update(betas=three, start_trees=[[int(x) for x in t] for t in st])
        if sl:
            e["slices"] = sl
        out.append(e)
    return out


def main(ref):
    import oracle as O
    data = os.path.join(ref, "tests", "data")
    inst = {}
    for name in INSTANCES:
        m, nlab, ixs, iy = read_instance(os.path.join(data, name + ".txt"))
        rec = dict(m=m, nlab=nlab, ixs=ixs, iy=iy, tree=read_trees(os.path.join(data, name + ".tree"), m)[0])
        mp = os.path.join(data, name + "_multi.tree")
        if os.path.exists(mp):
            rec["multi"] = read_trees(mp, m)
        inst[name] = rec
    with open(os.path.join(HERE, "instances.json"), "w") as f:
        json.dump(inst, f, separators=(",", ":"))

    # (a) logged end-to-end results of the reference's Python tests
    e2e = []
    for order, fn in (("par", "test_python_results.txt"), ("preorder", "test_python_results_preorder.txt")):
        for line in open(os.path.join(ref, "tests", fn)):
            mm = re.match(r"ok\s+(\S+) (indep|pa|trunc)\s+(greedy|random) tc\s+: .* tc ([\d.]+)==([\d.]+) sc (\d+)==",
                          line)
            if mm:
                e2e.append(dict(instance=mm[1], order=order, scheme=mm[2], init=mm[3], tc=float(mm[4]),
                                sc=int(mm[6])))

    # (b) the reference's cpu_ref.h on the run_checks.sh schedule
    betas = julia_betas(0.2, 0.7, 7.0)
    cpuref = []
    for name in INSTANCES:
        rec = inst[name]
        if rec["nlab"] > 4200:
            continue
        net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
        trees = np.stack([tree_words(rec["tree"])] * 4 + [O.random_tree(net.m, 7, c) for c in range(4, 8)])
        for order in ("par", "preorder"):
            t, l, cnt, _ = O.ref_sweeps(net, trees, betas, 4, order=order, seed=7, sc_target=24.0)
            cpuref.append(dict(instance=name, order=order, betas=[0.2, 0.7, 7.0], niters=4, seed=7, sc_target=24.0,
                               nchains=8, proposals=int(cnt[0]), accepts=int(cnt[1]), sha256=digest(t, l)))

    # (d) par-order variants: band priorities and follow-up visits
    variants = []
    for name in ("sat60", "reg3_250", "lat14", "grid24"):
        rec = inst[name]
        net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
        trees = np.stack([tree_words(rec["tree"])] * 4 + [O.random_tree(net.m, 7, c) for c in range(4, 8)])
        for band, follow in ((0, 1), (2, 0), (5, 1), (16, 0)):
            t, l, cnt, _ = O.ref_sweeps(net, trees, betas, 4, order="par", seed=7, sc_target=24.0, par_band=band,
                                        par_follow=bool(follow))
            variants.append(dict(instance=name, order="par", par_band=band, par_follow=follow, betas=[0.2, 0.7, 7.0],
                                 niters=4, seed=7, sc_target=24.0, nchains=8, proposals=int(cnt[0]),
                                 accepts=int(cnt[1]), sha256=digest(t, l)))

    # (e) energy modes gpu / h100
    modes = []
    for name in ("sat60", "reg3_250", "lat14", "grid24"):
        rec = inst[name]
        net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
        trees = np.stack([tree_words(rec["tree"])] * 4 + [O.random_tree(net.m, 7, c) for c in range(4, 8)])
        for mode in ("gpu", "h100"):
            for order in ("par", "preorder"):
                t, l, cnt, _ = O.ref_sweeps(net, trees, betas, 4, order=order, seed=7, sc_target=24.0, mode=mode)
                modes.append(dict(instance=name, order=order, mode=mode, betas=[0.2, 0.7, 7.0], niters=4, seed=7,
                                  sc_target=24.0, nchains=8, proposals=int(cnt[0]), accepts=int(cnt[1]),
                                  sha256=digest(t, l)))

    # (f) small and degenerate networks
    from tests import _util
    edge = []
    ebetas = np.array([0.5, 1.0, 2.0, 4.0], np.float32)
    for name, (ixs, iy) in _util.EDGE.items():
        nlab = 1 + max(l for ix in ixs for l in ix)
        net = O.Net(ixs, iy, nlab)
        trees = np.stack([O.random_tree(net.m, 3, c) for c in range(16)])
        for order in ("par", "preorder"):
            t, l, cnt, _ = O.ref_sweeps(net, trees, ebetas, 3, order=order, seed=3, sc_target=2.0)
            edge.append(dict(instance=name, order=order, betas=[0.5, 1.0, 2.0, 4.0], niters=3, seed=3, sc_target=2.0,
                             nchains=16, proposals=int(cnt[0]), accepts=int(cnt[1]), sha256=digest(t, l)))

    # (c) sq32 / sq48 from the row-major path tree (tc / sc identical on RTX 6000 and H100)
    large = []
    for line in open(os.path.join(ref, "bench", "results", "large_compare_gpu_par.jsonl")):
        r = json.loads(line)
        if r.get("init") == "sweep" and r.get("niters") == 20 and r["instance"] in ("sq32", "sq48", "sq64"):
            large.append(dict(instance=r["instance"], nchains=r["nchains"], niters=r["niters"], beta0=r["beta0"],
                              tc=r["tc"], sc=r["sc"], order="par", scheme=r["scheme"]))
    exp = dict(e2e=e2e, cpuref=cpuref, large=large, variants=variants, modes=modes, edge=edge)
    exp["baseline"] = baseline(ref)
    exp["reference_instances"] = reference_instances(ref)
    dump_json(exp, os.path.join(HERE, "expected.json"))
    print(f"instances {len(inst)}, e2e {len(e2e)}, cpuref {len(cpuref)}, large {len(large)}, "
          f"variants {len(variants)}, modes {len(modes)}, edge {len(edge)}")


def instance_digest(ixs):
    h = hashlib.sha256()
    for ix in ixs:
        h.update((",".join(str(int(l)) for l in ix) + ";").encode())
    return h.hexdigest()


def reference_instances(ref):
    """Section (h): the reference's generators run from its source tree."""
    import importlib.util
    bench = os.path.join(ref, "bench")
    sys.path.insert(0, bench)
    try:
        def load(name):
            spec = importlib.util.spec_from_file_location("ref_" + name, os.path.join(bench, name + ".py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            return mod
        inst, lc = load("instances"), load("large_compare")
    finally:
        sys.path.remove(bench)

    def first_appearance(ixs):
        ids = {}
        return [[ids.setdefault(l, len(ids)) for l in ix] for ix in ixs]
    out = {"c1": first_appearance(inst.sat(60, seed=1)[0]), "c2": first_appearance(inst.sat(100, seed=1)[0]),
           "c4": lc.sq(64)[0], "c5": [[abs(l) - 1 for l in c] for c in inst.grid_ksat(24, 4.26, 3, 1, seed=1)[0]]}
    return {k: dict(m=len(v), sha256=instance_digest(v)) for k, v in out.items()}


def reference_root(argv):
    for a in argv:
        if not a.startswith("--"):
            return a
    if os.environ.get("TREESA_REFERENCE"):
        return os.environ["TREESA_REFERENCE"]
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        return json.load(f)["reference_path"]


if __name__ == "__main__":
    ref = reference_root(sys.argv[1:])
    if "--baseline" in sys.argv or "--instances" in sys.argv:
        path = os.path.join(HERE, "expected.json")
        with open(path) as f:
            exp = json.load(f)
        if "--baseline" in sys.argv:
            exp["baseline"] = baseline(ref)
        exp["reference_instances"] = reference_instances(ref)
        dump_json(exp, path)
    else:
        main(ref)

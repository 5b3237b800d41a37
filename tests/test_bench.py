"""bench.py host logic on the CPU: the workload definitions and the reference-GPU arm's fallback line."""
import io
import json
import types
from contextlib import redirect_stdout

import bench


def test_workloads_have_the_baseline_shapes():
    w = bench.workload(4096, "c2")
    assert w["rec"]["m"] == 426 and w["rec"]["nlab"] == 100 and len(w["betas"]) == 300 and w["niters"] == 10
    assert bench.visits_per_step(w, 2) == 300 * 10 * 4096 * 2 * 425
    w4 = bench.workload(72, "c4")
    assert w4["rec"]["m"] == 4096 and w4["niters"] == 20 and w4["order"] == "par"


def test_reference_gpu_arm_without_the_binary_prints_unavailable(monkeypatch):
    monkeypatch.setattr(bench, "REF_GPU", "/nonexistent/treesa_gpu_ref")
    out = io.StringIO()
    with redirect_stdout(out):
        rc = bench.reference_gpu_arm(bench.workload(8, "c2"), types.SimpleNamespace(steps=1, warmup=0), 0)
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    assert rc == 0 and line["impl"] == "reference_gpu" and "unavailable" in line


def test_instances_are_the_reference_generators_output(golden):
    """sat(60, 1) / sat(100, 1) are the reference's tests/data/sat60.txt / sat100.txt (C1 / C2)."""
    import workloads as WL
    for n in (60, 100):
        ixs, iy = WL.sat(n, 1)
        assert ixs == golden[0][f"sat{n}"]["ixs"] and iy == []
    ixs, iy, nlab = WL.instance("c5")
    assert len(ixs) == 2454 and nlab == 576 and all(len(set(ix)) == 3 for ix in ixs)
    ixs, iy, nlab = WL.instance("c3")
    assert len(ixs) == 5000 and nlab == 2000


def test_bench_start_trees_are_the_pinned_ones(golden):
    """The start trees bench.py builds on the host (spectral search, greedy tree) are the ones whose
    trajectories tests/golden pins against cpu_ref.h."""
    import numpy as np

    import workloads as WL
    for e in golden[1]["baseline"]:
        if "start_trees" not in e:
            continue
        W = WL.workload(e["nchains"], e["config"])
        got = WL.start_trees(W["rec"], e["config"])
        assert np.array_equal(got, np.array(e["start_trees"], np.uint32)), e["config"]


def test_oracle_reproduces_the_full_size_cpu_ref_digests(golden):
    """Our CPU restatement on C3 / C4 / C5 at full size (three levels of each schedule) against the
    digests of the reference's cpu_ref.h."""
    import numpy as np

    import oracle as O
    import workloads as WL
    from tests import _util
    for e in golden[1]["baseline"]:
        if e["config"] not in ("c3", "c4", "c5"):
            continue
        ixs, iy, nlab = WL.instance(e["config"])
        net = O.Net(ixs, iy, nlab)
        st = np.array(e["start_trees"], np.uint32)
        trees = np.stack([st[c % len(st)] for c in range(e["nchains"])])
        S = None
        if e.get("slices"):
            S1 = np.zeros(net.nw, np.uint64)
            for q in e["slices"]:
                S1[q >> 6] |= np.uint64(1) << np.uint64(q & 63)
            S = np.tile(S1, (e["nchains"], 1))
        t, lab, cnt = O.sweeps(net, trees, np.asarray(e["betas"], np.float32), e["niters"], order=e["order"],
                               seed=e["seed"], sc_target=e["sc_target"], S=S)
        assert _util.digest(t, lab) == e["sha256"], e["config"]
        assert cnt[0] == e["proposals"] and cnt[1] == e["accepts"]


def test_instances_equal_the_reference_generators_output(golden):
    """C1, C2, C4 and C5 as the reference's own generators build them (bench/instances.py sat / grid_ksat,
    bench/large_compare.py sq; digests made from the reference's tree by make_golden.py --instances)."""
    import hashlib

    import workloads as WL
    for cfg, e in golden[1]["reference_instances"].items():
        ixs, iy, nlab = WL.instance(cfg)
        h = hashlib.sha256()
        for ix in ixs:
            h.update((",".join(str(int(l)) for l in ix) + ";").encode())
        assert len(ixs) == e["m"] and h.hexdigest() == e["sha256"], cfg

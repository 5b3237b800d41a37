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

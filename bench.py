"""Benchmark of the TreeSA annealing sweep: node visits/s (BASELINE metric) on config C2.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload: random 3-SAT n=100, m=426 (the reference's tests/data/sat100.txt,
from tests/golden), spectral start (4 orderings), order par, sc_target 20, best-of-N, 4096 chains per GPU,
betas 0.01:0.05:15 (300 levels) x 10 sweeps.  One step = one whole anneal of that workload.
node visits = levels x sweeps x chains x (m-1) (reference bench/throughput.py:168).

value: all ranks' visits / max-over-ranks device time of K steps, chains resident in HBM (session reset,
       a device copy, starts each step); L2 (126 MB) flushed by a 256 MiB write between steps.
e2e:   the same metric through the C ABI (tsa_run) from host buffers: host chain init, upload, anneal,
       download and finalize inside the timed region.
--impl reference: the reference's own CPU path (csrc/cpu_ref.h built into oracle/_ref) on all host cores.
--impl reference_gpu: the reference's own CLI binary (csrc/treesa_gpu.cu compiled unchanged for sm_100a into
       oracle/_ref/treesa_gpu_ref by `make -C oracle refgpu REF=<reference>/csrc`) on the same workload and start trees, timed
       by its own kernel_s (value) and by the wall time of the process (e2e).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from workloads import CONFIGS, DEFAULT_CHAINS, start_trees, workload  # noqa: E402

METRIC = "node visits/s"
UNIT = "visits/s"


def config_dict(W, world):
    return {"workload": CONFIGS[W["config"]].format(n=W["nchains"]), "config": W["config"], "order": W["order"],
            "m": W["rec"]["m"], "labels": W["rec"]["nlab"], "chains_per_gpu": W["nchains"],
            "levels": len(W["betas"]), "sweeps_per_level": W["niters"],
            "parallelism": f"chains sharded over {world} GPU(s)",
            "l2": "flushed between steps (256 MiB write)"}


REF_GPU = os.path.join(ROOT, "oracle", "_ref", "treesa_gpu_ref")


def reference_gpu_run(W, trees, workdir, device):
    """One run of the reference's own CLI binary on the workload (its instance, multi-tree and betas file
    formats, csrc/treesa_gpu.cu:1035-1097 and :1305-1336): (its kernel seconds, process wall seconds,
    its JSON result)."""
    rec = W["rec"]
    inst, tree, betas, out = (os.path.join(workdir, f) for f in ("inst.txt", "trees.txt", "betas.txt", "out.json"))
    with open(inst, "w") as f:
        f.write(f"{rec['m']} {rec['nlab']}\n")
        for ix in rec["ixs"]:
            f.write(" ".join(str(x) for x in [len(ix)] + list(ix)) + "\n")
        f.write(" ".join(str(x) for x in [len(rec["iy"])] + list(rec["iy"])) + "\n")
    with open(tree, "w") as f:
        for t in np.atleast_2d(trees):
            for w in t:
                f.write(f"{int(w) & 0xFFFF} {int(w) >> 16}\n")
    with open(betas, "w") as f:
        f.write("\n".join(repr(float(b)) for b in W["betas"]) + "\n")
    cmd = [REF_GPU, "-i", inst, "--tree", tree, "--nchains", str(W["nchains"]), "--niters", str(W["niters"]),
           "--betas", "file:" + betas, "--mode", "tc", "--sc-target", str(W["sc_target"]), "--scheme", W["scheme"],
           "--order", W["order"], "--seed", str(W["seed"]), "--out", out, "--quiet"]
    if W["slicing"]:
        cmd.append("--slicing")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(device))
    t0 = time.time()
    p = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=1800)
    wall = time.time() - t0
    if p.returncode not in (0, 2):
        raise RuntimeError(f"reference binary failed ({p.returncode}): {p.stderr[-2000:]}")
    with open(out) as f:
        res = json.load(f)
    return float(res["kernel_s"]), wall, res


def reference_gpu_arm(W, args, device):
    import tempfile
    if not os.path.exists(REF_GPU):
        print(json.dumps({"impl": "reference_gpu", "unavailable": "oracle/_ref/treesa_gpu_ref not built "
                          "(make -C oracle refgpu REF=<reference>/csrc where the reference sources are)"}), flush=True)
        return 0
    trees = start_trees(W["rec"], config=W["config"])
    ks, ws = [], []
    with tempfile.TemporaryDirectory() as d:
        for _ in range(args.warmup):
            reference_gpu_run(W, trees, d, device)
        for _ in range(args.steps):
            k, w, res = reference_gpu_run(W, trees, d, device)
            ks.append(k)
            ws.append(w)
    vps = visits_per_step(W, 1)
    k, w = statistics.median(ks), statistics.median(ws)
    line = {"metric": METRIC, "value": vps / k, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * k, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u32", "data": "synthetic", "config": config_dict(W, 1),
            "impl": "reference_gpu", "reference_kernel": res.get("kernel"),
            "e2e": {"value": vps / w, "unit": UNIT, "note": "wall time of the reference's CLI process"},
            "best_tc": res.get("tc"), "best_sc": res.get("sc"), "valid": res.get("valid")}
    print(json.dumps(line), flush=True)
    return 0


def tc_at_wall(W, budget, device, scale="chains"):
    """BASELINE's second metric: the best tc (log2) each implementation reaches within `budget` seconds of
    wall time on the config's workload.  The schedule and start trees stay the config's; each
    implementation runs the largest population (scale "chains", in multiples of 32; best-of-N over more
    chains is the way a fixed budget buys a better expected best) or the most sweeps per beta level (scale
    "sweeps") that its calibrated wall time fits into the budget.  Ours is timed around one tsa_run call
    (host init, upload, anneal, download, finalize); the reference's GPU binary around its CLI process
    (input files written beforehand)."""
    import tempfile

    from treesa_gpu_b200 import engine
    rec = W["rec"]
    trees = start_trees(rec, config=W["config"])
    net = engine.Network(rec["ixs"], rec["iy"], rec["nlab"])

    key = "nchains" if scale == "chains" else "niters"
    unit = 32 if scale == "chains" else 1
    n0 = W[key]

    def ours(n):
        opts = dict(betas=W["betas"], niters=W["niters"], nchains=W["nchains"], sc_target=W["sc_target"],
                    order=W["order"], scheme=W["scheme"], seed=W["seed"], init_trees=trees, device=device,
                    slicing=W["slicing"])
        opts[key] = n
        t0 = time.time()
        rc, d = engine.run(net, **opts)
        return time.time() - t0, d["tc"], d["sc"]

    def ref(n, workdir):
        _, wall, res = reference_gpu_run(dict(W, **{key: n}), trees, workdir, device)
        return wall, res.get("tc"), res.get("sc")

    def fit(run):
        """Wall time is affine in the scaled quantity: two calibration runs, then runs that home in on
        [0.85, 1.0] x budget (at most five)."""
        run(n0)  # warm-up (context, caches)
        a, b = max(unit, n0 // 2 // unit * unit), 2 * n0
        ta, tb = run(a)[0], run(b)[0]
        slope = max((tb - ta) / (b - a), 1e-9)
        fixed = max(0.0, ta - a * slope)
        n = max(unit, int((budget - fixed) / slope) // unit * unit)
        best = None
        for _ in range(5):
            w, tc, sc = run(n)
            if w <= budget:
                best = dict(n=n, wall_s=w, tc=tc, sc=sc)
                if w >= 0.85 * budget:
                    break
                n = max(n + unit, int(n * (budget - fixed) / max(w - fixed, 1e-6) * 0.97) // unit * unit)
            else:
                n = max(unit, int(n * (budget - fixed) / max(w - fixed, 1e-6) * 0.95) // unit * unit)
        return dict(best or dict(n=n, wall_s=w, tc=tc, sc=sc, over_budget=True), scaled=key)

    out = {"metric": "best tc (log2) at fixed wall time", "unit": "log2 flops", "higher_is_better": False,
           "config": config_dict(W, 1), "wall_budget_s": budget, "scale": scale, "ours": fit(ours)}
    if os.path.exists(REF_GPU):
        with tempfile.TemporaryDirectory() as d:
            out["reference_gpu"] = fit(lambda n: ref(n, d))
    else:
        out["reference_gpu"] = {"unavailable": "oracle/_ref/treesa_gpu_ref not built"}
    print(json.dumps(out), flush=True)
    return 0


def visits_per_step(W, world):
    return len(W["betas"]) * W["niters"] * W["nchains"] * world * (W["rec"]["m"] - 1)


# ------------------------------------------------------------------------------------------------
# CPU: the reference's own cpu_ref.h (oracle/_ref), all host threads, bounded sample
# ------------------------------------------------------------------------------------------------
def cpu_model():
    """The host CPU's model name (/proc/cpuinfo), or the platform's processor string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_reference_rate(W, trees, target_s=12.0):
    import oracle as O
    rec = W["rec"]
    net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
    kind = "reference" if O.cpuref() is not None else "port"
    threads = os.cpu_count() or 1
    nch = 2 * threads
    start = np.stack([trees[c % len(trees)] for c in range(nch)])
    betas = np.asarray(W["betas"], np.float32)

    def run(nlev):
        if kind == "reference":
            t, l, cnt, secs = O.ref_sweeps(net, start, betas[:nlev], W["niters"], order=W["order"], seed=W["seed"],
                                           sc_target=W["sc_target"], nthreads=threads)
        else:
            t0 = time.time()
            O.sweeps(net, start, betas[:nlev], W["niters"], order=W["order"], seed=W["seed"], sc_target=W["sc_target"])
            secs = time.time() - t0
        return nch * nlev * W["niters"] * (net.m - 1), secs

    v1, s1 = run(2)
    nlev = int(max(2, min(len(betas), 2 * target_s / max(s1, 1e-3))))
    v, s = run(nlev)
    return dict(value=v / s, unit=UNIT, cores=threads, cpu_model=cpu_model(), kind=kind,
                sample=f"{nch} chains x first {nlev} of {len(betas)} levels x {W['niters']} sweeps "
                       f"({W['config']}, order {W['order']}), {s:.1f} s")


# ------------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.p = None
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", gpu_id], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_record(config="c2"):
    """The committed ncu summary of the config's sweep kernel (profiles/<config>_sweep_ncu.json): DRAM bytes
    per launch and, for the shared-memory kernels, warp instructions per node visit ({} if absent)."""
    p = os.path.join(ROOT, "profiles", f"{config}_sweep_ncu.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


def sm_count(device):
    import torch
    return torch.cuda.get_device_properties(device).multi_processor_count


# ------------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_gpu"])
    ap.add_argument("--chains", type=int, default=0, help="chains per GPU (default: the config's)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--levels", default="", help="profiling runs only: the first L beta levels (L), or levels "
                                                   "a..b-1 of the schedule (a:b)")
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS), help="BASELINE config (default c2)")
    ap.add_argument("--tc-scale", default="chains", choices=["chains", "sweeps"],
                    help="--tc-at-wall: what the budget buys, more chains (default) or more sweeps per level")
    ap.add_argument("--tc-at-wall", type=float, default=0.0,
                    help="instead of the throughput line: best tc of ours and of the reference's GPU binary within "
                         "this many seconds of wall time (BASELINE's second metric)")
    ap.add_argument("--order", default="", choices=["", "par", "preorder"],
                    help="sweep order instead of the config's (a side measurement, not a BASELINE config)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    nch = args.chains if args.chains > 0 else DEFAULT_CHAINS[args.config]
    W = workload(nch, args.config)
    if args.levels:
        a, _, b = args.levels.rpartition(":")
        W["betas"] = W["betas"][int(a or 0):int(b)]
    if args.order:
        W["order"] = args.order

    if args.impl == "reference":
        if rank != 0:
            return 0
        trees = start_trees(W["rec"], config=W["config"])
        for _ in range(args.warmup):
            cpu_reference_rate(W, trees, target_s=4.0)
        vals, t_total = [], 0.0
        for _ in range(args.steps):
            t0 = time.time()
            r = cpu_reference_rate(W, trees, target_s=8.0)
            t_total += time.time() - t0
            vals.append(r["value"])
        v = statistics.median(vals)
        cb = dict(r, value=v)
        line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
                "config": config_dict(W, 1), "impl": "reference", "cpu_baseline": cb,
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if args.impl == "reference_gpu":
        if rank != 0:
            return 0
        return reference_gpu_arm(W, args, local)

    if args.tc_at_wall > 0:
        if rank != 0 or world > 1:
            return 0
        import torch
        torch.cuda.set_device(local)
        return tc_at_wall(W, args.tc_at_wall, local, args.tc_scale)

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from treesa_gpu_b200 import engine

    rec = W["rec"]
    net = engine.Network(rec["ixs"], rec["iy"], rec["nlab"])
    trees = start_trees(rec, config=W["config"])
    nccl_id = None
    if world > 1:
        obj = [engine.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    stream = torch.cuda.current_stream()
    opts = dict(betas=W["betas"], niters=W["niters"], nchains=W["nchains"], sc_target=W["sc_target"],
                order=W["order"], scheme=W["scheme"], seed=W["seed"], init_trees=trees, device=local,
                slicing=W["slicing"],
                stream=stream.cuda_stream, rank=rank, world_size=world, nccl_id=nccl_id)
    sess = engine.Session(net, **opts)
    sess_info = sess.info()
    for _ in range(args.warmup):
        sess.reset()
        sess.run()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    gpu_id = "GPU-" + str(torch.cuda.get_device_properties(local).uuid) if hasattr(
        torch.cuda.get_device_properties(local), "uuid") else str(local)
    clk = Clocks(gpu_id)
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kernel_s, launches = 0.0, 0
    phase = dict(kernel_s=0.0, gather_s=0.0, resample_s=0.0, run_s=0.0, select_s=0.0, fetch_s=0.0, sent_bytes=0.0,
                 recv_bytes=0.0)
    tot = dict(proposals=0, accepts=0, visits=0, chunks=0, chunks_acc=0, slice_proposals=0)
    for k in range(args.steps):
        flush.zero_()
        evs[k][0].record(stream)
        sess.reset()
        sess.run()
        evs[k][1].record(stream)
        st = sess.stats()
        for key, v in sess.timing().items():
            phase[key] += v
        kernel_s += st["kernel_s"]
        launches += st["launches"]
        for key in tot:
            tot[key] += st[key]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = clk.stop()
    t_rank = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    t = torch.tensor([t_rank, kernel_s, phase["gather_s"], phase["resample_s"], phase["select_s"], phase["fetch_s"],
                      phase["sent_bytes"]], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    T, KS = float(t[0]), float(t[1])
    # where a step's time goes (max over ranks, per step): sweep kernels, energy gathers (NCCL allgather on
    # several GPUs) and population steps (record exchange) of the level-by-level schemes
    step_split = {"kernel_ms": 1e3 * KS / args.steps, "gather_ms": 1e3 * float(t[2]) / args.steps,
                  "resample_ms": 1e3 * float(t[3]) / args.steps, "select_ms": 1e3 * float(t[4]) / args.steps,
                  "fetch_ms": 1e3 * float(t[5]) / args.steps, "step_ms": 1e3 * T / args.steps,
                  "records_sent_MB_per_level_max_rank": float(t[6]) / args.steps / len(W["betas"]) / 1e6}
    rc, res = sess.result()
    sess.close()
    vps = visits_per_step(W, world)
    value = args.steps * vps / T

    # roofline of the dominant kernel (the sweep kernel).  Algorithmic bytes of the reference's algorithm
    # on packed u64 bitsets: a visit without a rule reads its children word (4 B); a proposal reads the
    # children of v and P (8 B) and five label sets (and S when slicing), and an accepted move writes
    # P's set and two children words; with chunk summaries a set costs 16 B per chunk the move touches
    # plus its summary; one whole-chain energy pass per level reads 3 sets and a children word per node.
    info = sess_info
    nw64 = (rec["nlab"] + 63) // 64
    bset = 8 * nw64
    nint = rec["m"] - 1
    P, A, V = tot["proposals"], tot["accepts"], tot["visits"]
    if info["kernel"] in (2, 4, 5, 6) and tot["chunks"] > 0:
        sum_b = 8 if nw64 >= 32 else 0
        sets = tot["chunks"] * 16 * (6 if W["slicing"] else 5) + P * 4 * sum_b
        alg = (V - P) * 4 + P * 8 + sets + tot["chunks_acc"] * 16 + A * (8 + sum_b)
    else:
        alg = (V - P) * 4 + P * (8 + (6 if W["slicing"] else 5) * bset) + A * (bset + 8)
    alg += launches * world * W["nchains"] * (nint * (3 * bset + 4) + bset)
    alg_rank = alg / world  # the counters are summed over ranks, the kernel time is the slowest rank's
    peak, peak_kind = measured_peak()
    achieved = alg_rank / KS / 1e9
    ncu = ncu_record(W["config"])
    trf = ncu.get("dram_bytes_per_launch")
    kvps = world * W["nchains"] * len(W["betas"]) * W["niters"] * nint * args.steps / KS
    hbm = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
           "traffic": trf, "peak_kind": (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                                         else "fallback")}
    kname = {1: "k_anneal_warp", 2: "k_anneal_block", 3: "k_anneal_pair", 4: "k_anneal_cluster",
             5: "k_anneal_block (global metadata)", 6: "k_anneal_block (global metadata, full scans)"}[info["kernel"]]
    extra = {"kernel": kname, "algorithmic_bytes_per_launch": alg_rank / max(1, launches),
             "kernel_visits_per_s": kvps, "kernel_s": KS, "launches_per_step": launches // args.steps}
    ipv = ncu.get("warp_inst_per_visit")
    if info["kernel"] in (1, 3) and ipv:
        # The chain lives in shared memory (HBM sees one record read and write per launch): the roof is
        # instruction issue.  achieved = warp instructions per node visit (ncu, committed) x the visits/s
        # measured here; peak = 4 schedulers x SMs x the SM clock sampled during the timed region.
        mhz = clocks["sm_mhz"] if clocks else 1965.0
        ipk = 4.0 * sm_count(local) * mhz * 1e6 / 1e9
        ach = ipv * (kvps / world) / 1e9
        roof = {"bound": "issue", "achieved": ach, "peak": ipk, "unit": "G warp-instructions/s", "frac": ach / ipk,
                "traffic": trf, "peak_kind": f"4 issue slots x {sm_count(local)} SMs x {mhz:.0f} MHz (sampled)",
                "warp_inst_per_visit": ipv, "hbm": hbm}
    else:
        roof = dict(hbm)
    roof.update(extra)

    # e2e through the C ABI with host buffers
    e2e_t, h2d, d2h = 0.0, 0, 0
    e2e_opts = dict(opts)
    for k in range(args.e2e_steps + 1 if args.e2e_steps > 0 else 0):
        if world > 1:  # the same NCCL id every call: the library reuses its communicator
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rc2, r2 = engine.run(net, **e2e_opts)
        b.record(stream)
        torch.cuda.synchronize()
        if k > 0:  # the first call is a warm-up
            e2e_t += a.elapsed_time(b) / 1e3
            h2d += r2["h2d_bytes"]
            d2h += r2["d2h_bytes"]
    te = torch.tensor([e2e_t], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = args.e2e_steps * vps / float(te[0]) if args.e2e_steps > 0 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_rate(W, trees)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * T / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
                "config": config_dict(W, world),
                "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d // max(1, args.e2e_steps),
                        "d2h_bytes_per_step": d2h // max(1, args.e2e_steps)},
                "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
                "step_split": step_split,
                "best_tc": res["tc"], "best_sc": res["sc"], "valid": bool(res["valid"] and res["labels_ok"])}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

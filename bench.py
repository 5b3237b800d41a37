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
       oracle/_ref/treesa_gpu_ref by `make -C oracle refgpu`) on the same workload and start trees, timed
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

METRIC = "node visits/s"
UNIT = "visits/s"


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


def workload(nchains, config="c2"):
    """The BASELINE configuration as (instance, schedule, options); start trees built by start_trees."""
    from tests import _instances, _util
    betas = _util.julia_betas(0.01, 0.05, 15.0)
    base = dict(config=config, nchains=nchains, betas=betas, niters=10, sc_target=20.0, order="par",
                scheme="indep", seed=1, slicing=False)
    if config in ("c1", "c2"):
        rec = _util.instance("sat60" if config == "c1" else "sat100")
        base.update(rec=rec)
        if config == "c1":
            base.update(order="preorder")
    else:
        ixs, iy = {"c3": lambda: _instances.reg3_dual(2000, 1), "c4": lambda: _instances.sq(64),
                   "c5": lambda: _instances.grid_ksat(24, 4.26, 1)}[config]()
        labs = {l for ix in ixs for l in ix}
        base.update(rec=dict(ixs=ixs, iy=iy, m=len(ixs), nlab=1 + max(labs)))
        if config == "c3":
            base.update(scheme="pa")
        elif config == "c4":
            base.update(niters=20)
        else:
            base.update(scheme="trunc", slicing=True, sc_target=30.0)
    return base


def config_dict(W, world):
    return {"workload": CONFIGS[W["config"]].format(n=W["nchains"]), "config": W["config"], "order": W["order"],
            "m": W["rec"]["m"], "labels": W["rec"]["nlab"], "chains_per_gpu": W["nchains"],
            "levels": len(W["betas"]), "sweeps_per_level": W["niters"],
            "parallelism": f"chains sharded over {world} GPU(s)",
            "l2": "flushed between steps (256 MiB write)"}


def start_trees(rec, seed=1, config="c2"):
    """C1: path tree in clause order; C4: row-major path; C5: greedy tree; C2/C3: 4 spectral path trees."""
    from tests import _instances
    from treesa_gpu_b200 import driver, engine, spectral
    m = rec["m"]
    if config in ("c1", "c4"):
        return _instances.path_words(list(range(m)), m)[None, :]
    if config == "c5":
        return engine.tree_words(driver.dict_to_children(driver.greedy_tree(rec["ixs"], rec["iy"]), m))[None, :]
    so = spectral.spectral_orders(rec["ixs"], rec["iy"], k=4, seed=seed)
    return np.stack([engine.tree_words(driver.dict_to_children(spectral.path_tree(o), m)) for _, _, o in so])


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
                          "(make -C oracle refgpu where the reference sources are)"}), flush=True)
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


def visits_per_step(W, world):
    return len(W["betas"]) * W["niters"] * W["nchains"] * world * (W["rec"]["m"] - 1)


# ------------------------------------------------------------------------------------------------
# CPU: the reference's own cpu_ref.h (oracle/_ref), all host threads, bounded sample
# ------------------------------------------------------------------------------------------------
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
    return dict(value=v / s, unit=UNIT, cores=threads, kind=kind,
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


def ncu_traffic(config="c2"):
    """DRAM bytes per launch of the sweep kernel from the committed ncu summary (None if absent)."""
    p = os.path.join(ROOT, "profiles", f"{config}_sweep_ncu.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


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
    ap.add_argument("--levels", type=int, default=0, help="first L beta levels only (profiling runs)")
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS), help="BASELINE config (default c2)")
    ap.add_argument("--order", default="", choices=["", "par", "preorder"],
                    help="sweep order instead of the config's (a side measurement, not a BASELINE config)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    nch = args.chains if args.chains > 0 else DEFAULT_CHAINS[args.config]
    W = workload(nch, args.config)
    if args.levels > 0:
        W["betas"] = W["betas"][:args.levels]
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
    tot = dict(proposals=0, accepts=0, visits=0, chunks=0, chunks_acc=0, slice_proposals=0)
    for k in range(args.steps):
        flush.zero_()
        evs[k][0].record(stream)
        sess.reset()
        sess.run()
        evs[k][1].record(stream)
        st = sess.stats()
        kernel_s += st["kernel_s"]
        launches += st["launches"]
        for key in tot:
            tot[key] += st[key]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = clk.stop()
    t_rank = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    t = torch.tensor([t_rank, kernel_s], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    T, KS = float(t[0]), float(t[1])
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
    trf = ncu_traffic(W["config"])
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": trf, "peak_kind": (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                                          else "fallback"),
            "kernel": {1: "k_anneal_warp", 2: "k_anneal_block", 3: "k_anneal_pair", 4: "k_anneal_cluster",
                       5: "k_anneal_block (global metadata)", 6: "k_anneal_block (global metadata, full scans)"}[
                           info["kernel"]],
            "algorithmic_bytes_per_launch": alg_rank / max(1, launches),
            "kernel_visits_per_s": world * W["nchains"] * len(W["betas"]) * W["niters"] * nint * args.steps / KS,
            "kernel_s": KS, "launches_per_step": launches // args.steps}

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
                "best_tc": res["tc"], "best_sc": res["sc"], "valid": bool(res["valid"] and res["labels_ok"])}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

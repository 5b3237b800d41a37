"""Host logic of the multi-GPU path on CPU: two ranks over torch.distributed (gloo, 127.0.0.1).

* chain sharding: rank r anneals global chains [r*n, (r+1)*n) with their own Philox streams, so two
  sharded ranks reproduce a single run of 2n chains exactly (checked with the CPU oracle as the engine);
* population exchange: the library's transfer plan (tsa_resample_plan), executed with real gloo
  send/recv of chain records, gives every rank exactly its ancestors' records;
* best-of-N across ranks: the (score, level, global chain) minimum over gathered per-rank bests equals the
  single-process choice.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    import oracle as O
    from tests import _util
    from tests.test_abi import _plan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        out = {}
        # (1) sharded trajectories
        rec = _util.instance("sat60")
        net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
        n = 6
        trees = np.stack([O.random_tree(net.m, 4, rank * n + c) for c in range(n)])
        betas = np.array([0.3, 1.1, 2.5], np.float32)
        t, lab, cnt = O.sweeps(net, trees, betas, 2, order="par", seed=4, c0=rank * n)
        g = [None] * WORLD
        dist.all_gather_object(g, t)
        out["sharded"] = np.concatenate(g)
        # (2) resample exchange of records over gloo
        nloc, rb = 11, 5
        rng = np.random.default_rng(123)  # same ancestors on every rank
        anc = rng.integers(0, nloc * WORLD, nloc * WORLD)
        recs = torch.arange(nloc * rb, dtype=torch.int64).reshape(nloc, rb) + rank * 1000
        src, so, si, ro, ri = _plan(anc, nloc, rank, WORLD)
        peer = 1 - rank
        send = recs[torch.as_tensor(si[so[peer]:so[peer + 1]], dtype=torch.long)].contiguous()
        recv = torch.empty((ro[peer + 1] - ro[peer], rb), dtype=torch.int64)
        ops = []
        if send.shape[0]:
            ops.append(dist.P2POp(dist.isend, send, peer))
        if recv.shape[0]:
            ops.append(dist.P2POp(dist.irecv, recv, peer))
        for r_ in dist.batch_isend_irecv(ops) if ops else []:
            r_.wait()
        pool = torch.cat([recs, recv])
        out["resampled"] = pool[torch.as_tensor(src, dtype=torch.long)].numpy()
        out["anc"] = anc
        # (3) best-of-N merge: per-rank best (score, level, chain) -> global minimum
        local = [(float(s), int(l), rank * 10 + int(c)) for s, l, c in
                 zip(rng.integers(0, 3, 4), rng.integers(0, 5, 4), range(4))]
        best = min(local)
        gb = [None] * WORLD
        dist.all_gather_object(gb, best)
        out["best"] = min(gb)
        out["all_local"] = local
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_two_rank_host_logic():
    import oracle as O
    from tests import _util
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(WORLD))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    # (1) the sharded run equals one run of all chains
    rec = _util.instance("sat60")
    net = O.Net(rec["ixs"], rec["iy"], rec["nlab"])
    trees = np.stack([O.random_tree(net.m, 4, c) for c in range(12)])
    t, _, _ = O.sweeps(net, trees, np.array([0.3, 1.1, 2.5], np.float32), 2, order="par", seed=4)
    assert (res[0]["sharded"] == t).all() and (res[1]["sharded"] == t).all()
    # (2) every rank holds its ancestors' records
    anc = res[0]["anc"]
    nloc, rb = 11, 5
    full = np.concatenate([np.arange(nloc * rb).reshape(nloc, rb) + r * 1000 for r in range(WORLD)])
    for r in range(WORLD):
        assert (res[r]["resampled"] == full[anc[r * nloc:(r + 1) * nloc]]).all()
    # (3) both ranks agree on the global best, which is the minimum over all ranks' candidates
    allc = res[0]["all_local"] + res[1]["all_local"]
    assert res[0]["best"] == res[1]["best"] == min(allc)

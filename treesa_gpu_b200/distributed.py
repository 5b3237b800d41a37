"""Multi-GPU annealing: one process per GPU (torchrun), chains sharded over ranks.

    torchrun --nproc-per-node 8 my_script.py      # in my_script: init_process_group("nccl")
    tree, info = treesa_gpu_b200.distributed.optimize_distributed(ixs, iy, nchains=4096, ...)

Rank r anneals global chains [r*nchains, (r+1)*nchains) (nchains per rank; every chain keeps the Philox
stream of its global id, so the trajectories do not depend on the number of GPUs).  Inside the library
(csrc/tsa_comm.cpp), NCCL allgathers every chain's energy after each evaluated level, so that every rank
makes the same best-of-N choice and draws the same resampling ancestors; the best chain's record is
broadcast by its owner, and resampled chains cross NVLink once per (chain, destination rank) by grouped
ncclSend/ncclRecv into the receiver's own buffer.  torch.distributed is only used to share the NCCL id.
Every rank returns the same (tree, info).
"""
import os

from . import driver, engine


_IDS = {}


def nccl_id_for_group(group=None):
    """The ncclUniqueId of this process group: created on rank 0 and broadcast once; later calls reuse it
    and with it the library's cached NCCL communicator."""
    import torch.distributed as dist
    key = id(group) if group is not None else "world"
    if key not in _IDS:
        obj = [engine.nccl_unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        _IDS[key] = obj[0]
    return _IDS[key]


def optimize_distributed(ixs, iy, group=None, device=None, **kw):
    """driver.optimize over all ranks of ``group`` (default: the world); ``nchains`` is per rank."""
    import torch
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if device is None:
        device = int(os.environ.get("LOCAL_RANK", torch.cuda.current_device()))
    if world == 1:
        return driver.optimize(ixs, iy, device=device, **kw)
    nid = nccl_id_for_group(group)
    return driver.optimize(ixs, iy, device=device, _rank=rank, _world_size=world, _nccl_id=nid, **kw)


def shard(nchains_total, world):
    """Chains per rank for a total population (weak scaling keeps nchains per rank fixed instead)."""
    if nchains_total % world:
        raise ValueError(f"{nchains_total} chains do not split evenly over {world} ranks")
    return nchains_total // world

"""Worker of tests/test_gpu_multi.py, launched by torchrun with one process per GPU.

Every rank anneals n chains of a sharded population through treesa_gpu_b200.distributed (NCCL inside the
library); rank 0 writes the results of all schemes to the JSON file named by argv[1]."""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import torch
    import torch.distributed as dist
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    from tests import _util
    from treesa_gpu_b200.distributed import optimize_distributed
    rec = _util.instance("sat60")
    out = {}
    for scheme in ("indep", "pa", "trunc"):
        for order in ("par", "preorder"):
            tree, info = optimize_distributed(rec["ixs"], rec["iy"], nchains=int(sys.argv[2]), niters=3,
                                              betas=[0.01 + 0.3 * i for i in range(20)], sc_target=30,
                                              scheme=scheme, order=order, init="random", seed=3)
            out[f"{scheme}-{order}"] = dict(tc=info["tc"], sc=info["sc"], best_chain=info["best_chain"],
                                            proposals=info["proposals"], nresample=info["nresample"],
                                            nchains=info["nchains"], valid=info["valid"],
                                            trace=[row[1:] for row in info["trace"]])
    allout = [None] * dist.get_world_size()
    dist.all_gather_object(allout, out)
    if dist.get_rank() == 0:
        with open(sys.argv[1], "w") as f:
            json.dump(allout, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

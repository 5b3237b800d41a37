"""treesa_gpu_b200: B200-native TreeSA contraction-order annealer (sm_100a), a drop-in backend for the
``treesa_gpu`` Python API.

    import treesa_gpu_b200 as treesa_gpu
    tree, info = treesa_gpu.optimize(ixs, iy, nchains=4096, niters=10, sc_target=20)

Modules: ``driver`` (optimize, tree <-> children conversion), ``trees`` (tc/sc and time models),
``spectral`` (start trees), ``engine`` (ctypes handles of libtreesa_b200.so), ``distributed``
(one process per GPU with NCCL selection).  Build the library with ``python -m treesa_gpu_b200.build``.
"""
from .driver import optimize, optimize_multi, runner_json, julia_betas, greedy_tree, dict_to_children, children_to_dict
from . import trees

__all__ = ["optimize", "optimize_multi", "runner_json", "julia_betas", "greedy_tree", "dict_to_children",
           "children_to_dict", "trees"]
__version__ = "0.1.0"

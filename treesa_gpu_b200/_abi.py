"""ctypes mirror of include/treesa_b200.h and the loader of libtreesa_b200.so.

The library is built in-tree by ``python -m treesa_gpu_b200.build`` (or ``__graft_entry__.build()``).
There is no fallback: if the shared library is missing, :func:`lib` raises.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtreesa_b200.so")
ABI_VERSION = 2

MODE = {"tc": 0, "gpu": 1, "h100": 2}
SCHEME = {"indep": 0, "pa": 1, "trunc": 2}
ORDER = {"par": 0, "preorder": 1}
SCHEME_NAME = {v: k for k, v in SCHEME.items()}
ORDER_NAME = {v: k for k, v in ORDER.items()}

ERRORS = {1: "invalid argument", 2: "invalid result tree", 3: "CUDA error", 4: "unsupported option",
          5: "out of memory", 6: "device wait timed out", 7: "NCCL error", 8: "time limit exceeded"}


class DeadlineError(RuntimeError):
    """A run stopped at its time limit (TSA_ERR_DEADLINE)."""


class Instance(C.Structure):
    _fields_ = [("m", C.c_int32), ("nlab", C.c_int32), ("ix_offsets", C.POINTER(C.c_int32)),
                ("ix_labels", C.POINTER(C.c_int32)), ("niy", C.c_int32), ("iy", C.POINTER(C.c_int32))]


class Options(C.Structure):
    _fields_ = [("betas", C.POINTER(C.c_float)), ("nbetas", C.c_int32), ("niters", C.c_int32),
                ("nchains", C.c_int32), ("mode", C.c_int32), ("sc_target", C.c_double),
                ("sc_weight", C.c_double), ("scheme", C.c_int32), ("trunc_frac", C.c_double),
                ("order", C.c_int32), ("seed", C.c_uint64), ("eval_every", C.c_int32),
                ("slicing", C.c_int32), ("slice_moves", C.c_int32), ("slice_every", C.c_int32),
                ("max_slices", C.c_int32), ("init_slices", C.POINTER(C.c_int32)), ("ninit_slices", C.c_int32),
                ("select_sc", C.c_int32), ("init_trees", C.POINTER(C.c_uint32)), ("ntrees", C.c_int32),
                ("gpu_model", C.POINTER(C.c_double)), ("h100_model", C.POINTER(C.c_double)),
                ("device", C.c_int32), ("stream", C.c_void_p), ("rank", C.c_int32), ("world_size", C.c_int32),
                ("nccl_id", C.c_void_p), ("verbose", C.c_int32), ("max_levels", C.c_int32),
                ("exp_mode", C.c_int32), ("kernel_hint", C.c_int32), ("par_follow", C.c_int32),
                ("par_band", C.c_int32), ("mode2", C.c_int32), ("niters2", C.c_int32),
                ("betas2", C.POINTER(C.c_float)), ("nbetas2", C.c_int32), ("timeout_s", C.c_float),
                ("wait_log2", C.c_int32), ("debug_flags", C.c_int32), ("reserved", C.c_int32 * 4)]


class Result(C.Structure):
    _fields_ = [("m", C.c_int32), ("tree", C.POINTER(C.c_uint32)), ("nsliced", C.c_int32),
                ("sliced", C.POINTER(C.c_int32)), ("tc", C.c_double), ("gpu_time", C.c_double),
                ("h100_time", C.c_double), ("sc", C.c_int32), ("valid", C.c_int32), ("labels_ok", C.c_int32),
                ("best_chain", C.c_int32), ("slicing", C.c_int32), ("n_repair", C.c_int32),
                ("tc_total", C.c_double), ("gpu_time_total", C.c_double), ("h100_time_total", C.c_double),
                ("t_anneal", C.c_double), ("t_init", C.c_double), ("kernel_s", C.c_double),
                ("proposals", C.c_uint64), ("accepts", C.c_uint64), ("warp_steps", C.c_uint64),
                ("node_visits", C.c_uint64), ("slice_proposals", C.c_uint64), ("slice_accepts", C.c_uint64),
                ("busy_lanes", C.c_uint64), ("nchains", C.c_int32), ("niters", C.c_int32),
                ("nlevels", C.c_int32), ("total_sweeps", C.c_int32), ("W", C.c_int32), ("nw", C.c_int32),
                ("scheme", C.c_int32), ("mode", C.c_int32), ("nresample", C.c_int32), ("order", C.c_int32),
                ("ntrace", C.c_int32), ("trace", C.POINTER(C.c_double)), ("kernel", C.c_char * 32),
                ("h2d_bytes", C.c_uint64), ("d2h_bytes", C.c_uint64), ("reserved", C.c_int32 * 12)]


TRACE_COLS = ["t", "level", "beta", "best_lcost_per_slice", "best_sc", "mean_E", "families", "mode",
              "best_nsliced", "mean_nsliced"]

EXPORTS = ["tsa_abi_version", "tsa_run", "tsa_result_free", "tsa_session_create", "tsa_session_run",
           "tsa_session_result", "tsa_session_reset", "tsa_session_destroy", "tsa_session_stats", "tsa_session_timing",
           "tsa_session_energies", "tsa_session_chains", "tsa_nccl_unique_id", "tsa_session_info",
           "tsa_resample", "tsa_resample_noalloc", "tsa_release_cached_memory", "tsa_abi_sizes"]


class Packed:
    """Owns the numpy buffers behind an Instance / Options pair (ctypes keeps raw pointers only)."""

    def __init__(self):
        self.keep = []

    def arr(self, a, dtype, ctype):
        a = np.ascontiguousarray(np.asarray(a, dtype=dtype))
        self.keep.append(a)
        return a.ctypes.data_as(C.POINTER(ctype)), a


def pack_instance(ixs_ids, iy_ids, nlab, keep):
    """ixs_ids: list of lists of label ids 0..nlab-1."""
    off = np.zeros(len(ixs_ids) + 1, np.int32)
    off[1:] = np.cumsum([len(ix) for ix in ixs_ids])
    flat = np.array([l for ix in ixs_ids for l in ix], np.int32) if off[-1] else np.zeros(1, np.int32)
    inst = Instance()
    inst.m = len(ixs_ids)
    inst.nlab = nlab
    inst.ix_offsets, _ = keep.arr(off, np.int32, C.c_int32)
    inst.ix_labels, _ = keep.arr(flat, np.int32, C.c_int32)
    iyv = np.array(list(iy_ids) or [0], np.int32)
    inst.niy = len(iy_ids)
    inst.iy, _ = keep.arr(iyv, np.int32, C.c_int32)
    return inst


def make_options(keep, betas, niters, nchains, sc_target=20.0, sc_weight=1.0, scheme="indep", trunc_frac=0.25,
                 order="par", seed=1, eval_every=1, slicing=False, slice_moves=1, slice_every=1, max_slices=0,
                 init_slices=(), select_sc=False, init_trees=None, gpu_model=None, h100_model=None, device=0,
                 stream=None, rank=0, world_size=1, nccl_id=None, verbose=False, max_levels=0, mode="tc",
                 exp_mode="host", kernel_hint=0, par_follow=False, par_band=0, betas2=None, niters2=0, mode2="gpu",
                 timeout_s=0.0, wait_log2=0, debug_flags=0):
    o = Options()
    o.betas, _ = keep.arr(np.asarray(betas, np.float32), np.float32, C.c_float)
    o.nbetas = len(betas)
    o.niters = int(niters)
    o.nchains = int(nchains)
    o.mode = MODE[mode]
    o.sc_target = float(sc_target)
    o.sc_weight = float(sc_weight)
    o.scheme = SCHEME[scheme]
    o.trunc_frac = float(trunc_frac)
    o.order = ORDER[order]
    o.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    o.eval_every = int(eval_every)
    o.slicing = int(bool(slicing))
    o.slice_moves = int(slice_moves)
    o.slice_every = int(slice_every)
    o.max_slices = int(max_slices)
    sl = list(init_slices or [])
    o.init_slices, _ = keep.arr(np.array(sl or [0], np.int32), np.int32, C.c_int32)
    o.ninit_slices = len(sl)
    o.select_sc = int(bool(select_sc))
    if init_trees is not None and len(init_trees):
        t = np.ascontiguousarray(np.asarray(init_trees, np.uint32))
        o.init_trees, _ = keep.arr(t.ravel(), np.uint32, C.c_uint32)
        o.ntrees = t.shape[0] if t.ndim == 2 else 1
    if gpu_model is not None:
        o.gpu_model, _ = keep.arr(np.asarray(gpu_model, np.float64), np.float64, C.c_double)
    if h100_model is not None:
        o.h100_model, _ = keep.arr(np.asarray(h100_model, np.float64), np.float64, C.c_double)
    o.device = int(device)
    o.stream = stream
    o.rank = int(rank)
    o.world_size = int(world_size)
    if nccl_id is not None:
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        keep.keep.append(buf)
        o.nccl_id = C.cast(buf, C.c_void_p)
    o.verbose = int(bool(verbose))
    o.max_levels = int(max_levels)
    o.exp_mode = {"host": 0, "device": 1}[exp_mode]
    o.kernel_hint = {0: 0, 1: 1, 2: 2, 3: 3, 4: 4, "auto": 0, "warp": 1, "block": 2, "pair": 3,
                     "cta_pair": 4}[kernel_hint]
    o.par_follow = int(bool(par_follow))
    o.par_band = int(par_band)
    if betas2 is not None and len(betas2):
        o.betas2, _ = keep.arr(np.asarray(betas2, np.float32), np.float32, C.c_float)
        o.nbetas2 = len(betas2)
        o.niters2 = int(niters2 or 0)
        o.mode2 = MODE[mode2]
    o.timeout_s = float(timeout_s or 0.0)
    o.wait_log2 = int(wait_log2)
    o.debug_flags = int(debug_flags)
    return o


def result_to_dict(r):
    """tsa_result -> the reference's JSON dict (csrc/treesa_gpu.cu:1896-1919) plus the tree list."""
    nint = r.m - 1
    tree = [[int(w & 0xFFFF), int(w >> 16)] for w in np.ctypeslib.as_array(r.tree, (nint,))] if nint > 0 else []
    sliced = [int(x) for x in np.ctypeslib.as_array(r.sliced, (r.nsliced,))] if r.nsliced > 0 else []
    trace = (np.ctypeslib.as_array(r.trace, (r.ntrace * 10,)).reshape(r.ntrace, 10).tolist()
             if r.ntrace > 0 else [])

    def num(x):
        return None if not np.isfinite(x) else float(x)

    d = dict(tc=float(r.tc), sc=int(r.sc), gpu_time=num(r.gpu_time), h100_time=num(r.h100_time),
             valid=bool(r.valid), labels_ok=bool(r.labels_ok), best_chain=int(r.best_chain),
             slicing=bool(r.slicing), nsliced=int(r.nsliced), n_repair=int(r.n_repair), tc_total=float(r.tc_total),
             gpu_time_total=num(r.gpu_time_total), h100_time_total=num(r.h100_time_total), sliced=sliced,
             t_anneal=float(r.t_anneal), t_init=float(r.t_init), kernel_s=float(r.kernel_s),
             proposals=int(r.proposals), accepts=int(r.accepts), warp_steps=int(r.warp_steps),
             node_visits=int(r.node_visits), slice_proposals=int(r.slice_proposals),
             slice_accepts=int(r.slice_accepts), busy_lanes=int(r.busy_lanes), order=ORDER_NAME.get(r.order, "par"),
             nchains=int(r.nchains), niters=int(r.niters), nlevels=int(r.nlevels), total_sweeps=int(r.total_sweeps),
             W=int(r.W), nw=int(r.nw), kernel=r.kernel.decode(), scheme=SCHEME_NAME.get(r.scheme, "indep"),
             mode=int(r.mode), nresample=int(r.nresample), trace_cols=list(TRACE_COLS), trace=trace, tree=tree,
             h2d_bytes=int(r.h2d_bytes), d2h_bytes=int(r.d2h_bytes))
    return d


_LIB = None


def lib():
    """The loaded libtreesa_b200.so (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} not built: run `python -m treesa_gpu_b200.build` (needs nvcc)")
    L = C.CDLL(LIB_PATH)
    L.tsa_abi_version.restype = C.c_int
    L.tsa_run.argtypes = [C.POINTER(Instance), C.POINTER(Options), C.POINTER(Result), C.c_char_p, C.c_size_t]
    L.tsa_run.restype = C.c_int
    L.tsa_result_free.argtypes = [C.POINTER(Result)]
    L.tsa_result_free.restype = None
    L.tsa_session_create.argtypes = [C.POINTER(Instance), C.POINTER(Options), C.POINTER(C.c_void_p), C.c_char_p,
                                     C.c_size_t]
    L.tsa_session_run.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    L.tsa_session_result.argtypes = [C.c_void_p, C.POINTER(Result), C.c_char_p, C.c_size_t]
    L.tsa_session_reset.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    L.tsa_session_destroy.argtypes = [C.c_void_p]
    L.tsa_session_destroy.restype = None
    L.tsa_session_stats.argtypes = [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_double)]
    L.tsa_session_timing.argtypes = [C.c_void_p, C.POINTER(C.c_double)]
    L.tsa_session_energies.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int32),
                                       C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
    L.tsa_session_chains.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.c_char_p,
                                     C.c_size_t]
    L.tsa_nccl_unique_id.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    L.tsa_release_cached_memory.argtypes = []
    L.tsa_abi_sizes.argtypes = [C.POINTER(C.c_int32)]
    L.tsa_session_info.argtypes = [C.c_void_p, C.POINTER(C.c_int32)]
    L.tsa_resample.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int32, C.c_uint32, C.c_void_p, C.c_char_p,
                               C.c_size_t]
    L.tsa_resample_noalloc.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int32, C.c_uint32, C.c_void_p,
                                       C.c_char_p, C.c_size_t]
    L.tsa_laplacian_vectors.argtypes = [C.c_int32, C.c_int32, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                        C.POINTER(C.c_double), C.c_int32, C.c_int32, C.POINTER(C.c_double),
                                        C.c_char_p, C.c_size_t]
    L.tsa_path_costs.argtypes = [C.POINTER(Instance), C.c_int32, C.POINTER(C.c_int32), C.c_int32,
                                 C.POINTER(C.c_double), C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
    v = L.tsa_abi_version()
    if v != ABI_VERSION:
        raise RuntimeError(f"libtreesa_b200.so ABI version {v}, expected {ABI_VERSION}")
    _LIB = L
    return L


def check(rc, err, what):
    if rc != 0:
        msg = err.value.decode(errors="replace") if hasattr(err, "value") else str(err)
        cls = DeadlineError if rc == 8 else RuntimeError
        raise cls(f"{what} failed ({rc}: {ERRORS.get(rc, 'error')}): {msg}")

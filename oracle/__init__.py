"""TEST INFRASTRUCTURE ONLY: ctypes wrappers of the CPU oracles.

* ``libtsa_oracle.so`` -- our CPU restatement of the reference path (tsa_oracle.cpp): the checker of the
  CUDA path in tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline.
* ``_ref/libtsa_cpuref.so`` -- the reference's own ``csrc/cpu_ref.h`` compiled from its sources
  (Makefile), used to pin the restatement and as the reference CPU arm of bench.py.

Only tests/, ``__graft_entry__.smoke()`` and bench.py (cpu_baseline leg and ``--impl reference``) import
this package; the product (treesa_gpu_b200) never does.
"""
import ctypes as C
import os
import subprocess

import numpy as np

from treesa_gpu_b200 import _abi

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libtsa_oracle.so")
CPUREF_SO = os.path.join(HERE, "_ref", "libtsa_cpuref.so")

_ORC = None
_REF = None


def reference_csrc():
    """The reference's csrc/ directory: $TREESA_REFERENCE/csrc, else BASELINE.json's reference_path; None
    where neither names an existing source tree (the GPU box keeps the prebuilt _ref/ files)."""
    import json
    root = os.environ.get("TREESA_REFERENCE")
    if not root:
        p = os.path.join(os.path.dirname(HERE), "BASELINE.json")
        if os.path.exists(p):
            with open(p) as f:
                root = json.load(f).get("reference_path")
    if root and os.path.exists(os.path.join(root, "csrc", "cpu_ref.h")):
        return os.path.join(root, "csrc")
    return None


def build(quiet=True):
    """Compile the oracle (and the reference harness where the reference sources exist)."""
    ref = reference_csrc()
    out = subprocess.run(["make", "-C", HERE] + ([f"REF={ref}"] if ref else []), capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout[-3000:] + out.stderr[-3000:])
    if not quiet:
        print(out.stdout)


def orc():
    global _ORC
    if _ORC is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.orc_run.argtypes = [C.POINTER(_abi.Instance), C.POINTER(_abi.Options), C.POINTER(_abi.Result), C.c_char_p,
                              C.c_size_t]
        L.orc_result_free.argtypes = [C.POINTER(_abi.Result)]
        L.orc_result_free.restype = None
        L.orc_sweeps.argtypes = [C.POINTER(_abi.Instance), C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_double,
                                 C.c_double,
                                 C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_uint32),
                                 C.POINTER(C.c_uint64), C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_longlong), C.c_char_p, C.c_size_t]
        L.orc_random_tree.argtypes = [C.c_int, C.c_uint64, C.c_int, C.POINTER(C.c_uint32)]
        L.orc_random_tree.restype = None
        L.orc_labels.argtypes = [C.POINTER(_abi.Instance), C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.c_char_p,
                                 C.c_size_t]
        L.orc_expf_checksum.argtypes = [C.c_uint32, C.c_uint32]
        L.orc_expf_checksum.restype = C.c_uint64
        L.orc_energy.argtypes = [C.POINTER(_abi.Instance), C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_float), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                 C.POINTER(C.c_double), C.POINTER(C.c_int), C.c_char_p, C.c_size_t]
        _ORC = L
    return _ORC


def cpuref():
    """The reference's cpu_ref.h harness, or None when it was never built (no reference sources)."""
    global _REF
    if _REF is None:
        if not os.path.exists(CPUREF_SO):
            build()
        if not os.path.exists(CPUREF_SO):
            return None
        L = C.CDLL(CPUREF_SO)
        L.ref_sweeps.restype = C.c_double
        L.ref_sweeps.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int, C.c_uint64,
                                 C.c_double, C.c_double, C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.POINTER(C.c_longlong), C.c_int,
                                 C.c_int, C.c_int, C.c_int]
        L.ref_max_threads.restype = C.c_int
        _REF = L
    return _REF


def _p(a, ct):
    return a.ctypes.data_as(C.POINTER(ct))


def nwords(nlab):
    return max(1, (nlab + 63) // 64)


class Net:
    """An instance with label ids 0..nlab-1, packed once for the C ABI."""

    def __init__(self, ixs, iy=(), nlab=None):
        self.ixs = [list(map(int, ix)) for ix in ixs]
        self.iy = list(map(int, iy))
        self.nlab = nlab if nlab is not None else 1 + max([l for ix in self.ixs for l in ix] + list(self.iy) + [-1])
        self.m = len(self.ixs)
        self.nw = nwords(self.nlab)
        self.keep = _abi.Packed()
        self.inst = _abi.pack_instance(self.ixs, self.iy, self.nlab, self.keep)
        self.off = np.zeros(self.m + 1, np.int32)
        self.off[1:] = np.cumsum([len(ix) for ix in self.ixs])
        self.flat = np.array([l for ix in self.ixs for l in ix] or [0], np.int32)


def run(net, **kw):
    """orc_run -> (rc, dict).  kw as _abi.make_options."""
    keep = _abi.Packed()
    o = _abi.make_options(keep, **kw)
    r = _abi.Result()
    err = C.create_string_buffer(512)
    rc = orc().orc_run(C.byref(net.inst), C.byref(o), C.byref(r), err, 512)
    if rc not in (0, 2):
        raise RuntimeError(f"orc_run failed ({rc}): {err.value.decode()}")
    d = _abi.result_to_dict(r)
    orc().orc_result_free(C.byref(r))
    return rc, d


def random_tree(m, seed, chain):
    out = np.zeros(m - 1, np.uint32)
    orc().orc_random_tree(m, seed, chain, _p(out, C.c_uint32))
    return out


def labels(net, tree):
    tree = np.ascontiguousarray(tree, np.uint32)
    out = np.zeros((net.m - 1) * net.nw, np.uint64)
    err = C.create_string_buffer(256)
    rc = orc().orc_labels(C.byref(net.inst), _p(tree, C.c_uint32), _p(out, C.c_uint64), err, 256)
    if rc != 0:
        raise ValueError("invalid tree: " + err.value.decode())
    return out.reshape(net.m - 1, net.nw)


def energy(net, tree, S=None):
    """(float lcost as the GPU's eval_chain, sc, |S|, host double tc, host sc)."""
    tree = np.ascontiguousarray(tree, np.uint32)
    lc, sc, ns, sch = C.c_float(), C.c_int(), C.c_int(), C.c_int()
    tch = C.c_double()
    Sp = None
    if S is not None:
        S = np.ascontiguousarray(S, np.uint64)
        Sp = _p(S, C.c_uint64)
    err = C.create_string_buffer(256)
    rc = orc().orc_energy(C.byref(net.inst), _p(tree, C.c_uint32), Sp, C.byref(lc), C.byref(sc), C.byref(ns),
                          C.byref(tch), C.byref(sch), err, 256)
    if rc != 0:
        raise ValueError(err.value.decode())
    return lc.value, sc.value, ns.value, tch.value, sch.value


def sweeps(net, trees, betas, niters, order="par", seed=1, sc_target=20.0, sc_weight=1.0, c0=0, S=None,
           par_band=0, par_follow=False, mode="tc"):
    """Our restatement: final (trees, labels, counters) after the schedule (sweep ids lev*niters+it)."""
    trees = np.ascontiguousarray(trees, np.uint32)
    nch = trees.shape[0]
    betas = np.ascontiguousarray(betas, np.float32)
    tout = np.zeros_like(trees)
    lout = np.zeros((nch, net.m - 1, net.nw), np.uint64)
    cnt = np.zeros(3, np.longlong)
    Sp = None
    if S is not None:
        S = np.ascontiguousarray(S, np.uint64)
        Sp = _p(S, C.c_uint64)
    err = C.create_string_buffer(256)
    rc = orc().orc_sweeps(C.byref(net.inst), _abi.ORDER[order], int(par_band), int(bool(par_follow)), _abi.MODE[mode], seed,
                          sc_target, sc_weight, _p(betas, C.c_float),
                          len(betas), niters, nch, c0, _p(trees, C.c_uint32), Sp, _p(tout, C.c_uint32),
                          _p(lout, C.c_uint64), _p(cnt, C.c_longlong), err, 256)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return tout, lout, cnt


def ref_sweeps(net, trees, betas, niters, order="par", seed=1, sc_target=20.0, sc_weight=1.0, c0=0, S=None,
               nthreads=0, par_band=0, par_follow=False, mode="tc"):
    """The reference's cpu_ref.h: final (trees, labels, counters, seconds)."""
    L = cpuref()
    if L is None:
        raise RuntimeError("reference harness oracle/_ref/libtsa_cpuref.so not built")
    trees = np.ascontiguousarray(trees, np.uint32)
    nch = trees.shape[0]
    lin = np.stack([labels(net, t) for t in trees]) if nch else np.zeros((0, net.m - 1, net.nw), np.uint64)
    lin = np.ascontiguousarray(lin, np.uint64)
    betas = np.ascontiguousarray(betas, np.float32)
    tout = np.zeros_like(trees)
    lout = np.zeros((nch, net.m - 1, net.nw), np.uint64)
    cnt = np.zeros(2, np.longlong)
    Sp = None
    if S is not None:
        S = np.ascontiguousarray(S, np.uint64)
        Sp = _p(S, C.c_uint64)
    secs = L.ref_sweeps(net.m, net.nlab, _p(net.off, C.c_int), _p(net.flat, C.c_int), _abi.ORDER[order], seed,
                        sc_target, sc_weight, _p(betas, C.c_float), len(betas), niters, nch, c0,
                        _p(trees, C.c_uint32), _p(lin, C.c_uint64), Sp, _p(tout, C.c_uint32), _p(lout, C.c_uint64),
                        _p(cnt, C.c_longlong), nthreads, int(par_band), int(bool(par_follow)), _abi.MODE[mode])
    return tout, lout, cnt, secs

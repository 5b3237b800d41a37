"""Thin Python handles over the C ABI of libtreesa_b200.so (include/treesa_b200.h).

``Network`` packs an instance with label ids 0..nlab-1; ``run`` is one tsa_run call; ``Session`` keeps the
chains resident on the device (tsa_session_*) for benchmarks and tests.  No computation happens here.
"""
import ctypes as C

import numpy as np

from . import _abi


class Network:
    """Tensor network with label ids 0..nlab-1 (driver.label_map applied)."""

    def __init__(self, ixs, iy=(), nlab=None):
        self.ixs = [[int(l) for l in ix] for ix in ixs]
        self.iy = [int(l) for l in iy]
        self.nlab = int(nlab) if nlab is not None else 1 + max([l for ix in self.ixs for l in ix] + self.iy + [-1])
        self.m = len(self.ixs)
        self.keep = _abi.Packed()
        self.inst = _abi.pack_instance(self.ixs, self.iy, self.nlab, self.keep)

    @property
    def nw(self):
        """u64 words per label set in the device layout (padded to even above one word)."""
        n = max(1, (self.nlab + 63) // 64)
        return n + (n & 1) if n > 1 else n


def tree_words(tree):
    """[(left, right), ...] or an (m-1, 2) array -> uint32 words left | right << 16."""
    t = np.asarray(tree, np.int64).reshape(-1, 2)
    return (t[:, 0] | (t[:, 1] << 16)).astype(np.uint32)


def run(net, **opts):
    """One tsa_run; returns (rc, result dict).  rc 2 (invalid tree) still returns the result."""
    L = _abi.lib()
    keep = _abi.Packed()
    o = _abi.make_options(keep, **opts)
    r = _abi.Result()
    err = C.create_string_buffer(1024)
    rc = L.tsa_run(C.byref(net.inst), C.byref(o), C.byref(r), err, 1024)
    if rc not in (0, 2):
        L.tsa_result_free(C.byref(r))
        _abi.check(rc, err, "tsa_run")
    d = _abi.result_to_dict(r)
    L.tsa_result_free(C.byref(r))
    return rc, d


class Session:
    """Chains resident on one device between calls (tsa_session_*)."""

    def __init__(self, net, **opts):
        self.L = _abi.lib()
        self.net = net
        self.keep = _abi.Packed()
        self.opts = _abi.make_options(self.keep, **opts)
        self.nchains = int(opts["nchains"])
        self.h = C.c_void_p()
        err = C.create_string_buffer(1024)
        rc = self.L.tsa_session_create(C.byref(net.inst), C.byref(self.opts), C.byref(self.h), err, 1024)
        _abi.check(rc, err, "tsa_session_create")

    def _call(self, fn, *args, what=""):
        err = C.create_string_buffer(1024)
        rc = fn(self.h, *args, err, 1024)
        _abi.check(rc, err, what)
        return rc

    def run(self):
        self._call(self.L.tsa_session_run, what="tsa_session_run")

    def reset(self):
        self._call(self.L.tsa_session_reset, what="tsa_session_reset")

    def result(self):
        r = _abi.Result()
        err = C.create_string_buffer(1024)
        rc = self.L.tsa_session_result(self.h, C.byref(r), err, 1024)
        if rc not in (0, 2):
            _abi.check(rc, err, "tsa_session_result")
        d = _abi.result_to_dict(r)
        self.L.tsa_result_free(C.byref(r))
        return rc, d

    def stats(self):
        c = (C.c_uint64 * 12)()
        ks = C.c_double()
        self.L.tsa_session_stats(self.h, c, C.byref(ks))
        names = ["proposals", "accepts", "phases", "visits", "slice_proposals", "slice_accepts", "busy_lanes",
                 "launches", "chunks", "chunks_acc", "h2d_bytes", "d2h_bytes"]
        d = {k: int(v) for k, v in zip(names, c)}
        d["kernel_s"] = ks.value
        return d

    def timing(self):
        """Seconds of the last run on this rank: sweep kernels, energy gathers and population steps (device
        time of level-by-level runs), the whole call's wall time, host selection and best-record fetches;
        and the record bytes sent to / received from other ranks (tsa_session_timing)."""
        t = (C.c_double * 8)()
        self.L.tsa_session_timing(self.h, t)
        return dict(zip(["kernel_s", "gather_s", "resample_s", "run_s", "select_s", "fetch_s", "sent_bytes",
                         "recv_bytes"], [float(x) for x in t]))

    def energies(self):
        lc = np.zeros(self.nchains, np.float32)
        sc = np.zeros(self.nchains, np.int32)
        ns = np.zeros(self.nchains, np.int32)
        self._call(self.L.tsa_session_energies, lc.ctypes.data_as(C.POINTER(C.c_float)),
                   sc.ctypes.data_as(C.POINTER(C.c_int32)), ns.ctypes.data_as(C.POINTER(C.c_int32)),
                   what="tsa_session_energies")
        return lc, sc, ns

    def info(self):
        v = (C.c_int32 * 8)()
        self.L.tsa_session_info(self.h, v)
        keys = ["m", "nint", "nw", "rec_bytes", "kernel", "warps_per_cta", "grid", "smem"]
        return dict(zip(keys, [int(x) for x in v]))

    def chains(self):
        nint = self.net.m - 1
        t = np.zeros((self.nchains, nint), np.uint32)
        lab = np.zeros((self.nchains, nint, self.info()["nw"]), np.uint64)
        self._call(self.L.tsa_session_chains, t.ctypes.data_as(C.POINTER(C.c_uint32)),
                   lab.ctypes.data_as(C.POINTER(C.c_uint64)), what="tsa_session_chains")
        return t, lab

    def close(self):
        if self.h:
            self.L.tsa_session_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def resample(records_ptr, anc, rec_bytes, stream=None):
    """tsa_resample: device records (pointer, nchains x rec_bytes) <- their ancestors, in place."""
    anc = np.ascontiguousarray(anc, np.int32)
    err = C.create_string_buffer(512)
    rc = _abi.lib().tsa_resample(C.c_void_p(records_ptr), anc.ctypes.data_as(C.POINTER(C.c_int32)), len(anc),
                                 int(rec_bytes), stream, err, 512)
    _abi.check(rc, err, "tsa_resample")


def nccl_unique_id():
    """128-byte ncclUniqueId for a multi-GPU run (rank 0 creates it and shares it)."""
    buf = C.create_string_buffer(128)
    err = C.create_string_buffer(512)
    rc = _abi.lib().tsa_nccl_unique_id(buf, err, 512)
    _abi.check(rc, err, "tsa_nccl_unique_id")
    return buf.raw


def laplacian_vectors(n, rows, cols, w, k=3, device=0):
    """Eigenvectors 2..k+1 of the weighted graph Laplacian on the GPU (tsa_laplacian_vectors, cuSOLVER)."""
    L = _abi.lib()
    r = np.ascontiguousarray(rows, np.int32)
    c = np.ascontiguousarray(cols, np.int32)
    ww = np.ascontiguousarray(w, np.float64)
    V = np.zeros((n, k), np.float64)
    err = C.create_string_buffer(512)
    p = lambda x, t: x.ctypes.data_as(C.POINTER(t))  # noqa: E731
    rc = L.tsa_laplacian_vectors(int(n), len(ww), p(r, C.c_int32), p(c, C.c_int32), p(ww, C.c_double), int(k),
                                 int(device), p(V, C.c_double), err, 512)
    _abi.check(rc, err, "tsa_laplacian_vectors")
    return V


def path_costs(net, orders, device=0):
    """(tc, sc) arrays of the path trees of a batch of tensor orderings on the GPU (tsa_path_costs)."""
    L = _abi.lib()
    o = np.ascontiguousarray(orders, np.int32)
    if o.ndim == 1:
        o = o[None, :]
    tc = np.zeros(o.shape[0], np.float64)
    sc = np.zeros(o.shape[0], np.int32)
    err = C.create_string_buffer(512)
    rc = L.tsa_path_costs(C.byref(net.inst), o.shape[0], o.ctypes.data_as(C.POINTER(C.c_int32)), int(device),
                          tc.ctypes.data_as(C.POINTER(C.c_double)), sc.ctypes.data_as(C.POINTER(C.c_int32)), err, 512)
    _abi.check(rc, err, "tsa_path_costs")
    return tc, sc


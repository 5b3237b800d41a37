"""C-ABI checks that need no GPU: the library loads, exports every entry point include/treesa_b200.h
declares, validates its arguments before touching a device, and plans population exchanges correctly."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from treesa_gpu_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "treesa_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tsa_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _abi.lib()
    assert L.tsa_abi_version() == _abi.ABI_VERSION
    names = declared()
    assert "tsa_run" in names and "tsa_session_create" in names
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/treesa_b200.h but not exported"
    assert L.tsa_release_cached_memory() == 0  # an empty block cache is released without a device


def test_ctypes_structs_match_the_library():
    """The ctypes mirrors of tsa_instance / tsa_options / tsa_result have the library's sizes."""
    sizes = (C.c_int32 * 3)()
    assert _abi.lib().tsa_abi_sizes(sizes) == 0
    assert list(sizes) == [C.sizeof(_abi.Instance), C.sizeof(_abi.Options), C.sizeof(_abi.Result)]
    assert _abi.Options.timeout_s.offset == 220 and _abi.Options.wait_log2.offset == 224
    assert _abi.Options.debug_flags.offset == 228 and _abi.Options.reserved.offset == 232


def _create(ixs, iy=(), nlab=None, **kw):
    from treesa_gpu_b200 import engine
    L = _abi.lib()
    net = engine.Network(ixs, iy, nlab)
    keep = _abi.Packed()
    opts = dict(betas=[1.0], niters=1, nchains=4)
    opts.update(kw)
    o = _abi.make_options(keep, **opts)
    h = C.c_void_p()
    err = C.create_string_buffer(512)
    rc = L.tsa_session_create(C.byref(net.inst), C.byref(o), C.byref(h), err, 512)
    if rc == 0:
        L.tsa_session_destroy(h)
    return rc, err.value.decode()


def test_argument_errors_are_reported_not_fatal():
    tri = [[0, 1], [1, 2], [2, 0]]
    assert _create([[0], [0]]) == (1, "need at least 3 tensors")
    assert _create([[0, 0], [0, 1], [1]])[0] == 1  # repeated label in a tensor
    assert _create(tri, nlab=2)[0] == 1  # label out of range
    assert _create(tri, iy=[5], nlab=3)[0] == 1  # open label out of range
    rc, msg = _create(tri, betas2=[1.0, 2.0], mode2="tc")  # stage 2 runs a model energy
    assert rc == 1 and "stage-2" in msg
    assert _create(tri, betas=[])[0] == 1
    assert _create(tri, nchains=0)[0] == 1
    rc, msg = _create(tri, init_slices=[7])
    assert rc == 1 and "init_slices" in msg
    assert _create(tri, rank=2, world_size=2)[0] == 1
    rc, msg = _create(tri, par_band=1)  # the reference's --par-band check (csrc/treesa_gpu.cu:1527)
    assert rc == 1 and "2..16" in msg
    assert _create(tri, par_band=17)[0] == 1
    assert _create(tri, kernel_hint=3, par_follow=True)[0] == 1
    rc, msg = _create(tri, timeout_s=-1.0)
    assert rc == 1 and "timeout_s" in msg
    rc, msg = _create(tri, wait_log2=5)
    assert rc == 1 and "wait_log2" in msg
    rc, msg = _create(tri, debug_flags=6)
    assert rc == 1 and "debug_flags" in msg
    big = [[i, (i + 1) % 32769] for i in range(32769)]  # node ids are 16-bit: at most 32768 tensors
    rc, msg = _create(big)
    assert rc == 1 and "16-bit" in msg


def test_run_reports_errors_through_the_python_api():
    import treesa_gpu_b200 as t
    with pytest.raises(ValueError):
        t.optimize([[0, 1], [1, 2], [2, 0]], [], mode="bogus")
    with pytest.raises(ValueError):
        t.optimize([[0, 1], [1, 2], [2, 0]], [], select="bogus")
    with pytest.raises(TypeError):
        t.optimize([[0, 1], [1, 2], [2, 0]], [], no_such_option=1)


def _plan(anc, nloc, rank, world):
    L = _abi.lib()
    L.tsa_resample_plan.argtypes = [C.POINTER(C.c_int)] + [C.c_int] * 3 + [C.POINTER(C.c_int)] * 5
    a = np.ascontiguousarray(anc, np.int32)
    src = np.zeros(nloc, np.int32)
    so = np.zeros(world + 1, np.int32)
    si = np.zeros(nloc * world, np.int32)
    ro = np.zeros(world + 1, np.int32)
    ri = np.zeros(nloc, np.int32)
    p = lambda x: x.ctypes.data_as(C.POINTER(C.c_int))  # noqa: E731
    L.tsa_resample_plan(p(a), nloc, rank, world, p(src), p(so), p(si), p(ro), p(ri))
    return src, so, si, ro, ri


@pytest.mark.parametrize("world", [2, 3, 4])
def test_resample_plan_moves_every_chain_from_its_ancestor(world):
    """Simulate the exchange: every rank packs what it sends, receives what it needs, and gathers."""
    rng = np.random.default_rng(world)
    nloc = 37
    ng = nloc * world
    recs = np.arange(ng) * 1000 + 7  # a record = its global id, recognisably
    for trial in range(20):
        anc = rng.integers(0, ng, ng) if trial % 2 else np.sort(rng.integers(0, ng, ng))
        plans = [_plan(anc, nloc, r, world) for r in range(world)]
        for r in range(world):
            src, so, si, ro, ri = plans[r]
            received = []
            for q in range(world):
                if q == r:
                    continue
                # what q sends to r, in q's order, must be exactly the ids r expects from q
                qso, qsi = plans[q][1], plans[q][2]
                sent = [q * nloc + x for x in qsi[qso[r]:qso[r + 1]]]
                assert sent == list(ri[ro[q]:ro[q + 1]])
            for q in range(world):
                received += [recs[g] for g in ri[ro[q]:ro[q + 1]]]
            pool = list(recs[r * nloc:(r + 1) * nloc]) + received
            new = [pool[s] for s in src]
            assert new == [recs[a] for a in anc[r * nloc:(r + 1) * nloc]]
            # no record travels twice to the same rank
            for q in range(world):
                ids = list(ri[ro[q]:ro[q + 1]])
                assert len(ids) == len(set(ids))

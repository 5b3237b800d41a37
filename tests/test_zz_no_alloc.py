"""tsa_resample_noalloc: the population resample for callers that cannot allocate device memory when they
call it (a process whose device memory belongs to its own fixed pool, a loop where cudaMalloc would
synchronize the device).  Called through the C ABI, its records must equal those of tsa_resample,
the allocating entry point, on two calls in a row (the second with other ancestors, over the scratch the
first call left behind).  The data are bytes, so the comparison is exact.  This file sorts last so that a
run stopping at its first failure has run every other test; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(fn, ptr, anc, rec_bytes, stream):
    anc = np.ascontiguousarray(anc, np.int32)
    err = C.create_string_buffer(512)
    rc = fn(C.c_void_p(ptr), anc.ctypes.data_as(C.POINTER(C.c_int32)), len(anc), rec_bytes, C.c_void_p(stream), err,
            512)
    return rc, err.value.decode()


def test_noalloc_resample_equals_allocating_resample_twice():
    import torch
    from treesa_gpu_b200 import _abi
    L = _abi.lib()
    rng = np.random.default_rng(2024)
    nchains, rec_bytes = 700, 10240  # 7 MB of records, like 700 chains of the sat100 layout
    host = rng.integers(0, 256, (nchains, rec_bytes), dtype=np.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    a = torch.from_numpy(host.copy()).cuda()
    b = torch.from_numpy(host.copy()).cuda()
    for call in range(2):
        anc = rng.integers(0, nchains, nchains)
        rc1, e1 = _call(L.tsa_resample, a.data_ptr(), anc, rec_bytes, stream)
        rc2, e2 = _call(L.tsa_resample_noalloc, b.data_ptr(), anc, rec_bytes, stream)
        assert rc1 == 0 and rc2 == 0, (e1, e2)
        torch.cuda.synchronize()
        assert torch.equal(a, b), f"call {call}: records differ"
        host = host[anc]
        assert (b.cpu().numpy() == host).all()


def test_noalloc_resample_rejects_populations_above_its_scratch():
    import torch
    from treesa_gpu_b200 import _abi
    L = _abi.lib()
    small = torch.zeros(16, dtype=torch.uint8, device="cuda")
    rc, msg = _call(L.tsa_resample_noalloc, small.data_ptr(), np.zeros(70000, np.int32), 16, None)
    assert rc == 1 and "exceed" in msg
    rc, msg = _call(L.tsa_resample_noalloc, small.data_ptr(), np.zeros(8, np.int32), (65 << 20) // 8 // 16 * 16, None)
    assert rc == 1 and "exceed" in msg

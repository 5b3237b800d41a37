"""tsa_resample (population resampling of caller-held records, the reference's Runner::resample) on the
GPU: every record becomes its ancestor's, for random and for degenerate ancestor maps; bad arguments are
rejected before any device work."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nchains,rec_bytes", [(1, 16), (37, 10240), (512, 4096)])
def test_resample_gathers_ancestors(nchains, rec_bytes):
    import torch
    from treesa_gpu_b200 import engine
    rng = np.random.default_rng(nchains)
    host = rng.integers(0, 256, (nchains, rec_bytes), dtype=np.uint8)
    for anc in (rng.integers(0, nchains, nchains), np.zeros(nchains, np.int64), np.arange(nchains)[::-1]):
        dev = torch.from_numpy(host.copy()).cuda()
        engine.resample(dev.data_ptr(), anc, rec_bytes, torch.cuda.current_stream().cuda_stream)
        assert (dev.cpu().numpy() == host[anc]).all()


def test_resample_rejects_bad_arguments():
    import torch
    from treesa_gpu_b200 import engine
    dev = torch.zeros(4 * 32, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        engine.resample(dev.data_ptr(), [0, 1, 2, 4], 32)
    with pytest.raises(RuntimeError):
        engine.resample(dev.data_ptr(), [0, 1, 2, 3], 24)

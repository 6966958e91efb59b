"""Failure detection on the device without faulting the GPU: a bounded wait that runs out gives
up, records DEV_WAIT_TIMEOUT (1) in the device error word and returns; sfc_device_error reports
the code once and clears it; the context stays usable afterwards."""
import numpy as np
import pytest

import stage_oracle as so
from gpu_util import assert_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


def test_bounded_wait_times_out_and_reports(sf):
    sf.device_error()  # start from a clear word
    sf.selftest_bounded_wait(64, complete=True)
    assert sf.device_error() == 0  # a wait that completes records nothing
    sf.selftest_bounded_wait(64, complete=False)
    assert sf.device_error() == 1  # DEV_WAIT_TIMEOUT
    assert sf.device_error() == 0  # read once, then cleared
    # the context still runs kernels correctly
    raw = so.synth_tensor(so.Q4_K, so.tensor_key(5, "after.timeout"), 64, 512, 0.02)
    x = so.synth_normal_f32(5, "after.timeout.x", 512).reshape(1, 512)
    w = sf.prepare_weights(sf.Q4_K, torch.from_numpy(raw).cuda(), 64, 512)
    y = sf.matmul(sf.Q4_K, w, 64, 512, torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), so.matmul(so.Q4_K, raw, 64, 512, x), what="GEMV after a timed-out wait")
    assert sf.device_error() == 0


def test_selftest_rejects_zero_budget(sf):
    with pytest.raises(sf.StageError, match="spin_limit"):
        sf.selftest_bounded_wait(0, complete=False)

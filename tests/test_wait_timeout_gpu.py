"""The bounded inter-CTA wait gives up instead of hanging (failure detection
without a GPU fault): a probe kernel waits on an mbarrier phase that nothing
completes, with a 50 ms limit, and must return with the timeout recorded in
the device status word; the context stays usable afterwards."""
import pytest
import torch

from rnn_kernel_b200 import _lib
from tests.gpu_parity import assert_parity, run_pair

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_reports():
    lib = _lib.load()
    _lib.device_status(reset=True)
    res = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    rc = lib.gru_selftest_wait_timeout(50, res.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert int(res.item()) == 0
    assert _lib.device_status(reset=True) & 1  # GRU_STATUS_WAIT_TIMEOUT
    assert _lib.device_status() == 0
    # the context still runs the real kernels correctly
    mine, theirs, truth = run_pair(4, 32, 1, 2, 3, seed=9)
    assert_parity(mine, theirs, truth)
    assert _lib.device_status() == 0


def test_selftest_rejects_bad_limits():
    lib = _lib.load()
    assert lib.gru_selftest_wait_timeout(0, None, None) == 1
    assert lib.gru_selftest_wait_timeout(20000, None, None) == 1

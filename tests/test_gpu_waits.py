"""GPU: an expired bounded device wait reaches the caller as a RuntimeError, and the
context stays usable afterwards.

The kernels never trap or spin without a limit: every mbarrier wait and every
d-split exchange counter wait gives up after a bounded number of polls, records
UTTT_ERR_TIMEOUT in the workspace status word and lets the launch return.  The
self-test kernel runs those same wait helpers on events that never happen (an
mbarrier phase with no arrival, an exchange counter nothing increments) with a
short poll limit, so the wait expires in microseconds with no copy or MMA in
flight.
"""

import pytest
import torch

from utttcompanion_b200 import _lib
from utttcompanion_b200 import fastweight as fw

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", [0, 1], ids=["mbarrier", "exchange_counter"])
def test_expired_wait_raises_runtime_error_and_context_survives(kind):
    lib = _lib.load()
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.uttt_selftest_wait(kind, 4096, ws.data_ptr(), ws.numel(), stream), "uttt_selftest_wait")
    with pytest.raises(RuntimeError, match="wait"):
        fw.check_status(ws, "uttt_selftest_wait")
    assert int(ws[260:264].view(torch.int32).item()) == 1           # the kernel returned
    assert lib.uttt_read_status(ws.data_ptr(), 0, stream) == 0      # check_status cleared the word
    # the context is still usable: an ordinary op runs and gives the right answer
    x = torch.randn(1024, device="cuda")
    assert torch.allclose((x * 2).sum(), x.sum() * 2, rtol=1e-4, atol=1e-3)
    torch.cuda.synchronize()


def test_wait_selftest_rejects_bad_arguments():
    lib = _lib.load()
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.uttt_selftest_wait(2, 16, ws.data_ptr(), ws.numel(), stream) == _lib.UTTT_ERR_INVALID
    assert lib.uttt_selftest_wait(0, 0, ws.data_ptr(), ws.numel(), stream) == _lib.UTTT_ERR_INVALID
    assert lib.uttt_selftest_wait(0, 16, ws.data_ptr(), 64, stream) == _lib.UTTT_ERR_WORKSPACE

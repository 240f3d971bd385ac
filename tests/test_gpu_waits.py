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


def test_peer_exchange_wait_expires_when_the_peer_never_arrives():
    """uttt_split_exchange_finish on one GPU with a second, local exchange area standing in for a
    peer that never runs: the stores into it stay in bounds, its flag for this rank is never
    raised, so the flag wait gives up after the poll limit, records UTTT_ERR_TIMEOUT and the
    kernel returns; the context keeps working."""
    import ctypes
    lib = _lib.load()
    rows, d, world = 4, 256, 2
    nbytes = lib.uttt_split_exchange_bytes(world, rows, d)
    own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    fake_peer = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    areas = (ctypes.c_void_p * 2)(own.data_ptr(), fake_peer.data_ptr())
    z = torch.randn(rows, d, device="cuda")
    x = torch.randn(rows, d, device="cuda").to(torch.bfloat16)
    lw, lb = torch.ones(d, device="cuda"), torch.zeros(d, device="cuda")
    out = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.uttt_split_exchange_finish(rows, d, z.data_ptr(), x.data_ptr(), lw.data_ptr(), lb.data_ptr(),
                                              1e-5, out.data_ptr(), _lib.DTYPE_BF16, 1, 0, world, rows,
                                              ctypes.cast(areas, ctypes.c_void_p), 4096, ws.data_ptr(), ws.numel(),
                                              stream), "uttt_split_exchange_finish")
    with pytest.raises(RuntimeError, match="wait"):
        fw.check_status(ws, "uttt_split_exchange_finish")
    # this rank's partial rows went into the stand-in peer's receive slot [parity 0][rank 0]
    flags = (world * rows * 4 + 255) // 256 * 256
    recv = fake_peer[flags + 256:].view(torch.float32)[: rows * d].reshape(rows, d)
    assert torch.equal(recv, z)
    # the exchange's epoch in this rank's own area was bumped after the call
    assert int(own[flags:flags + 4].view(torch.int32).item()) == 1
    y = torch.randn(1024, device="cuda")
    assert torch.allclose((y * 2).sum(), y.sum() * 2, rtol=1e-4, atol=1e-3)
    torch.cuda.synchronize()

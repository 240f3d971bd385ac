"""GPU: the tensor-core conventions (UMMA descriptors, 128B swizzle, TMEM
drain, software BF16 producers) against a plain FP32 matmul."""

import pytest
import torch

from utttcompanion_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 5, 7])
@pytest.mark.parametrize("N", [64, 128, 256])
def test_selftest_gemm_orientations(mode, N):
    lib = _lib.load()
    torch.manual_seed(mode * 7 + N)
    M, K = 256, 192
    dev = "cuda"
    a32 = torch.randn(M, K, device=dev)
    b32 = torch.randn(N, K, device=dev)
    a_bf = a32.to(torch.bfloat16)
    b_bf = b32.to(torch.bfloat16)
    if mode & 4:
        a_arg = a32.t().contiguous()            # FP32, K x M
        a_ref = a32.to(torch.bfloat16).float()
    elif mode & 1:
        a_arg = a_bf.t().contiguous()           # K x M
        a_ref = a_bf.float()
    else:
        a_arg = a_bf.contiguous()
        a_ref = a_bf.float()
    b_arg = b_bf.t().contiguous() if mode & 2 else b_bf.contiguous()
    d = torch.full((M, N), float("nan"), device=dev)
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    st = lib.uttt_selftest_gemm(mode, M, N, K, a_arg.data_ptr(), b_arg.data_ptr(), d.data_ptr(), ws.data_ptr(),
                                256, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "selftest_gemm")
    torch.cuda.synchronize()
    assert lib.uttt_read_status(ws.data_ptr(), 1, torch.cuda.current_stream().cuda_stream) == 0
    ref = a_ref @ b_bf.float().t()
    err = (d - ref).norm() / ref.norm()
    assert torch.isfinite(d).all()
    assert err < 1e-5, float(err)

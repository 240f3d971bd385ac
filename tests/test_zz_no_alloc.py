"""GPU: the allocation-free chunk write (static device scratch) against the
workspace-taking entry point, through the C ABI, on two calls in a row.

The allocation-free variant serves callers that cannot call cudaMalloc (a
serving loop whose HBM is reserved up front, or a foreign-language binding
with no device allocator).  It must give the same state as the regular
entry point within the tolerances the other parity tests use, keep working
on a second call that reuses the shared scratch, and refuse sizes beyond its
fixed scratch before doing any work.  This file is collected last so that a
run stopping at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle.numerics import rel_l2
from utttcompanion_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(seed, B, Tn, d, h):
    g = torch.Generator(device="cuda").manual_seed(seed)

    def unit(shape):
        x = torch.randn(shape, generator=g, device="cuda")
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16).contiguous()

    st = {"k": unit((B, Tn, d)), "v": unit((B, Tn, d)),
          "eta": torch.rand((B, Tn), generator=g, device="cuda") * 0.04 + 0.005,
          "alpha": torch.rand((B, Tn), generator=g, device="cuda") * 0.01,
          "ln_w": 1 + 0.1 * torch.randn(d, generator=g, device="cuda"),
          "ln_b": 0.1 * torch.randn(d, generator=g, device="cuda")}
    st["mask"] = torch.ones((B, Tn), device="cuda")
    st["mask"][1, Tn - 40:] = 0
    for n, shp in (("w_up", (B, d, h)), ("w_gate", (B, d, h)), ("w_down", (B, h, d))):
        st[n] = (torch.randn(shp, generator=g, device="cuda") * 0.02).contiguous()
        st["s" + n[1:]] = (torch.randn(shp, generator=g, device="cuda") * 1e-3).contiguous()
    return st


def _args(st, B, Tn, C, d, h, loss):
    p = lambda t: t.data_ptr()  # noqa: E731
    return [B, Tn, C, d, h, 0, (Tn + C - 1) // C, p(st["k"]), p(st["k"]), p(st["v"]), p(st["eta"]),
            p(st["alpha"]), p(st["mask"]), p(st["w_up"]), p(st["w_gate"]), p(st["w_down"]), p(st["s_up"]),
            p(st["s_gate"]), p(st["s_down"]), p(st["ln_w"]), p(st["ln_b"]), 0.9, 1.0, 1, 1e-5, None,
            _lib.DTYPE_F32, p(loss), None]


def test_noalloc_chunk_write_matches_workspace_entry_point_twice():
    lib = _lib.load()
    B, Tn, C, d, h = 2, 160, 64, 256, 384
    ref = _inputs(11, B, Tn, d, h)
    na = {k: v.clone() for k, v in ref.items()}
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = lib.uttt_chunk_write_workspace(B, C, d, h)
    assert ws_bytes <= 8 << 20
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    loss_ref = torch.empty((B, Tn), device="cuda")
    loss_na = torch.empty((B, Tn), device="cuda")
    names = ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down")
    for call in range(2):
        before = {n: ref[n].clone() for n in names}
        _lib.check(lib.uttt_chunk_write(*_args(ref, B, Tn, C, d, h, loss_ref), B, None, None, None, ws.data_ptr(),
                                        ws_bytes, stream),
                   "uttt_chunk_write")
        _lib.check(lib.uttt_chunk_write_noalloc(*_args(na, B, Tn, C, d, h, loss_na), stream),
                   "uttt_chunk_write_noalloc")
        torch.cuda.synchronize()
        assert lib.uttt_read_status(ws.data_ptr(), 1, stream) == 0
        # every bounded device wait of the allocation-free call ended (its status word is 0)
        assert lib.uttt_chunk_write_noalloc_status(0, stream) == 0, call
        for n in names:
            got, want = na[n].cpu().numpy(), ref[n].cpu().numpy()
            assert np.isfinite(got).all(), (call, n)
            if n.startswith("w"):
                assert rel_l2(got, want) < 1e-3, (call, n)
                base = before[n].cpu().numpy()
                assert rel_l2(got - base, want - base) < 2e-2, (call, n)
            else:
                assert rel_l2(got, want) < 2e-2, (call, n)
        assert rel_l2(loss_na.cpu().numpy(), loss_ref.cpu().numpy()) < 1e-2, call


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    B, Tn, C, d, h = 64, 2048, 64, 1024, 2816       # config-2 batch needs far more than 8 MiB
    assert lib.uttt_chunk_write_workspace(B, C, d, h) > 8 << 20
    dummy = ctypes.c_void_p(16)                       # never dereferenced: rejected on the host
    args = [B, Tn, C, d, h, 0, 1] + [dummy] * 14 + [0.0, 0.0, 1, 1e-5, None, _lib.DTYPE_F32, None, None, None]
    assert lib.uttt_chunk_write_noalloc(*args) == _lib.UTTT_ERR_WORKSPACE
    with pytest.raises(ValueError, match="workspace"):
        _lib.check(lib.uttt_chunk_write_noalloc(*args), "uttt_chunk_write_noalloc")

"""GPU parity of the sliding-window prefill / chunk attention (uttt_attn_prefill).

The kernel writes the RoPE'd queries and the new keys / values into its
scratch buffers; the reference recomputes the causal sliding-window softmax
attention (SlidingWindowAttention, model/uttt_layer.py:961-1168: a query at
buffer index p sees keys in (p - W, p]) in FP32 from those same BF16 tensors,
so the test isolates the attention.  Bound: |out - ref| <= 4e-3 + 4e-3 |ref|,
the BF16 rounding of the output plus FP32 accumulation (the probabilities
enter the P.V product as a BF16 hi + lo pair, about 16 significant bits).
"""

import numpy as np
import pytest
import torch

from utttcompanion_b200 import _lib
from utttcompanion_b200.model import rope_tables

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("hd,n_heads,n_kv,W,B,T,hist", [
    (64, 4, 4, 128, 1, 256, 0),        # CONFIG_TINY-like prefill (one query head per group)
    (64, 12, 4, 512, 2, 64, 37),       # 151M: three query heads per group, a chunk after history
    (128, 20, 5, 512, 1, 64, 511),     # 1.58B: a write chunk behind a full window of history
    (128, 20, 5, 512, 1, 700, 0),      # 1.58B prefill longer than the window
    (128, 8, 1, 128, 3, 33, 5),        # eight heads per group, ragged T
    (64, 2, 2, 16, 2, 1, 15),          # one new token
])
def test_prefill_attention_matches_fp32_reference(hd, n_heads, n_kv, W, B, T, hist):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(hd * 1000 + T + hist)
    start = hist + 3                   # absolute position of the first new token
    L = hist + T
    qkv_dim = (n_heads + 2 * n_kv) * hd
    qkv = torch.randn(B * T, qkv_dim, device=dev, generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(hd, start + T + 8, 10000.0)
    cos, sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
    qs = torch.empty(B * T, n_heads, hd, dtype=torch.bfloat16, device=dev)
    kb = torch.randn(B, n_kv, L, hd, device=dev, generator=g).to(torch.bfloat16)   # history rows stay
    vb = torch.randn(B, n_kv, L, hd, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(B * T, n_heads, hd, dtype=torch.bfloat16, device=dev)
    st = lib.uttt_attn_prefill(B, T, start, hist, n_heads, n_kv, hd, W, qkv.data_ptr(), qkv_dim, cos.data_ptr(),
                               sin.data_ptr(), qs.data_ptr(), kb.data_ptr(), vb.data_ptr(), out.data_ptr(), _stream())
    _lib.check(st, "uttt_attn_prefill")
    torch.cuda.synchronize()
    q = qs.float().reshape(B, T, n_heads, hd)
    k, v = kb.float(), vb.float()
    rep = n_heads // n_kv
    idx = torch.arange(L, device=dev)
    ref = torch.empty(B, T, n_heads, hd, device=dev)
    for t in range(T):
        p = hist + t
        keep = (idx <= p) & (idx > p - W)
        for hh in range(n_heads):
            s = (k[:, hh // rep] @ q[:, t, hh].unsqueeze(-1)).squeeze(-1) / hd ** 0.5     # (B, L)
            s = s.masked_fill(~keep, float("-inf"))
            ref[:, t, hh] = torch.softmax(s, dim=-1).unsqueeze(1).bmm(v[:, hh // rep]).squeeze(1)
    got = out.float().reshape(B, T, n_heads, hd)
    err = (got - ref).abs()
    bound = 4e-3 + 4e-3 * ref.abs()
    assert bool((err <= bound).all()), float(err.max())
    assert np.isfinite(got.cpu().numpy()).all()

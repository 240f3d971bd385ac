"""Drop-in fast-weight readout functions (``model/uttt_layer.py:211-257,648-695``).

``swiglu_fast_forward`` / ``swiglu_packed_forward`` keep the reference's
positional signatures and return ``x``'s dtype.  Operands are BF16 on the
tensor cores (the reference's serving dtype); statistics and accumulation
are FP32.  As in the reference, the LayerNorm affine is applied in the
activation dtype (``ln_weight.to(x.dtype)``).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .fastweight import _ptr, _require_cuda, _stream, workspace


def fast_readout(x: torch.Tensor, w_up: torch.Tensor, w_gate: Optional[torch.Tensor], w_down: torch.Tensor,
                 ln_weight: torch.Tensor, ln_bias: torch.Tensor, eps: float = 1e-5,
                 state_index: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                 packed: bool = False, ln_prepared: bool = False,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """f_W(x) for (B, T, d) ``x``.  ``packed``: ``w_up`` is the BF16 [W_up | W_gate] copy.

    ``ln_prepared``: ``ln_weight``/``ln_bias`` are already FP32 contiguous and
    rounded to the activation dtype (skips two casts per call, e.g. inside a
    captured decode graph).  ``out``: preallocated BF16 (B, T, d) output.
    """
    _require_cuda(x, w_up, w_down)
    if x.dim() != 3:
        raise ValueError("x must be (B, T, d)")
    B, T, d = x.shape
    h = w_down.shape[-2]
    xb = x.to(torch.bfloat16).contiguous()
    if packed:
        if w_up.dtype != torch.bfloat16 or w_down.dtype != torch.bfloat16:
            raise ValueError("packed read copies must be BF16")
        wd_kind = _lib.DTYPE_BF16
        wu, wg, wd = w_up.contiguous(), None, w_down.contiguous()
    elif w_up.dtype == torch.bfloat16:
        wd_kind = _lib.DTYPE_BF16
        wu, wg, wd = torch.cat((w_up, w_gate), dim=-1).contiguous(), None, w_down.contiguous()
    else:
        wd_kind = _lib.DTYPE_F32
        wu, wg, wd = (w.to(torch.float32).contiguous() for w in (w_up, w_gate, w_down))
    S = wu.shape[0]
    if state_index is None and S != B:
        if S == 1:
            state_index = torch.zeros(B, dtype=torch.int32, device=x.device)
        else:
            raise ValueError(f"cannot broadcast {S} fast-weight states over batch {B}")
    if state_index is not None:
        state_index = state_index.to(device=x.device, dtype=torch.int32).contiguous()
    act = x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    if ln_prepared:
        lw, lb = ln_weight, ln_bias
    else:
        lw = ln_weight.to(act).to(torch.float32).contiguous()
        lb = ln_bias.to(act).to(torch.float32).contiguous()
    odt = out_dtype or x.dtype
    if out is None:
        out = torch.empty(B, T, d, dtype=torch.bfloat16 if odt == torch.bfloat16 else torch.float32,
                          device=x.device)
    lib = _lib.load()
    ws = workspace(lib.uttt_fast_readout_workspace(B, T, d, h), x.device, slot=1)
    st = lib.uttt_fast_readout(B, T, d, h, xb.data_ptr(), wd_kind, wu.data_ptr(), _ptr(wg), wd.data_ptr(),
                               _ptr(state_index), lw.data_ptr(), lb.data_ptr(), float(eps), out.data_ptr(),
                               _lib.DTYPE_BF16 if out.dtype == torch.bfloat16 else _lib.DTYPE_F32,
                               ws.data_ptr(), ws.numel(), _stream(x.device))
    _lib.check(st, "uttt_fast_readout")
    return out if out.dtype == odt else out.to(odt)


def swiglu_fast_forward(x, w_up, w_gate, w_down, ln_weight, ln_bias, eps=1e-5):
    """Drop-in for ``swiglu_fast_forward`` (``model/uttt_layer.py:211-247``)."""
    return fast_readout(x, w_up, w_gate, w_down, ln_weight, ln_bias, eps)


def swiglu_packed_forward(x, packed_up_gate, w_down, ln_weight, ln_bias, eps=1e-5):
    """Drop-in for ``swiglu_packed_forward`` (``model/uttt_layer.py:250-257``)."""
    return fast_readout(x, packed_up_gate.to(torch.bfloat16), None, w_down.to(torch.bfloat16), ln_weight,
                        ln_bias, eps, packed=True)


def inference_read_weights(w_up, w_gate, w_down, dtype=torch.bfloat16):
    """BF16 read copies ``cat(w_up, w_gate)`` and ``w_down`` (``model/uttt_layer.py:648-668``)."""
    return torch.cat((w_up.to(dtype), w_gate.to(dtype)), dim=-1).contiguous(), w_down.to(dtype).contiguous()

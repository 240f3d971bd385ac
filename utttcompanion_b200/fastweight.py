"""Tensor-level mirror of the reference's fast-weight operator functions.

Same names, positional signatures, return values and error behaviour as
``model/uttt_layer.py`` of Phova/uTTTCompanion, so that
``setattr(model.uttt_layer, name, fn)`` (the plug-in mechanism the reference
itself uses, ``engine/personalizer.py:221-233``) swaps them in.  Every call
runs the sm_100a kernels of ``libuttt_b200.so``; there is no CPU path:
CPU tensors raise ``ValueError``.
"""

from __future__ import annotations

import ctypes
import threading
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int, int], torch.Tensor] = {}
# Every buffer ever handed out stays allocated: a captured CUDA graph keeps the
# raw pointers of the workspaces it was recorded with, so a buffer outgrown by
# a later, larger call must not return to the allocator while a graph could
# still replay into it.
_retired: Dict[Tuple[int, int, int], list] = {}


def workspace(nbytes: int, device: torch.device, slot: int = 0) -> torch.Tensor:
    """A cached, zero-initialised device workspace of at least ``nbytes`` (per device, slot and
    current stream, so work queued on different streams never shares scratch).

    Growing a slot allocates a new buffer (at least twice the old size) and keeps
    the old one alive for the life of the process, so pointers captured by CUDA
    graphs stay valid."""
    dev = device.index if device.index is not None else torch.cuda.current_device()
    key = (dev, slot, torch.cuda.current_stream(dev).cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 20, 0 if ws is None else 2 * ws.numel())
            if ws is not None:
                _retired.setdefault(key, []).append(ws)
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and (not isinstance(t, torch.Tensor) or not t.is_cuda):
            raise ValueError("uTTT B200 ops need CUDA tensors (no CPU fallback)")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def check_status(ws: torch.Tensor, what: str) -> None:
    """Synchronise and raise if a bounded device wait expired during ``what``."""
    lib = _lib.load()
    st = lib.uttt_read_status(ws.data_ptr(), 1, _stream(ws.device))
    if st != 0:
        _lib.check(st, what)


def chunk_write(k: torch.Tensor, v: torch.Tensor, eta: torch.Tensor, alpha: torch.Tensor,
                w_up: torch.Tensor, w_gate: torch.Tensor, w_down: torch.Tensor,
                s_up: torch.Tensor, s_gate: torch.Tensor, s_down: torch.Tensor,
                ln_weight: torch.Tensor, ln_bias: torch.Tensor, token_mask: Optional[torch.Tensor],
                momentum_beta: float, max_inner_grad_norm: float, normalize_by_dim: bool, eps: float,
                chunk_size: int = 64, chunk_begin: int = 0, n_chunks: Optional[int] = None,
                out: Optional[torch.Tensor] = None, token_loss: Optional[torch.Tensor] = None,
                clip_scale: Optional[torch.Tensor] = None, state_rows: Optional[torch.Tensor] = None,
                partial_sum=None, guard=None) -> None:
    """In-place multi-chunk write over ``(B, T, d)`` BF16 keys/values.

    Applies ``n_chunks`` consecutive chunk steps (``SharedFastWeightPool.chunk_step``
    chained by ``uTTTLayer.forward``, ``model/uttt_layer.py:1447-1475``) to FP32
    masters ``w_*``/``s_*`` in place.  ``out`` (optional) receives ``v_hat``,
    which is the readout f_W(k) when the caller reads with q = k.
    ``state_rows`` (int32 (B,), distinct): row b updates state ``state_rows[b]``
    of masters holding any number of states (ragged batches); by default row b
    updates state b.  ``partial_sum`` (hidden split): the masters are this
    rank's slices of the hidden units and ``partial_sum(t)`` must replace the
    FP32 tensor ``t`` by its sum over the ranks (e.g. ``HiddenSplit.all_reduce``);
    it is called between launches for every chunk's partial Z and, with
    clipping, the squared gradient norms.
    ``guard`` = (w_up0, w_gate0, w_down0, anchor_lambda, final_rows, drift_sums): the stability
    guard folded into the write (``uttt_chunk_write_guarded``): on the last chunk, rows with
    ``final_rows[b] != 0`` (int32 (B,)) are pulled towards W_0 right after their update and
    ``drift_sums`` (FP32 (B, 4), zero on entry) receives each pulled matrix's ||W - W0||^2.
    """
    _require_cuda(k, v, eta, alpha, w_up, w_gate, w_down, s_up, s_gate, s_down, ln_weight, ln_bias, token_mask,
                  state_rows)
    B, T, d = k.shape
    h = w_up.shape[-1]
    S = w_up.shape[0]
    for t in (w_up, w_gate, w_down, s_up, s_gate, s_down):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("fast-weight masters must be contiguous FP32")
    if w_up.shape != (S, d, h) or w_gate.shape != (S, d, h) or w_down.shape != (S, h, d):
        raise ValueError("fast-weight shapes must be (S,d,h),(S,d,h),(S,h,d)")
    if state_rows is None:
        if S != B:
            raise ValueError(f"{S} fast-weight states for {B} rows: pass state_rows")
    else:
        if state_rows.dtype != torch.int32 or state_rows.numel() != B or not state_rows.is_contiguous():
            raise ValueError("state_rows must be a contiguous int32 tensor with one entry per row")
    for t in (s_up, s_gate, s_down):
        if t.shape[0] != S:
            raise ValueError("momentum buffers must hold as many states as the masters")
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or not k.is_contiguous() or not v.is_contiguous():
        raise ValueError("k and v must be contiguous BF16 (B, T, d)")
    if n_chunks is None:
        n_chunks = (T - chunk_begin * chunk_size + chunk_size - 1) // chunk_size
    lib = _lib.load()
    need = lib.uttt_chunk_write_workspace(B, chunk_size, d, h)
    ws = workspace(need, k.device)
    out_dtype = _lib.DTYPE_F32
    if out is not None:
        out_dtype = _lib.DTYPE_BF16 if out.dtype == torch.bfloat16 else _lib.DTYPE_F32
    hook = None
    if partial_sum is not None:
        base = ws.data_ptr()

        def _sum(ptr, count, ctx, stream):
            try:
                off = ptr - base
                partial_sum(ws[off:off + 4 * count].view(torch.float32))
                return 0
            except Exception:                           # reported as UTTT_ERR_CUDA by the call
                import traceback
                traceback.print_exc()
                return 1
        hook = _lib.PARTIAL_SUM_FN(_sum)
    if guard is not None:
        if partial_sum is not None or out is not None or clip_scale is not None:
            raise ValueError("the guarded write takes no hidden split, readout or clip-scale output")
        w0u, w0g, w0d, lam, final_rows, sums = guard
        for t in (w0u, w0g, w0d, sums):
            if t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("W_0 and the drift sums must be contiguous FP32")
        if final_rows.dtype != torch.int32 or final_rows.numel() != B or sums.numel() < 4 * B:
            raise ValueError("final_rows must be int32 (B,) and drift_sums (B, 4)")
        st = lib.uttt_chunk_write_guarded(
            B, T, chunk_size, d, h, chunk_begin, n_chunks, _ptr(k), _ptr(k), _ptr(v), _ptr(eta), _ptr(alpha),
            _ptr(token_mask), _ptr(w_up), _ptr(w_gate), _ptr(w_down), _ptr(s_up), _ptr(s_gate), _ptr(s_down),
            _ptr(ln_weight), _ptr(ln_bias), float(momentum_beta), float(max_inner_grad_norm),
            int(bool(normalize_by_dim)), float(eps), _ptr(token_loss), S, _ptr(state_rows), _ptr(w0u), _ptr(w0g),
            _ptr(w0d), float(lam), _ptr(final_rows), _ptr(sums), ws.data_ptr(), ws.numel(), _stream(k.device))
        _lib.check(st, "uttt_chunk_write_guarded")
        return
    st = lib.uttt_chunk_write(
        B, T, chunk_size, d, h, chunk_begin, n_chunks, _ptr(k), _ptr(k), _ptr(v), _ptr(eta), _ptr(alpha),
        _ptr(token_mask), _ptr(w_up), _ptr(w_gate), _ptr(w_down), _ptr(s_up), _ptr(s_gate), _ptr(s_down),
        _ptr(ln_weight), _ptr(ln_bias), float(momentum_beta), float(max_inner_grad_norm),
        int(bool(normalize_by_dim)), float(eps), _ptr(out), out_dtype, _ptr(token_loss), _ptr(clip_scale),
        S, _ptr(state_rows), None if hook is None else ctypes.cast(hook, ctypes.c_void_p), None, ws.data_ptr(),
        ws.numel(), _stream(k.device))
    _lib.check(st, "uttt_chunk_write")


def _as_f32_2d(t: torch.Tensor, B: int, C: int) -> torch.Tensor:
    return t.reshape(B, C).to(torch.float32).contiguous()


def fused_chunk_ttt_step(q_chunk, k_chunk, v_chunk, eta_chunk, alpha_chunk, w_up, w_gate, w_down, s_up, s_gate,
                         s_down, ln_weight, ln_bias, token_mask, momentum_beta, max_inner_grad_norm,
                         normalize_by_dim, eps, read_w_up=None, read_w_gate=None, read_w_down=None):
    """Drop-in for ``fused_chunk_ttt_step`` (``model/uttt_layer.py:414-534``), with its parameter
    names (the reference's callers pass them by keyword, ``:732``).

    Returns ``(out, w_up', w_gate', w_down', s_up', s_gate', s_down', surprise)``
    as new tensors (the inputs are not modified), FP32 masters, ``out`` in
    q's dtype.  The surprise is the reference's batch-global mean of the
    unweighted per-token loss over valid tokens.
    """
    q, k, v, eta, alpha = q_chunk, k_chunk, v_chunk, eta_chunk, alpha_chunk
    _require_cuda(q, k, v, w_up)
    B, C, d = k.shape
    if C > 64:
        raise ValueError("chunk length must be <= 64")
    if w_up.dtype == torch.float64:
        raise ValueError("FP64 masters are not supported by the B200 kernels")
    new = [t.to(torch.float32).contiguous().clone() for t in (w_up, w_gate, w_down, s_up, s_gate, s_down)]
    kb = k.to(torch.bfloat16).contiguous()
    vb = v.to(torch.bfloat16).contiguous()
    eta32 = _as_f32_2d(eta, B, C)
    alpha32 = _as_f32_2d(alpha, B, C)
    mask32 = None if token_mask is None else _as_f32_2d(token_mask, B, C)
    ln_w = ln_weight.to(torch.float32).contiguous()
    ln_b = ln_bias.to(torch.float32).contiguous()
    loss = torch.empty(B, C, dtype=torch.float32, device=k.device)
    same_read = read_w_up is None and read_w_gate is None and read_w_down is None
    fused_out = same_read and (q is k or (q.data_ptr() == k.data_ptr() and q.shape == k.shape
                                          and q.dtype == k.dtype))
    out32 = torch.empty(B, C, d, dtype=torch.float32, device=k.device) if fused_out else None
    if not fused_out:
        from .readout import swiglu_fast_forward
        out = swiglu_fast_forward(q, w_up if read_w_up is None else read_w_up,
                                  w_gate if read_w_gate is None else read_w_gate,
                                  w_down if read_w_down is None else read_w_down, ln_weight, ln_bias, eps)
    chunk_write(kb, vb, eta32, alpha32, *new, ln_w, ln_b, mask32, momentum_beta, max_inner_grad_norm,
                normalize_by_dim, eps, chunk_size=C, out=out32, token_loss=loss)
    if fused_out:
        out = out32.to(q.dtype)
    if mask32 is None:
        surprise = loss.mean()
    else:
        surprise = (loss * mask32).sum() / mask32.sum().clamp_min(1.0)
    return (out, *new, surprise)

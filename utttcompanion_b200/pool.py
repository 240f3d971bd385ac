"""Drop-ins for the rest of the reference's fast-weight operator surface.

* ``SharedFastWeightPoolB200`` -- the ``SharedFastWeightPool`` API
  (``model/uttt_layer.py:541-874``: ``init_state``, ``inference_read_weights``,
  ``forward_readout``, ``chunk_step``, ``apply_elastic_pull``, ``compute_drift``)
  over device FP32 masters, every op on this package's kernels.  It accepts
  the reference's ``FastWeightState`` or this package's ``FastState`` (any
  object with ``w_up .. ln_bias`` tensors) and returns ``FastState``.
* module functions with the reference's positional signatures:
  ``fused_fast_q_proj`` (:1175-1190), ``fused_slow_projections`` (:1193-1231),
  ``apply_rope`` (:946-958) and ``analytical_swiglu_chunk_grad`` (:279-411).
* ``install(module)`` -- the reference's own plug-in mechanism
  (``setattr`` on ``model.uttt_layer``, ``engine/personalizer.py:221-233``).
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from . import _lib
from .fastweight import _require_cuda, _stream, chunk_write, fused_chunk_ttt_step, workspace
from .model import FastState
from .readout import fast_readout, swiglu_fast_forward, swiglu_packed_forward


def _state_tensors(state):
    return tuple(getattr(state, n) for n in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down", "ln_weight",
                                              "ln_bias"))


def _as_fast_state(state) -> FastState:
    if isinstance(state, FastState):
        return state
    t = [x.to(torch.float32).contiguous() for x in _state_tensors(state)]
    return FastState(*t, int(getattr(state, "step", 0)), float(getattr(state, "last_surprise_loss", 0.0)),
                     list(getattr(state, "surprise_history", [])))


def _linear_segments(x2d: torch.Tensor, w: torch.Tensor, segs, eps: float) -> None:
    lib = _lib.load()
    M, K = x2d.shape
    N = w.shape[0]
    arr = (_lib.Segment * len(segs))(*segs)
    ws = workspace(lib.uttt_linear_workspace(M, N), x2d.device, slot=2)
    _lib.check(lib.uttt_linear(M, N, K, x2d.data_ptr(), w.data_ptr(), len(segs), arr, float(eps), ws.data_ptr(),
                               ws.numel(), _stream(x2d.device)), "uttt_linear")


def _seg(start, length, op, out, out_ld, aux=None, aux_ld=0, scale=0.0, out_f32=False):
    return _lib.Segment(start, length, op, int(out_f32), out.data_ptr(), out_ld,
                        None if aux is None else aux.data_ptr(), aux_ld, scale)


def fused_fast_q_proj(x, wq_w, q_norm_w, eps):
    """``RMSNorm(x W_q^T) * gamma_q`` (``model/uttt_layer.py:1175-1190``); BF16 out."""
    _require_cuda(x, wq_w)
    d = wq_w.shape[0]
    xb = x.to(torch.bfloat16).reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty(xb.shape[0], d, dtype=torch.bfloat16, device=x.device)
    # the segment holds only a raw pointer: the converted tensor must outlive the launch call,
    # or the allocator may hand its memory to the next allocation before the kernel is queued
    gamma = q_norm_w.to(torch.float32).contiguous()
    _linear_segments(xb, wq_w.to(torch.bfloat16).contiguous(), [_seg(0, d, _lib.SEG_RMSNORM, out, d, gamma)], eps)
    del gamma
    return out.reshape(*x.shape[:-1], d)


def fused_slow_projections(x, wq_w, wk_w, wv_w, q_norm_w, k_norm_w, w_eta_w, w_eta_b, w_alpha_w, w_alpha_b,
                           base_inner_lr, base_weight_decay, eps):
    """q, k, v, eta, alpha of a uTTTLayer (``model/uttt_layer.py:1193-1231``) as ONE packed GEMM."""
    _require_cuda(x, wq_w)
    d = wq_w.shape[0]
    xb = x.to(torch.bfloat16).reshape(-1, x.shape[-1]).contiguous()
    R = xb.shape[0]
    w = torch.cat([wq_w, wk_w, wv_w, w_eta_w, w_alpha_w]).to(torch.bfloat16).contiguous()
    q = torch.empty(R, d, dtype=torch.bfloat16, device=x.device)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    eta = torch.empty(R, 1, dtype=torch.float32, device=x.device)
    alpha = torch.empty_like(eta)
    # Segments hold raw pointers, so every converted operand is kept alive (named) until the launch
    # call has queued the kernel: a temporary freed earlier could be handed to the next conversion,
    # and two segments would then read the same memory (eta would read alpha's bias).
    gq, gk, b_eta, b_alpha = (t.to(torch.float32).contiguous() for t in (q_norm_w, k_norm_w, w_eta_b, w_alpha_b))
    _linear_segments(xb, w, [
        _seg(0, d, _lib.SEG_RMSNORM, q, d, gq),
        _seg(d, d, _lib.SEG_RMSNORM, k, d, gk),
        _seg(2 * d, d, _lib.SEG_RMSNORM, v, d),
        _seg(3 * d, 1, _lib.SEG_SIGMOID, eta, 1, b_eta, 0, base_inner_lr, out_f32=True),
        _seg(3 * d + 1, 1, _lib.SEG_SIGMOID, alpha, 1, b_alpha, 0, base_weight_decay, out_f32=True),
    ], eps)
    del gq, gk, b_eta, b_alpha
    shp = x.shape[:-1]
    return (q.reshape(*shp, d), k.reshape(*shp, d), v.reshape(*shp, d),
            eta.to(torch.bfloat16).reshape(*shp, 1), alpha.to(torch.bfloat16).reshape(*shp, 1))


def apply_rope(q, k, cos, sin):
    """Rotate-half RoPE of (B, H, T, D) q and k (``model/uttt_layer.py:946-958``)."""
    _require_cuda(q, k, cos, sin)
    lib = _lib.load()
    T, D = q.shape[-2], q.shape[-1]
    cs = cos.reshape(-1, D)[-T:].to(torch.bfloat16).contiguous()
    sn = sin.reshape(-1, D)[-T:].to(torch.bfloat16).contiguous()
    outs = []
    for x in (q, k):
        xb = x.to(torch.bfloat16).contiguous()
        out = torch.empty_like(xb)
        _lib.check(lib.uttt_apply_rope(xb.numel() // D, T, D, xb.data_ptr(), cs.data_ptr(), sn.data_ptr(),
                                       out.data_ptr(), _stream(x.device)), "uttt_apply_rope")
        outs.append(out.to(x.dtype))
    return outs[0], outs[1]


def analytical_swiglu_chunk_grad(k_chunk, v_chunk, eta_chunk, w_up, w_gate, w_down, ln_weight, ln_bias,
                                 token_mask=None, normalize_by_dim=False, eps=1e-5):
    """Drop-in for ``analytical_swiglu_chunk_grad`` (``model/uttt_layer.py:279-411``).

    The B200 write never materialises gradients (they are consumed inside the
    update epilogue), so this runs the same kernels on a scratch copy with no
    decay, no momentum and no clipping: the written momentum is then -grad.
    Gradients are returned in FP32 (the reference returns them in the
    activation dtype); the surprise is the batch-global mean.
    """
    _require_cuda(k_chunk, w_up)
    B, C, d = k_chunk.shape
    W = [t.to(torch.float32).contiguous().clone() for t in (w_up, w_gate, w_down)]
    S = [torch.zeros_like(t) for t in W]
    eta = eta_chunk.reshape(B, C).to(torch.float32).contiguous()
    alpha = torch.zeros_like(eta)
    mask = None if token_mask is None else token_mask.reshape(B, C).to(torch.float32).contiguous()
    loss = torch.empty(B, C, dtype=torch.float32, device=k_chunk.device)
    chunk_write(k_chunk.to(torch.bfloat16).contiguous(), v_chunk.to(torch.bfloat16).contiguous(), eta, alpha, *W,
                *S, ln_weight.to(torch.float32).contiguous(), ln_bias.to(torch.float32).contiguous(), mask, 0.0, 0.0,
                normalize_by_dim, eps, chunk_size=C, token_loss=loss)
    surprise = loss.mean() if mask is None else (loss * mask).sum() / mask.sum().clamp_min(1.0)
    return -S[0], -S[1], -S[2], surprise


class SharedFastWeightPoolB200:
    """``SharedFastWeightPool`` on the B200 kernels (same method names and returns)."""

    def __init__(self, w_up_init, w_gate_init, w_down_init, ln_weight, ln_bias, momentum_beta=0.90,
                 max_inner_grad_norm=1.0, normalize_loss_by_dim=False, rms_norm_eps=1e-5, device="cuda"):
        f32 = lambda t: torch.as_tensor(t).to(device=device, dtype=torch.float32).contiguous()  # noqa: E731
        self.w_up_init, self.w_gate_init, self.w_down_init = f32(w_up_init), f32(w_gate_init), f32(w_down_init)
        self.ln_weight, self.ln_bias = f32(ln_weight), f32(ln_bias)
        self.d_model, self.d_ff = self.w_up_init.shape
        self.momentum_beta = momentum_beta
        self.max_inner_grad_norm = max_inner_grad_norm
        self.normalize_loss_by_dim = normalize_loss_by_dim
        self.eps = rms_norm_eps
        self.device = torch.device(device)

    @classmethod
    def from_reference(cls, pool, device="cuda") -> "SharedFastWeightPoolB200":
        """Wrap a reference ``SharedFastWeightPool`` module's W_0 and settings."""
        return cls(pool.w_up_init.detach(), pool.w_gate_init.detach(), pool.w_down_init.detach(),
                   pool.ln_weight.detach(), pool.ln_bias.detach(), pool.momentum_beta, pool.max_inner_grad_norm,
                   pool.normalize_loss_by_dim, pool.eps, device)

    def init_state(self, batch_size: int = 1, device=None, dtype=None, detach: bool = True) -> FastState:
        """Independent copies of W_0 with zero momentum (``:582-630``); FP32 masters."""
        rep = [w.unsqueeze(0).expand(batch_size, *w.shape).contiguous()
               for w in (self.w_up_init, self.w_gate_init, self.w_down_init)]
        return FastState(*rep, *(torch.zeros_like(t) for t in rep), self.ln_weight.clone(), self.ln_bias.clone())

    def inference_read_weights(self, state, dtype=torch.bfloat16, device=None):
        """BF16 read copies ``cat(w_up, w_gate)``, ``w_down`` (``:648-668``), packed by a kernel."""
        st = _as_fast_state(state)
        S, d, h = st.w_up.shape
        lib = _lib.load()
        packed = torch.empty(S, d, 2 * h, dtype=torch.bfloat16, device=st.w_up.device)
        down = torch.empty(S, h, d, dtype=torch.bfloat16, device=st.w_up.device)
        _lib.check(lib.uttt_pack_read_copies(S, d, h, st.w_up.data_ptr(), st.w_gate.data_ptr(), st.w_down.data_ptr(),
                                             packed.data_ptr(), down.data_ptr(), _stream(st.w_up.device)),
                   "uttt_pack_read_copies")
        return packed, down

    def forward_readout(self, x, state):
        """``f_W(x)`` through the state's frozen weights (``:670-695``)."""
        st = _as_fast_state(state)
        return swiglu_fast_forward(x, st.w_up, st.w_gate, st.w_down, st.ln_weight, st.ln_bias, self.eps)

    def chunk_step(self, state, q_chunk, k_chunk, v_chunk, eta_chunk, alpha_chunk, token_mask=None,
                   update_fast_weights=True, read_state=None):
        """One chunk write (``:697-771``): returns ``(out, new_state, surprise)``."""
        st = _as_fast_state(state)
        rs = st if read_state is None else _as_fast_state(read_state)
        if not update_fast_weights:
            out = self.forward_readout(q_chunk, rs)
            return out, st, q_chunk.new_zeros((), dtype=torch.float32)
        res = fused_chunk_ttt_step(q_chunk, k_chunk, v_chunk, eta_chunk, alpha_chunk, st.w_up, st.w_gate, st.w_down,
                                   st.s_up, st.s_gate, st.s_down, st.ln_weight, st.ln_bias, token_mask,
                                   self.momentum_beta, float(self.max_inner_grad_norm or 0.0),
                                   self.normalize_loss_by_dim, self.eps,
                                   None if read_state is None else rs.w_up,
                                   None if read_state is None else rs.w_gate,
                                   None if read_state is None else rs.w_down)
        new = FastState(*res[1:7], st.ln_weight, st.ln_bias, st.step + 1, st.last_surprise_loss,
                        st.surprise_history)
        return res[0], new, res[7]

    def apply_elastic_pull(self, state, anchor_lambda: float = 0.02,
                           max_drift_ratio: Optional[float] = None) -> FastState:
        """Elastic pull (+ drift clamp) toward W_0 (``:773-832``), as a new state."""
        st = _as_fast_state(state)
        if anchor_lambda <= 0.0 and max_drift_ratio is None:
            return st
        w = [t.clone() for t in (st.w_up, st.w_gate, st.w_down)]
        B, d, h = w[0].shape
        lib = _lib.load()
        ws = workspace(lib.uttt_guard_workspace(B), w[0].device, slot=3)
        ratio = float(max_drift_ratio) if (max_drift_ratio is not None and max_drift_ratio > 0.0) else 0.0
        _lib.check(lib.uttt_elastic_pull(B, d, h, w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(),
                                         self.w_up_init.data_ptr(), self.w_gate_init.data_ptr(),
                                         self.w_down_init.data_ptr(), float(anchor_lambda), ratio, ws.data_ptr(),
                                         ws.numel(), _stream(w[0].device)), "uttt_elastic_pull")
        return FastState(*w, st.s_up, st.s_gate, st.s_down, st.ln_weight, st.ln_bias, st.step,
                         st.last_surprise_loss, list(st.surprise_history))

    def compute_drift(self, state) -> Dict[str, float]:
        """Frobenius drift from W_0 (``:834-874``), one host sync."""
        st = _as_fast_state(state)
        B, d, h = st.w_up.shape
        lib = _lib.load()
        out = torch.empty(4 * B + 4, dtype=torch.float32, device=st.w_up.device)
        _lib.check(lib.uttt_drift_sums(B, d, h, st.w_up.data_ptr(), st.w_gate.data_ptr(), st.w_down.data_ptr(),
                                       self.w_up_init.data_ptr(), self.w_gate_init.data_ptr(),
                                       self.w_down_init.data_ptr(), out.data_ptr(), _stream(st.w_up.device)),
                   "uttt_drift_sums")
        v = out.double().tolist()
        d_up = math.sqrt(sum(v[4 * b + 0] for b in range(B)))
        d_gate = math.sqrt(sum(v[4 * b + 1] for b in range(B)))
        d_down = math.sqrt(sum(v[4 * b + 2] for b in range(B)))
        b_up, b_gate, b_down = (math.sqrt(v[4 * B + m]) for m in range(3))
        total = math.sqrt(d_up ** 2 + d_gate ** 2 + d_down ** 2)
        base = math.sqrt(b_up ** 2 + b_gate ** 2 + b_down ** 2) + 1e-8
        return {
            "drift_frobenius": total, "base_frobenius": base, "drift_pct": total / base * 100.0,
            "w_up_drift": d_up, "w_gate_drift": d_gate, "w_down_drift": d_down,
            "w_up_drift_pct": d_up / (b_up + 1e-8) * 100.0,
            "w_gate_drift_pct": d_gate / (b_gate + 1e-8) * 100.0,
            "w_down_drift_pct": d_down / (b_down + 1e-8) * 100.0,
            "step": st.step, "last_surprise_loss": st.last_surprise_loss,
        }


DROP_INS = {
    "fused_chunk_ttt_step": fused_chunk_ttt_step,
    "analytical_swiglu_chunk_grad": analytical_swiglu_chunk_grad,
    "swiglu_fast_forward": swiglu_fast_forward,
    "swiglu_packed_forward": swiglu_packed_forward,
    "fused_fast_q_proj": fused_fast_q_proj,
    "fused_slow_projections": fused_slow_projections,
    "apply_rope": apply_rope,
}


def install(uttt_layer_module) -> Dict[str, object]:
    """``setattr`` the B200 drop-ins onto the reference's ``model.uttt_layer``
    module (its own plug-in mechanism); returns the replaced originals."""
    replaced = {}
    for name, fn in DROP_INS.items():
        if hasattr(uttt_layer_module, name):
            replaced[name] = getattr(uttt_layer_module, name)
        setattr(uttt_layer_module, name, fn)
    return replaced

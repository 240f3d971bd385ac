"""Oracle restatement of the shared fast-weight operator (numpy).

Reference: ``model/uttt_layer.py`` of Phova/uTTTCompanion.

Array conventions follow the reference exactly: ``x, k, v, q`` are
``(B, T, d)``; ``w_up, w_gate`` are ``(B, d, h)``; ``w_down`` is
``(B, h, d)``; ``ln_weight, ln_bias`` are ``(d,)``; ``eta, alpha`` are
``(B, T, 1)``; ``token_mask`` is ``(B, T)`` float or None.

``prec`` selects the activation rounding (see ``numerics.Precision``):
``bf16`` reproduces the dtype flow of the reference when its activations are
BF16 and its master state FP32, which is how ``fused_chunk_ttt_step`` is
called on the serving path.  ``autocast=True`` reproduces the same op under
``torch.autocast`` (LayerNorm then returns FP32 and the residual add is FP32).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from .numerics import Precision, round_bf16, sigmoid, silu


def _as(prec: Precision, x):
    return np.asarray(x, dtype=prec.dtype)


def _read_weight(prec: Precision, w):
    """``w.to(dtype=orig_dtype)`` -- ``model/uttt_layer.py:237-239,345-347``."""
    return prec.act(w)


def _layer_norm(z, weight, bias, eps, stat_dtype):
    """``F.layer_norm`` over the last dim with biased variance."""
    z = np.asarray(z, dtype=stat_dtype)
    mean = z.mean(axis=-1, keepdims=True)
    diff = z - mean
    var = np.square(diff).mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + stat_dtype(eps))
    return diff * rstd * np.asarray(weight, stat_dtype) + np.asarray(bias, stat_dtype)


def swiglu_fast_forward(x, w_up, w_gate, w_down, ln_weight, ln_bias, eps=1e-5,
                        prec: Precision = Precision("f32"), autocast: bool = False):
    """``f_W(x) = x + LN(silu(x W_gate) * (x W_up) W_down)``.

    Follows ``model/uttt_layer.py:211-247`` (and ``swiglu_packed_forward``
    250-257, which is the same function of packed read copies).
    """
    x = prec.act(x)
    u = prec.mm(x, _read_weight(prec, w_up))                        # :239
    g = prec.mm(x, _read_weight(prec, w_gate))                      # :240
    h = prec.act(prec.act(silu(g)) * u)                            # :241
    z = prec.mm(h, _read_weight(prec, w_down))                      # :242
    lw = prec.act(ln_weight)                                       # ln_weight.to(orig_dtype)
    lb = prec.act(ln_bias)
    ln = _layer_norm(z, lw, lb, eps, prec.stat_dtype)              # :244-246
    if prec.mode == "bf16" and autocast:
        return np.asarray(x, np.float32) + ln                      # FP32 under autocast
    return prec.act(x + prec.act(ln))                              # :247


@dataclass
class ChunkGrad:
    grad_w_up: np.ndarray
    grad_w_gate: np.ndarray
    grad_w_down: np.ndarray
    surprise: float
    # per-state pieces (no counterpart in the reference's return value; they
    # let a batched engine recombine the reference's batch-global mean)
    token_loss: Optional[np.ndarray] = None


def analytical_swiglu_chunk_grad(k, v, eta, w_up, w_gate, w_down, ln_weight, ln_bias,
                                 token_mask=None, normalize_by_dim=False, eps=1e-5,
                                 prec: Precision = Precision("f32")) -> ChunkGrad:
    """Closed-form gradient of the per-token weighted MSE surprise loss.

    Follows ``model/uttt_layer.py:279-411`` step by step (line numbers in
    the comments).
    """
    cdt = prec.stat_dtype
    k = prec.act(k)
    bsz, chunk_len, dim = k.shape
    wu = _read_weight(prec, w_up)                                  # :345
    wg = _read_weight(prec, w_gate)                                # :346
    wd = _read_weight(prec, w_down)                                # :347
    u = prec.mm(k, wu)                                             # :348
    g = prec.mm(k, wg)                                             # :349
    h = prec.act(prec.act(silu(g)) * u)                            # :350
    z = prec.mm(h, wd)                                             # :352

    z32 = np.asarray(z, cdt)                                       # :355
    mean = z32.mean(axis=-1, keepdims=True)                        # :356
    diff = z32 - mean                                              # :357
    var = np.square(diff).mean(axis=-1, keepdims=True)             # :358
    rstd = 1.0 / np.sqrt(var + cdt(eps))                           # :359
    z_hat = diff * rstd                                            # :360

    gamma = np.asarray(ln_weight, cdt).reshape(1, 1, dim)          # :362
    beta = np.asarray(ln_bias, cdt).reshape(1, 1, dim)             # :363
    v_hat = np.asarray(k, cdt) + (z_hat * gamma + beta)            # :364

    err = v_hat - np.asarray(prec.act(v), cdt)                     # :367
    inv_scale = cdt(1.0 / float(dim)) if normalize_by_dim else cdt(1.0)   # :368
    token_loss = cdt(0.5) * np.square(err).sum(axis=-1) * inv_scale       # :369

    eta_c = np.asarray(eta, cdt)
    if token_mask is not None:                                     # :371-375
        m = np.asarray(token_mask, cdt)
        valid_counts = np.maximum(m.sum(axis=-1, keepdims=True), cdt(1.0))
        surprise = (token_loss * m).sum() / max(m.sum(), cdt(1.0))
        weight_factor = (eta_c * m[..., None]) / valid_counts[..., None]
    else:                                                          # :376-378
        surprise = token_loss.mean()
        weight_factor = eta_c * cdt(1.0 / float(chunk_len))

    dz_hat = (weight_factor * inv_scale) * err * gamma             # :383
    mean_dz_hat = dz_hat.mean(axis=-1, keepdims=True)              # :385
    mean_dz_hat_z = (dz_hat * z_hat).mean(axis=-1, keepdims=True)  # :386
    delta_z = prec.act(rstd * (dz_hat - mean_dz_hat - z_hat * mean_dz_hat_z))  # :387

    grad_w_down = prec.mm(np.swapaxes(h, 1, 2), delta_z)           # :391
    delta_h = prec.mm(delta_z, np.swapaxes(wd, 1, 2))              # :393

    g32 = np.asarray(g, cdt)                                       # :396
    u32 = np.asarray(u, cdt)
    dh32 = np.asarray(delta_h, cdt)
    sigma_g = sigmoid(g32)                                         # :399
    delta_u = prec.act(dh32 * (g32 * sigma_g))                     # :400
    dsilu = sigma_g * (cdt(1.0) + g32 * (cdt(1.0) - sigma_g))      # :401
    delta_g = prec.act(dh32 * u32 * dsilu)                         # :402

    kt = np.swapaxes(k, 1, 2)                                      # :405
    grad_w_up = prec.mm(kt, delta_u)                               # :406
    grad_w_gate = prec.mm(kt, delta_g)                             # :407
    return ChunkGrad(grad_w_up, grad_w_gate, grad_w_down, float(surprise), token_loss)


@dataclass
class ChunkStep:
    out: np.ndarray
    w_up: np.ndarray
    w_gate: np.ndarray
    w_down: np.ndarray
    s_up: np.ndarray
    s_gate: np.ndarray
    s_down: np.ndarray
    surprise: float
    token_loss: Optional[np.ndarray] = None
    clip_scale: Optional[np.ndarray] = None
    alpha_bar: Optional[np.ndarray] = None


def fused_chunk_ttt_step(q, k, v, eta, alpha, w_up, w_gate, w_down, s_up, s_gate, s_down,
                         ln_weight, ln_bias, token_mask, momentum_beta, max_inner_grad_norm,
                         normalize_by_dim, eps, read_w_up=None, read_w_gate=None,
                         read_w_down=None, prec: Precision = Precision("f32"),
                         autocast: bool = False) -> ChunkStep:
    """Gradient + per-state Frobenius clip + momentum + decay + readout.

    Follows ``model/uttt_layer.py:414-534``.
    """
    grads = analytical_swiglu_chunk_grad(
        k, v, eta, w_up, w_gate, w_down, ln_weight, ln_bias, token_mask,
        normalize_by_dim, eps, prec)
    mdt = np.float64 if np.asarray(w_up).dtype == np.float64 else np.float32   # :467
    bsz = np.asarray(w_up).shape[0]
    gu = np.asarray(grads.grad_w_up, mdt)
    gg = np.asarray(grads.grad_w_gate, mdt)
    gd = np.asarray(grads.grad_w_down, mdt)
    if max_inner_grad_norm > 0.0:                                   # :468-485
        norm_sq = (np.square(gu).sum(axis=(1, 2)) + np.square(gg).sum(axis=(1, 2))
                   + np.square(gd).sum(axis=(1, 2)))
        clip = np.minimum(mdt(max_inner_grad_norm) / np.sqrt(norm_sq + mdt(1e-8)), mdt(1.0))
        clip = clip.astype(mdt).reshape(bsz, 1, 1)
        step_up, step_gate, step_down = gu * clip, gg * clip, gd * clip
    else:                                                           # :486-489
        clip = np.ones((bsz, 1, 1), mdt)
        step_up, step_gate, step_down = gu, gg, gd

    beta = mdt(momentum_beta)
    s_up_new = beta * np.asarray(s_up, mdt) - step_up               # :493-499
    s_gate_new = beta * np.asarray(s_gate, mdt) - step_gate
    s_down_new = beta * np.asarray(s_down, mdt) - step_down

    a = np.asarray(alpha, mdt)
    if token_mask is None:                                          # :501-502
        alpha_bar = a.mean(axis=1, keepdims=True)
    else:                                                           # :503-506
        m = np.asarray(token_mask, mdt)[..., None]
        alpha_bar = (a * m).sum(axis=1, keepdims=True) / np.maximum(m.sum(axis=1, keepdims=True), mdt(1))
    decay = mdt(1.0) - alpha_bar                                    # :507

    w_up_new = decay * np.asarray(w_up, mdt) + s_up_new             # :509-511
    w_gate_new = decay * np.asarray(w_gate, mdt) + s_gate_new
    w_down_new = decay * np.asarray(w_down, mdt) + s_down_new

    if token_mask is not None:                                      # :513-520
        active = (np.asarray(token_mask) != 0).any(axis=1).reshape(bsz, 1, 1)
        w_up_new = np.where(active, w_up_new, w_up).astype(mdt)
        w_gate_new = np.where(active, w_gate_new, w_gate).astype(mdt)
        w_down_new = np.where(active, w_down_new, w_down).astype(mdt)
        s_up_new = np.where(active, s_up_new, s_up).astype(mdt)
        s_gate_new = np.where(active, s_gate_new, s_gate).astype(mdt)
        s_down_new = np.where(active, s_down_new, s_down).astype(mdt)

    out = swiglu_fast_forward(                                      # :525-533
        q,
        w_up if read_w_up is None else read_w_up,
        w_gate if read_w_gate is None else read_w_gate,
        w_down if read_w_down is None else read_w_down,
        ln_weight, ln_bias, eps, prec, autocast)
    return ChunkStep(out, w_up_new, w_gate_new, w_down_new, s_up_new, s_gate_new, s_down_new,
                     grads.surprise, grads.token_loss, clip.reshape(bsz), alpha_bar.reshape(bsz))


# ------------------------------------------------------------------------------
# Pool-level helpers
# ------------------------------------------------------------------------------

@dataclass
class OracleState:
    """Mirror of ``FastWeightState`` (``model/uttt_layer.py:59-204``)."""
    w_up: np.ndarray
    w_gate: np.ndarray
    w_down: np.ndarray
    s_up: np.ndarray
    s_gate: np.ndarray
    s_down: np.ndarray
    ln_weight: np.ndarray
    ln_bias: np.ndarray
    step: int = 0
    last_surprise_loss: float = 0.0
    surprise_history: List[float] = field(default_factory=list)

    def copy(self) -> "OracleState":
        return OracleState(self.w_up.copy(), self.w_gate.copy(), self.w_down.copy(),
                           self.s_up.copy(), self.s_gate.copy(), self.s_down.copy(),
                           self.ln_weight.copy(), self.ln_bias.copy(), int(self.step),
                           float(self.last_surprise_loss), list(self.surprise_history))


def init_state(w_up0, w_gate0, w_down0, ln_w, ln_b, batch_size=1, dtype=np.float32) -> OracleState:
    """``SharedFastWeightPool.init_state`` (``model/uttt_layer.py:582-630``)."""
    def rep(w):
        return np.repeat(np.asarray(w, dtype)[None], batch_size, axis=0)
    up, gate, down = rep(w_up0), rep(w_gate0), rep(w_down0)
    return OracleState(up, gate, down, np.zeros_like(up), np.zeros_like(gate), np.zeros_like(down),
                       np.asarray(ln_w, dtype).copy(), np.asarray(ln_b, dtype).copy())


def inference_read_weights(w_up, w_gate, w_down):
    """BF16 read copies ``cat(w_up, w_gate)`` and ``w_down`` (``model/uttt_layer.py:648-668``)."""
    return (round_bf16(np.concatenate([w_up, w_gate], axis=-1)), round_bf16(w_down))


def apply_elastic_pull(w_up, w_gate, w_down, w_up0, w_gate0, w_down0,
                       anchor_lambda=0.02, max_drift_ratio=None):
    """Slow-anchor pull + optional drift clamp (``model/uttt_layer.py:773-832``)."""
    if anchor_lambda <= 0.0 and max_drift_ratio is None:
        return w_up, w_gate, w_down
    dt = np.asarray(w_up).dtype
    lam = dt.type(anchor_lambda)
    one = dt.type(1.0)
    u0, g0, d0 = (np.asarray(w, dt)[None] for w in (w_up0, w_gate0, w_down0))
    up = (one - lam) * w_up + lam * u0                              # :799-801
    gate = (one - lam) * w_gate + lam * g0
    down = (one - lam) * w_down + lam * d0
    if max_drift_ratio is not None and max_drift_ratio > 0.0:       # :803-818
        f = np.float32 if dt != np.float64 else np.float64
        base_norm = np.sqrt(np.square(u0.astype(f)).sum() + np.square(g0.astype(f)).sum()
                            + np.square(d0.astype(f)).sum() + f(1e-8))
        du, dg, dd = up - u0, gate - g0, down - d0
        drift = np.sqrt(np.square(du.astype(f)).sum(axis=(1, 2), keepdims=True)
                        + np.square(dg.astype(f)).sum(axis=(1, 2), keepdims=True)
                        + np.square(dd.astype(f)).sum(axis=(1, 2), keepdims=True) + f(1e-8))
        scale = np.minimum(f(max_drift_ratio) * base_norm / drift, f(1.0)).astype(dt)
        up, gate, down = u0 + du * scale, g0 + dg * scale, d0 + dd * scale
    return up, gate, down


def compute_drift(w_up, w_gate, w_down, w_up0, w_gate0, w_down0):
    """Frobenius drift report (``model/uttt_layer.py:834-874``)."""
    f = np.float64
    d_up = float(np.linalg.norm((np.asarray(w_up, np.float32) - np.asarray(w_up0, np.float32)[None]).astype(f)))
    d_gate = float(np.linalg.norm((np.asarray(w_gate, np.float32) - np.asarray(w_gate0, np.float32)[None]).astype(f)))
    d_down = float(np.linalg.norm((np.asarray(w_down, np.float32) - np.asarray(w_down0, np.float32)[None]).astype(f)))
    b_up = float(np.linalg.norm(np.asarray(w_up0, f)))
    b_gate = float(np.linalg.norm(np.asarray(w_gate0, f)))
    b_down = float(np.linalg.norm(np.asarray(w_down0, f)))
    total = (d_up ** 2 + d_gate ** 2 + d_down ** 2) ** 0.5
    base = (b_up ** 2 + b_gate ** 2 + b_down ** 2) ** 0.5 + 1e-8
    return {
        "drift_frobenius": total, "base_frobenius": base, "drift_pct": total / base * 100.0,
        "w_up_drift": d_up, "w_gate_drift": d_gate, "w_down_drift": d_down,
        "w_up_drift_pct": d_up / (b_up + 1e-8) * 100.0,
        "w_gate_drift_pct": d_gate / (b_gate + 1e-8) * 100.0,
        "w_down_drift_pct": d_down / (b_down + 1e-8) * 100.0,
    }

"""Numeric helpers for the oracle: BF16 rounding emulation and precision modes.

The reference computes its GPU path in BF16 activations with FP32 master
state (``model/uttt_layer.py:343-409`` rounds every bmm output to the
activation dtype; ``:467-511`` does the update in FP32).  numpy has no
bfloat16, so ``round_bf16`` reproduces ``tensor.to(torch.bfloat16)``
(round-to-nearest-even on the upper 16 bits of the FP32 pattern).
"""

from __future__ import annotations

import numpy as np


def round_bf16(x) -> np.ndarray:
    """Round an array to bfloat16 precision (RNE), returned as float32.

    Same rounding as ``torch.Tensor.to(torch.bfloat16)`` for finite values;
    NaN stays NaN.
    """
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits(x) -> np.ndarray:
    """Return the uint16 bfloat16 bit patterns of ``round_bf16(x)``."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    """Inverse of :func:`bf16_bits`."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


class Precision:
    """How the oracle rounds activations.

    ``f64`` / ``f32``: every op in that dtype (the reference run with FP64 or
    FP32 tensors).  ``bf16``: activations are rounded to BF16 after every
    op whose PyTorch output dtype is BF16 in the reference's BF16 path, while
    statistics and master state stay FP32.
    """

    def __init__(self, mode: str):
        if mode not in ("f64", "f32", "bf16"):
            raise ValueError(f"unknown precision mode {mode!r}")
        self.mode = mode
        self.dtype = np.float64 if mode == "f64" else np.float32
        self.stat_dtype = np.float64 if mode == "f64" else np.float32

    def act(self, x):
        """Round to the activation dtype (identity except in bf16 mode)."""
        if self.mode == "bf16":
            return round_bf16(x)
        return np.asarray(x, dtype=self.dtype)

    def mm(self, a, b):
        """Matmul with activation-dtype output (BF16 bmm accumulates in FP32)."""
        a = np.asarray(a, dtype=self.dtype)
        b = np.asarray(b, dtype=self.dtype)
        return self.act(np.matmul(a, b))

    def __repr__(self):  # pragma: no cover
        return f"Precision({self.mode})"


def silu(x):
    x = np.asarray(x)
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    x = np.asarray(x)
    return 1.0 / (1.0 + np.exp(-x))


def rel_l2(a, b) -> float:
    """||a-b|| / max(||b||, tiny), computed in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = max(float(np.linalg.norm(b)), 1e-30)
    return float(np.linalg.norm(a - b)) / den

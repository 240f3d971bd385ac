"""CPU: the identity the clip-norm pass is built on.

The norm pass forms the squared Frobenius norm of each weight gradient without the
gradient: for K (C x d) and a hidden tile's dU (C x 128),
||K^T dU||_F^2 = <K K^T, dU dU^T> summed over the C x C token pairs, and likewise
||H^T dZ||_F^2 = <H H^T, dZ dZ^T>.  The kernels (``chunk_gram_kernel`` for K K^T and
dZ dZ^T per row, two tensor-core MMAs per hidden tile for dU^T dU + dG^T dG and H^T H)
sum the tile terms over the hidden tiles; this checks that decomposition, with padded
token columns and a ragged last tile, against the gradients of the oracle's analytical
chunk gradient (model/uttt_layer.py:391-407)."""

import numpy as np

from oracle import fastweight as ofw
from oracle.numerics import Precision


def _tiles(h, ht=128):
    return [(j, min(j + ht, h)) for j in range(0, h, ht)]


def test_gram_norm_equals_gradient_norm_over_hidden_tiles():
    rng = np.random.default_rng(3)
    C, d, h = 64, 256, 320                       # a ragged last hidden tile (320 = 2 x 128 + 64)
    valid = 50                                   # padded token columns carry zero dU, dG and dZ
    K = rng.standard_normal((C, d))
    dU = rng.standard_normal((C, h))
    dG = rng.standard_normal((C, h))
    H = rng.standard_normal((C, h))
    dZ = rng.standard_normal((C, d))
    for t in (dU, dG, H, dZ):
        t[valid:] = 0.0
    direct = (np.square(K.T @ dU).sum() + np.square(K.T @ dG).sum() + np.square(H.T @ dZ).sum())
    gk, gz = K @ K.T, dZ @ dZ.T
    gram = 0.0
    for lo, hi in _tiles(h):
        m_ug = dU[:, lo:hi] @ dU[:, lo:hi].T + dG[:, lo:hi] @ dG[:, lo:hi].T
        m_h = H[:, lo:hi] @ H[:, lo:hi].T
        gram += (gk * m_ug).sum() + (gz * m_h).sum()
    assert abs(gram - direct) <= 1e-9 * direct


def test_gram_norm_matches_the_oracles_gradients():
    """The clip norm of one chunk from the oracle's own gradients against the Gram form
    built from the same forward / backward intermediates."""
    rng = np.random.default_rng(5)
    B, C, d, h = 1, 64, 128, 160
    k = rng.standard_normal((B, C, d)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, C, d)).astype(np.float32)
    v /= np.linalg.norm(v, axis=-1, keepdims=True)
    eta = np.full((B, C, 1), 0.01, np.float32)
    wu = (rng.standard_normal((B, d, h)) * d ** -0.5).astype(np.float32)
    wg = (rng.standard_normal((B, d, h)) * d ** -0.5).astype(np.float32)
    wd = (rng.standard_normal((B, h, d)) * 0.3 * h ** -0.5).astype(np.float32)
    lnw, lnb = np.ones(d, np.float32), np.zeros(d, np.float32)
    g = ofw.analytical_swiglu_chunk_grad(k, v, eta, wu, wg, wd, lnw, lnb, None, True, 1e-5, Precision("f32"))
    direct = float(sum(np.square(x.astype(np.float64)).sum() for x in (g.grad_w_up, g.grad_w_gate, g.grad_w_down)))
    # the same forward / backward intermediates in float64, then the Gram form tile by tile
    K = k[0].astype(np.float64)
    u, gg = K @ wu[0], K @ wg[0]
    sg = 1.0 / (1.0 + np.exp(-gg))
    Hm = gg * sg * u
    z = Hm @ wd[0]
    mu = z.mean(-1, keepdims=True)
    rstd = 1.0 / np.sqrt(((z - mu) ** 2).mean(-1, keepdims=True) + 1e-5)
    zh = (z - mu) * rstd
    err = K + zh - v[0]
    dzh = (eta[0] / C) * (1.0 / d) * err
    dZ = rstd * (dzh - dzh.mean(-1, keepdims=True) - zh * (dzh * zh).mean(-1, keepdims=True))
    dH = dZ @ wd[0].T
    dU, dG = dH * gg * sg, dH * u * sg * (1 + gg * (1 - sg))
    gk, gz = K @ K.T, dZ @ dZ.T
    gram = 0.0
    for lo, hi in _tiles(h):
        gram += (gk * (dU[:, lo:hi] @ dU[:, lo:hi].T + dG[:, lo:hi] @ dG[:, lo:hi].T)).sum()
        gram += (gz * (Hm[:, lo:hi] @ Hm[:, lo:hi].T)).sum()
    assert abs(gram - direct) <= 1e-4 * direct, (gram, direct)

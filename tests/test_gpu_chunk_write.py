"""GPU parity of the tcgen05 chunk-TTT write against the reference's fixtures
and against the oracle.

Tolerances (BF16 operands, FP32 accumulation and FP32 masters):
  updated state   rel-L2 <= 1e-3         (north-star bound for the FP32 state)
  update  W'-W    rel-L2 <= 2e-2         (the reference rounds every gradient to BF16)
  readout / v_hat max |diff| <= 2e-2     (BF16 activations)
  token loss      rel <= 1e-2
"""

import os

import numpy as np
import pytest
import torch

from oracle import fastweight as ofw
from oracle.numerics import Precision, rel_l2, round_bf16
from utttcompanion_b200 import fastweight as fw

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

DEV = "cuda"


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def T(x, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x)).to(device=DEV, dtype=dtype)


def _run_write(g, B, C, d, h, mask, beta, clip, eps, normalize=True, out=False):
    ws = [T(g[n]).contiguous() for n in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down")]
    k, v = T(g["k"], torch.bfloat16), T(g["v"], torch.bfloat16)
    eta, alpha = T(g["eta"]).reshape(B, C), T(g["alpha"]).reshape(B, C)
    m = None if mask is None else T(mask).reshape(B, C)
    o = torch.empty(B, C, d, device=DEV) if out else None
    loss = torch.empty(B, C, device=DEV)
    fw.chunk_write(k, v, eta, alpha, *ws, T(g["ln_weight"]), T(g["ln_bias"]), m, beta, clip, normalize, eps,
                   chunk_size=C, out=o, token_loss=loss)
    torch.cuda.synchronize()
    fw.check_status(fw.workspace(0, torch.device(DEV)), "chunk_write")
    return [w.cpu().numpy() for w in ws], (None if o is None else o.cpu().numpy()), loss.cpu().numpy()


@pytest.mark.parametrize("name", ["bf16_plain", "bf16_full", "bf16_clipbite"])
def test_chunk_write_matches_reference_fixture(name):
    g = load("chunk_" + name)
    B, C, d = g["k"].shape
    h = g["w_up"].shape[-1]
    beta, clip, normalize, eps = (float(x) for x in g["meta"])
    mask = g.get("mask")
    new, out, loss = _run_write(g, B, C, d, h, mask, beta, clip, eps, bool(normalize), out=True)
    names = ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down")
    for arr, nm in zip(new, names):
        ref = g["new_" + nm]
        if nm.startswith("w"):
            assert rel_l2(arr, ref) < 1e-3, (nm, rel_l2(arr, ref))
            assert rel_l2(arr - g[nm], ref - g[nm]) < 2e-2, (nm, rel_l2(arr - g[nm], ref - g[nm]))
        else:
            assert rel_l2(arr, ref) < 2e-2, (nm, rel_l2(arr, ref))
    if mask is not None:
        inactive = ~(mask != 0).any(axis=1)
        for arr, nm in zip(new, names):
            np.testing.assert_array_equal(arr[inactive], g[nm][inactive])
    # surprise: the reference's batch-global masked mean of the token losses
    if mask is None:
        surprise = loss.mean()
    else:
        surprise = (loss * mask).sum() / max(mask.sum(), 1.0)
    assert abs(surprise - float(g["surprise"])) <= 1e-2 * abs(float(g["surprise"])) + 1e-6
    if name == "bf16_plain":   # q == k, read = W: the write also yields the readout
        assert np.max(np.abs(out - g["out"])) < 2e-2


def test_fused_chunk_ttt_step_dropin_q_is_k():
    g = load("chunk_bf16_plain")
    beta, clip, normalize, eps = (float(x) for x in g["meta"])
    q = T(g["q"], torch.bfloat16)
    args = [q, q, T(g["v"], torch.bfloat16), T(g["eta"], torch.bfloat16), T(g["alpha"], torch.bfloat16)]
    args += [T(g[n]) for n in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down", "ln_weight", "ln_bias")]
    res = fw.fused_chunk_ttt_step(*args, None, beta, clip, bool(normalize), eps)
    assert len(res) == 8 and res[0].dtype == torch.bfloat16
    assert np.max(np.abs(res[0].float().cpu().numpy() - g["out"])) < 2e-2
    assert rel_l2(res[1].cpu().numpy(), g["new_w_up"]) < 1e-3
    assert abs(float(res[7]) - float(g["surprise"])) < 1e-2 * abs(float(g["surprise"]))
    # inputs untouched (the reference returns new tensors)
    np.testing.assert_array_equal(args[5].cpu().numpy(), g["w_up"])


def _oracle_sequence(k, v, eta, alpha, W, S, lnw, lnb, mask, beta, clip, C, eps):
    """Chain the oracle's chunk step over T tokens (uTTTLayer.forward's chunk loop)."""
    B, Tn, d = k.shape
    W = [w.copy() for w in W]
    S = [s.copy() for s in S]
    losses = np.zeros((B, Tn), np.float32)
    prec = Precision("bf16")
    for off in range(0, Tn, C):
        e = min(off + C, Tn)
        m = None if mask is None else mask[:, off:e]
        r = ofw.fused_chunk_ttt_step(k[:, off:e], k[:, off:e], v[:, off:e], eta[:, off:e, None],
                                     alpha[:, off:e, None], *W, *S, lnw, lnb, m, beta, clip, True, eps, prec=prec)
        W = [r.w_up, r.w_gate, r.w_down]
        S = [r.s_up, r.s_gate, r.s_down]
        losses[:, off:e] = r.token_loss
    return W, S, losses


@pytest.mark.parametrize("beta,clip,masked", [(0.0, 0.0, False), (0.9, 1.0, True), (0.5, 0.05, False)])
def test_multi_chunk_sequence_matches_oracle(beta, clip, masked):
    rng = np.random.default_rng(7)
    B, Tn, C, d, h = 3, 200, 64, 256, 384      # ragged last chunk (200 = 3*64 + 8)
    def unit(shape):
        x = rng.standard_normal(shape)
        return round_bf16(x / np.linalg.norm(x, axis=-1, keepdims=True))
    k, v = unit((B, Tn, d)), unit((B, Tn, d))
    eta = rng.uniform(0.005, 0.05, (B, Tn)).astype(np.float32)
    alpha = rng.uniform(0.0, 0.01, (B, Tn)).astype(np.float32)
    W = [rng.normal(0, 0.02, (B, d, h)).astype(np.float32), rng.normal(0, 0.02, (B, d, h)).astype(np.float32),
         rng.normal(0, 0.02, (B, h, d)).astype(np.float32)]
    S = [rng.normal(0, 1e-3, w.shape).astype(np.float32) for w in W]
    lnw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    lnb = (0.1 * rng.standard_normal(d)).astype(np.float32)
    mask = None
    if masked:
        mask = np.ones((B, Tn), np.float32)
        mask[1, 150:] = 0
        mask[2, 64:128] = 0       # a fully masked middle chunk keeps the state
    Wr, Sr, lr = _oracle_sequence(k, v, eta, alpha, W, S, lnw, lnb, mask, beta, clip, C, 1e-5)
    wt = [T(x).contiguous() for x in W + S]
    loss = torch.empty(B, Tn, device=DEV)
    fw.chunk_write(T(k, torch.bfloat16), T(v, torch.bfloat16), T(eta), T(alpha), *wt, T(lnw), T(lnb),
                   None if mask is None else T(mask), beta, clip, True, 1e-5, chunk_size=C, token_loss=loss)
    torch.cuda.synchronize()
    fw.check_status(fw.workspace(0, torch.device(DEV)), "chunk_write")
    for got, ref, base, nm in zip(wt[:3], Wr, W, ("w_up", "w_gate", "w_down")):
        got = got.cpu().numpy()
        assert rel_l2(got, ref) < 1e-3, nm
        assert rel_l2(got - base, ref - base) < 2e-2, (nm, rel_l2(got - base, ref - base))
    for got, ref, nm in zip(wt[3:], Sr, ("s_up", "s_gate", "s_down")):
        assert rel_l2(got.cpu().numpy(), ref) < 2e-2, nm
    lg = loss.cpu().numpy()
    valid = np.ones_like(lg, bool) if mask is None else mask != 0
    assert rel_l2(lg[valid], lr[valid]) < 1e-2


@pytest.mark.parametrize("B,d,h,Tn", [(3, 256, 384, 150), (6, 256, 384, 64)])
def test_guarded_write_equals_write_then_elastic_pull(B, d, h, Tn):
    """uttt_chunk_write_guarded (the elastic pull inside each final row's last update, and the drift
    sums of the pulled state) against uttt_chunk_write followed by the stand-alone guard pass
    (uttt_elastic_pull, pinned to the reference's apply_elastic_pull by the elastic fixture) and
    uttt_drift_sums: B = 3 runs the d-split kernels over 3 chained chunks, B = 6 the plain ones;
    rows whose final flag is 0 are left unpulled.  Bounds: state rel-L2 <= 1e-6 (FP32 rounding of
    one fused multiply-add), sums rel <= 1e-4 (atomic summation order)."""
    from utttcompanion_b200 import _lib
    rng = np.random.default_rng(B)

    def unit(shape):
        x = rng.standard_normal(shape)
        return round_bf16(x / np.linalg.norm(x, axis=-1, keepdims=True))
    k, v = unit((B, Tn, d)), unit((B, Tn, d))
    eta = rng.uniform(0.005, 0.05, (B, Tn)).astype(np.float32)
    alpha = rng.uniform(0.0, 0.01, (B, Tn)).astype(np.float32)
    W0 = [rng.normal(0, d ** -0.5, (d, h)).astype(np.float32), rng.normal(0, d ** -0.5, (d, h)).astype(np.float32),
          rng.normal(0, 0.1 * h ** -0.5, (h, d)).astype(np.float32)]
    W = [(w[None] + rng.normal(0, 1e-2, (B,) + w.shape)).astype(np.float32) for w in W0]
    S = [rng.normal(0, 1e-3, w.shape).astype(np.float32) for w in W]
    lnw, lnb = np.ones(d, np.float32), np.zeros(d, np.float32)
    final = np.array([1 if b % 3 != 1 else 0 for b in range(B)], np.int32)
    lam = 0.02
    a = [T(x).contiguous() for x in W + S]
    g = [T(x).contiguous() for x in W + S]
    w0 = [T(x).contiguous() for x in W0]
    fw.chunk_write(T(k, torch.bfloat16), T(v, torch.bfloat16), T(eta), T(alpha), *a, T(lnw), T(lnb), None, 0.9, 1.0,
                   True, 1e-5, chunk_size=64)
    pulled = [x.clone() for x in a[:3]]
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    sel = [b for b in range(B) if final[b]]
    for b in sel:                                           # the stand-alone guard pass on the final rows
        one = [x[b:b + 1].contiguous() for x in pulled]
        ws = fw.workspace(lib.uttt_guard_workspace(1), torch.device(DEV), slot=3)
        _lib.check(lib.uttt_elastic_pull(1, d, h, *(x.data_ptr() for x in one), *(x.data_ptr() for x in w0), lam, 0.0,
                                         ws.data_ptr(), ws.numel(), stream), "uttt_elastic_pull")
        for x, o in zip(pulled, one):
            x[b].copy_(o[0])
    ref_sums = torch.zeros(4 * B + 4, device=DEV)
    _lib.check(lib.uttt_drift_sums(B, d, h, *(x.data_ptr() for x in pulled), *(x.data_ptr() for x in w0),
                                   ref_sums.data_ptr(), stream), "uttt_drift_sums")
    sums = torch.zeros(B, 4, device=DEV)
    fw.chunk_write(T(k, torch.bfloat16), T(v, torch.bfloat16), T(eta), T(alpha), *g, T(lnw), T(lnb), None, 0.9, 1.0,
                   True, 1e-5, chunk_size=64, guard=(*w0, lam, T(final, torch.int32), sums))
    torch.cuda.synchronize()
    fw.check_status(fw.workspace(0, torch.device(DEV)), "chunk_write_guarded")
    for got, want, nm in zip(g[:3], pulled, ("w_up", "w_gate", "w_down")):
        err = rel_l2(got.cpu().numpy(), want.cpu().numpy())
        assert err <= 1e-6, (nm, err)
    for got, want in zip(g[3:], a[3:]):                     # momentum is not pulled
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) <= 1e-6
    rs = ref_sums[:4 * B].reshape(B, 4).cpu().numpy()
    gs = sums.cpu().numpy()
    for b in range(B):
        if final[b]:
            assert np.allclose(gs[b, :3], rs[b, :3], rtol=1e-4), (b, gs[b], rs[b])
        else:
            assert (gs[b] == 0).all()

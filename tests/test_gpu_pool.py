"""GPU parity of the remaining drop-ins: stability guard, analytical gradient,
slow projections, q projection, apply_rope and the pool's chunk_step.

Bounds: guard/drift to FP32 rounding (rel 1e-5); gradients rel-L2 <= 2e-2
against the reference's BF16-rounded gradients; projections and RoPE within
one BF16 ULP (+1e-2) of the oracle's BF16 emulation."""

import os

import numpy as np
import pytest
import torch

from oracle import fastweight as ofw
from oracle import model as om
from oracle.numerics import Precision, rel_l2, round_bf16
from utttcompanion_b200 import pool as bp
from utttcompanion_b200.model import FastState

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def T(x, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x)).to(device="cuda", dtype=dtype)


def _pool_from(g):
    d, h = g["w_up0"].shape
    return bp.SharedFastWeightPoolB200(g["w_up0"], g["w_gate0"], g["w_down0"], np.ones(d, np.float32),
                                       np.zeros(d, np.float32))


def test_elastic_pull_drift_clamp_and_drift_report_match_reference():
    g = load("elastic")
    pool = _pool_from(g)
    st = FastState(T(g["w_up"]), T(g["w_gate"]), T(g["w_down"]), *(torch.zeros_like(T(g[n])) for n in
                                                                    ("w_up", "w_gate", "w_down")),
                   pool.ln_weight, pool.ln_bias)
    pulled = pool.apply_elastic_pull(st, 0.02, 0.35)
    for got, key in ((pulled.w_up, "p_up"), (pulled.w_gate, "p_gate"), (pulled.w_down, "p_down")):
        assert rel_l2(got.cpu().numpy(), g[key]) < 1e-5, key
    plain = pool.apply_elastic_pull(st, 0.05, None)
    for got, key in ((plain.w_up, "n_up"), (plain.w_gate, "n_gate"), (plain.w_down, "n_down")):
        assert rel_l2(got.cpu().numpy(), g[key]) < 1e-6, key
    one = FastState(*(t[:1].contiguous() for t in (st.w_up, st.w_gate, st.w_down, st.s_up, st.s_gate, st.s_down)),
                    st.ln_weight, st.ln_bias)
    drift = pool.compute_drift(one)
    for key, val in zip(g["drift_keys"], g["drift_vals"]):
        assert abs(drift[str(key)] - val) <= 1e-5 * max(1.0, abs(val)), key


def test_analytical_gradient_dropin_matches_reference():
    g = load("chunk_bf16_plain")
    beta, clip, normalize, eps = (float(x) for x in g["meta"])
    gu, gg, gd, surprise = bp.analytical_swiglu_chunk_grad(
        T(g["k"], torch.bfloat16), T(g["v"], torch.bfloat16), T(g["eta"]), T(g["w_up"]), T(g["w_gate"]),
        T(g["w_down"]), T(g["ln_weight"]), T(g["ln_bias"]), None, bool(normalize), eps)
    torch.cuda.synchronize()
    for got, key in ((gu, "grad_w_up"), (gg, "grad_w_gate"), (gd, "grad_w_down")):
        assert rel_l2(got.cpu().numpy(), g[key]) < 2e-2, (key, rel_l2(got.cpu().numpy(), g[key]))
    assert abs(float(surprise) - float(g["grad_surprise"])) < 1e-2 * abs(float(g["grad_surprise"]))


def _close(got, ref, tol=1e-2):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    bad = np.abs(got - ref) > tol + np.abs(ref) / 128
    assert not bad.any(), (float(np.max(np.abs(got - ref))), int(bad.sum()))


@pytest.mark.parametrize("param_dtype", [torch.float32, torch.bfloat16])
def test_slow_projections_and_q_proj_match_oracle(param_dtype):
    """Norm weights and gate biases as an FP32 model and as a BF16 model holds them: the BF16
    case makes the drop-in convert them, and each converted operand must stay distinct (eta's
    bias is not alpha's)."""
    rng = np.random.default_rng(0)
    d = 256
    x = round_bf16(rng.standard_normal((2, 7, d)))
    w = {n: round_bf16(rng.normal(0, 0.05, (d, d))) for n in ("w_q", "w_k", "w_v")}
    w_eta, w_alpha = round_bf16(rng.normal(0, 0.05, (1, d))), round_bf16(rng.normal(0, 0.05, (1, d)))
    b_eta, b_alpha = np.array([0.1], np.float32), np.array([-1.386], np.float32)
    qn, kn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32), (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    if param_dtype == torch.bfloat16:          # what the model holds after .to(bfloat16)
        b_eta, b_alpha, qn, kn = (round_bf16(a) for a in (b_eta, b_alpha, qn, kn))
    q, k, v, eta, alpha = bp.fused_slow_projections(
        T(x, torch.bfloat16), T(w["w_q"], torch.bfloat16), T(w["w_k"], torch.bfloat16), T(w["w_v"], torch.bfloat16),
        T(qn, param_dtype), T(kn, param_dtype), T(w_eta, torch.bfloat16), T(b_eta, param_dtype),
        T(w_alpha, torch.bfloat16), T(b_alpha, param_dtype), 0.015, 0.005, 1e-5)
    qf = bp.fused_fast_q_proj(T(x, torch.bfloat16), T(w["w_q"], torch.bfloat16), T(qn, param_dtype), 1e-5)
    torch.cuda.synchronize()
    cfg = om.ModelConfig(d_model=d, n_layers=1, n_heads=4, n_kv_heads=4, base_inner_lr=0.015, base_weight_decay=0.005)
    weights = {"layers.0.uttt.w_q.weight": w["w_q"], "layers.0.uttt.w_k.weight": w["w_k"],
               "layers.0.uttt.w_v.weight": w["w_v"], "layers.0.uttt.q_norm.weight": qn,
               "layers.0.uttt.k_norm.weight": kn, "layers.0.uttt.w_eta.weight": w_eta,
               "layers.0.uttt.w_eta.bias": b_eta, "layers.0.uttt.w_alpha.weight": w_alpha,
               "layers.0.uttt.w_alpha.bias": b_alpha}
    m = om.OracleModel.__new__(om.OracleModel)
    m.cfg, m.prec, m.autocast, m.w = cfg, Precision("bf16"), True, {k2: round_bf16(v2) if "norm" not in k2 and
                                                                    "bias" not in k2 else v2
                                                                    for k2, v2 in weights.items()}
    oq, ok, ov, oeta, oalpha = m.slow_projections(0, x)
    for got, ref in ((q, oq), (k, ok), (v, ov), (qf, oq)):
        _close(got.float().cpu().numpy(), ref)
    _close(eta.float().cpu().numpy(), oeta, 1e-4)
    _close(alpha.float().cpu().numpy(), oalpha, 1e-5)


def test_apply_rope_matches_oracle():
    rng = np.random.default_rng(1)
    B, H, Tn, D = 2, 3, 9, 64
    q = round_bf16(rng.standard_normal((B, H, Tn, D)))
    k = round_bf16(rng.standard_normal((B, 1, Tn, D)))
    cos, sin = om.rope_tables(D, 32)
    start = 5
    qr, kr = bp.apply_rope(T(q, torch.bfloat16), T(k, torch.bfloat16), T(cos[start:start + Tn])[None, None],
                           T(sin[start:start + Tn])[None, None])
    torch.cuda.synchronize()
    m = om.OracleModel.__new__(om.OracleModel)
    m.prec, m.cos, m.sin = Precision("bf16"), cos, sin
    np.testing.assert_array_equal(qr.float().cpu().numpy(), m._rope(q, start))
    np.testing.assert_array_equal(kr.float().cpu().numpy(), m._rope(k, start))


def test_pool_chunk_step_matches_oracle_with_read_snapshot():
    g = load("chunk_bf16_full")
    beta, clip, normalize, eps = (float(x) for x in g["meta"])
    d = g["k"].shape[-1]
    pool = bp.SharedFastWeightPoolB200(g["w_up"][0], g["w_gate"][0], g["w_down"][0], g["ln_weight"], g["ln_bias"],
                                       beta, clip, bool(normalize), eps)
    st = FastState(*(T(g[n]) for n in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down")),
                   T(g["ln_weight"]), T(g["ln_bias"]))
    rd = FastState(*(T(g[n]) for n in ("read_w_up", "read_w_gate", "read_w_down")),
                   *(torch.zeros_like(T(g[n])) for n in ("w_up", "w_gate", "w_down")), T(g["ln_weight"]),
                   T(g["ln_bias"]))
    out, new, surprise = pool.chunk_step(st, T(g["q"], torch.bfloat16), T(g["k"], torch.bfloat16),
                                         T(g["v"], torch.bfloat16), T(g["eta"], torch.bfloat16),
                                         T(g["alpha"], torch.bfloat16), T(g["mask"]), True, rd)
    torch.cuda.synchronize()
    assert new.step == 1
    for n in ("w_up", "w_gate", "w_down"):
        assert rel_l2(getattr(new, n).cpu().numpy(), g["new_" + n]) < 1e-3, n
    _close(out.float().cpu().numpy(), g["out"], 3e-2)
    assert abs(float(surprise) - float(g["surprise"])) < 1e-2 * abs(float(g["surprise"]))

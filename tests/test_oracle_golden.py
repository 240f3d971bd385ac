"""Pin the numpy oracle against fixtures produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py`` (which imports the
reference implementation).  FP64 cases must agree to ~1e-10, FP32 to FP32
rounding, and the BF16-activation cases to BF16 rounding noise.
"""

import os

import numpy as np
import pytest

from oracle import fastweight as fw
from oracle import model as om
from oracle.numerics import Precision, rel_l2

from conftest import GOLDEN


def load(name):
    out = dict(np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False))
    if name.startswith("model_"):
        out.update(np.load(os.path.join(GOLDEN, "model_shared.npz"), allow_pickle=False))
    return out


CHUNK_CASES = ["f64_plain", "f64_full", "f32_plain", "f32_full", "bf16_plain", "bf16_full", "bf16_clipbite"]


def _chunk_tols(name):
    if name.startswith("f64"):
        return 1e-10, 1e-12
    if name.startswith("f32"):
        return 2e-5, 1e-6
    return 2e-2, 1e-6   # bf16 activations: grads are BF16-rounded bmm outputs


@pytest.mark.parametrize("name", CHUNK_CASES)
def test_chunk_grad_and_step_match_reference(name):
    g = load("chunk_" + name)
    prec = Precision("bf16" if bool(g["act_is_bf16"]) else ("f64" if name.startswith("f64") else "f32"))
    beta, clip, normalize, eps = g["meta"]
    mask = g.get("mask")
    grad_tol, state_tol = _chunk_tols(name)
    grads = fw.analytical_swiglu_chunk_grad(g["k"], g["v"], g["eta"], g["w_up"], g["w_gate"], g["w_down"],
                                            g["ln_weight"], g["ln_bias"], mask, bool(normalize), float(eps), prec)
    for ours, key in ((grads.grad_w_up, "grad_w_up"), (grads.grad_w_gate, "grad_w_gate"),
                      (grads.grad_w_down, "grad_w_down")):
        assert rel_l2(ours, g[key]) < grad_tol, (key, rel_l2(ours, g[key]))
    assert abs(grads.surprise - float(g["grad_surprise"])) <= 1e-6 * max(1.0, abs(float(g["grad_surprise"]))) + \
        (1e-3 if prec.mode == "bf16" else 0)

    res = fw.fused_chunk_ttt_step(g["q"], g["k"], g["v"], g["eta"], g["alpha"], g["w_up"], g["w_gate"],
                                  g["w_down"], g["s_up"], g["s_gate"], g["s_down"], g["ln_weight"],
                                  g["ln_bias"], mask, float(beta), float(clip), bool(normalize), float(eps),
                                  g.get("read_w_up"), g.get("read_w_gate"), g.get("read_w_down"), prec=prec)
    for ours, key in ((res.w_up, "new_w_up"), (res.w_gate, "new_w_gate"), (res.w_down, "new_w_down")):
        assert rel_l2(ours, g[key]) < state_tol, (key, rel_l2(ours, g[key]))
    # momentum holds the (clipped) step itself, so it carries the gradient's rounding
    for ours, key in ((res.s_up, "new_s_up"), (res.s_gate, "new_s_gate"), (res.s_down, "new_s_down")):
        assert rel_l2(ours, g[key]) < grad_tol, (key, rel_l2(ours, g[key]))
    # the update itself (W' - W) is the sensitive quantity
    for ours, key, base in ((res.w_up, "new_w_up", "w_up"), (res.w_down, "new_w_down", "w_down")):
        assert rel_l2(ours - g[base], g[key] - g[base]) < grad_tol * 2, key
    out_tol = 1e-10 if prec.mode == "f64" else (1e-5 if prec.mode == "f32" else 2e-2)
    assert np.max(np.abs(res.out - g["out"])) < out_tol
    if mask is not None:
        inactive = ~(mask != 0).any(axis=1)
        assert inactive.any()
        np.testing.assert_array_equal(res.w_up[inactive], g["w_up"][inactive])


@pytest.mark.parametrize("name", ["f32", "bf16", "bf16_t1", "bf16_t70"])
def test_swiglu_readout_matches_reference(name):
    g = load("swiglu_" + name)
    prec = Precision("bf16" if bool(g["act_is_bf16"]) else "f32")
    y = fw.swiglu_fast_forward(g["x"], g["w_up"], g["w_gate"], g["w_down"], g["ln_weight"], g["ln_bias"], 1e-5, prec)
    tol = 1e-5 if prec.mode == "f32" else 2e-2
    assert np.max(np.abs(y - g["out"])) < tol
    assert np.max(np.abs(y - g["out_packed"])) < tol


def test_elastic_pull_and_drift_match_reference():
    g = load("elastic")
    up, gate, down = fw.apply_elastic_pull(g["w_up"], g["w_gate"], g["w_down"], g["w_up0"], g["w_gate0"],
                                           g["w_down0"], 0.02, 0.35)
    for ours, key in ((up, "p_up"), (gate, "p_gate"), (down, "p_down")):
        assert rel_l2(ours, g[key]) < 1e-6
    up, gate, down = fw.apply_elastic_pull(g["w_up"], g["w_gate"], g["w_down"], g["w_up0"], g["w_gate0"],
                                           g["w_down0"], 0.05, None)
    for ours, key in ((up, "n_up"), (gate, "n_gate"), (down, "n_down")):
        assert rel_l2(ours, g[key]) < 1e-6
    drift = fw.compute_drift(g["w_up"][:1], g["w_gate"][:1], g["w_down"][:1], g["w_up0"], g["w_gate0"], g["w_down0"])
    for key, val in zip(g["drift_keys"], g["drift_vals"]):
        assert abs(drift[str(key)] - val) <= 1e-5 * max(1.0, abs(val)), key


def _small_model(g, prec):
    cfg = om.ModelConfig(**{k: v for k, v in eval(str(g["cfg_json"])).items()
                            if k in om.ModelConfig.__dataclass_fields__})
    weights = {k[3:]: g[k] for k in g if k.startswith("W::")}
    model = om.OracleModel(weights, cfg, prec, g["rope_cos"], g["rope_sin"])
    return model, cfg


def _state(g, model, dt):
    st = model.state_for_forward(1, update=True)
    st.w_up, st.w_gate, st.w_down = (g["state_w_up"].astype(dt), g["state_w_gate"].astype(dt),
                                     g["state_w_down"].astype(dt))
    return st


@pytest.mark.parametrize("name", ["f64", "f32", "bf16"])
def test_small_model_decode_and_write_match_reference(name):
    g = load("model_" + name)
    model, cfg = _small_model(g, name)
    assert int(g["active_limit"]) == model.active_limit
    dt = np.float64 if name == "f64" else np.float32
    state = _state(g, model, dt)
    ids = [int(x) for x in g["ids"]]
    logits = model.teacher_forced_logits(g["prompt"], ids, state)
    tol = {"f64": 1e-9, "f32": 2e-5, "bf16": 3e-2}[name]
    err = max(float(np.max(np.abs(a - b))) for a, b in zip(logits, g["logits"]))
    assert err < tol, err
    if name != "bf16":
        got, margins, _ = model.generate_greedy(g["prompt"], state, len(ids))
        assert got == ids
    new_state, mean_surprise, per_layer, _ = model.test_time_update(g["inter"][None], state, g["mask"][None])
    st_tol = {"f64": 1e-10, "f32": 1e-5, "bf16": 5e-3}[name]   # bf16: w_down moves ~30% of its norm per turn here
    for ours, key in ((new_state.w_up, "new_w_up"), (new_state.w_gate, "new_w_gate"),
                      (new_state.w_down, "new_w_down")):
        assert rel_l2(ours, g[key]) < st_tol, (key, rel_l2(ours, g[key]))
    # the written delta, relative to its own size
    d_tol = {"f64": 1e-8, "f32": 1e-3, "bf16": 3e-2}[name]
    for ours, key, base in ((new_state.w_up, "new_w_up", "state_w_up"), (new_state.w_down, "new_w_down", "state_w_down")):
        assert rel_l2(ours - g[base], g[key] - g[base]) < d_tol, key
    for ours, key in ((new_state.s_up, "new_s_up"), (new_state.s_down, "new_s_down")):
        assert rel_l2(ours, g[key]) < d_tol, key
    assert new_state.step == int(g["new_step"])
    assert abs(mean_surprise - float(g["mean_surprise"])) < (1e-9 if name == "f64" else 1e-3)
    np.testing.assert_allclose(per_layer, g["layer_surprises"], rtol=1e-3 if name != "f64" else 1e-9)


def test_oracle_matches_reference_config1_run():
    """BASELINE config 1 as the reference ran it (seed-0 init, 64 stop-free greedy steps, the
    write of prompt + reply): the oracle's FP32 path reproduces the reference's FP32 run (ids
    exactly, logits and state to FP32 rounding) and its BF16 path the reference's BF16 run to
    BF16 rounding noise (CPU autocast and the oracle's emulation round at the same points but
    accumulate in a different order)."""
    from oracle.numerics import from_bf16_bits
    from utttcompanion_b200.model import rope_tables
    from utttcompanion_b200.workloads import CONFIG_TINY, reference_init_state_dict
    g = load("config1_reference")
    cfg = CONFIG_TINY
    sd = {k: v.numpy() for k, v in reference_init_state_dict(cfg, seed=0).items()}
    ocfg = om.ModelConfig(**{k: v for k, v in cfg.to_dict().items() if k in om.ModelConfig.__dataclass_fields__})
    cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len + 1024, cfg.rope_theta)
    for mode in ("f32", "bf16"):
        o = om.OracleModel(sd, ocfg, mode, cos.numpy(), sin.numpy())
        assert o.active_limit == int(g["active_limit"])
        ids = [int(x) for x in g[mode + "_ids"]]
        st = o.state_for_forward(1, update=True)
        tf = o.teacher_forced_logits(g["prompt"], ids, st)
        ref = g["f32_logits"] if mode == "f32" else from_bf16_bits(g["bf16_logits_bits"])
        err = max(float(np.max(np.abs(np.asarray(a, np.float64) - b))) for a, b in zip(tf, ref))
        assert err < (2e-5 if mode == "f32" else 3e-2), (mode, err)
        if mode == "f32":
            got, _, _ = o.generate_greedy(g["prompt"], o.state_for_forward(1, update=True), 64)
            assert got == ids
        new, ms, pl, _ = o.test_time_update(g["inter"][None], st, g["mask"][None])
        assert new.step == int(g[mode + "_new_step"])
        for n in ("w_up", "w_gate", "w_down"):
            bound = 1e-5 if mode == "f32" else (1e-4 if n != "w_down" else 8e-3)
            assert rel_l2(getattr(new, n), g[f"{mode}_new_{n}"]) < bound, (mode, n)
        assert abs(ms - float(g[mode + "_mean_surprise"])) < (1e-6 if mode == "f32" else 1e-3)

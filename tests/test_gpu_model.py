"""GPU parity of the B200 model engine (decode + chunk-first TTT write).

Bounds (north star): logits |diff| <= 2e-2 (+ one BF16 ULP of the value);
greedy ids identical wherever the reference's top-1/top-2 margin exceeds
twice the logits bound (a near-tie below that may legitimately flip between
two BF16 implementations, as the reference itself saw between its graph and
eager decoders); updated FP32 state rel-L2 <= 5e-3 and the written delta
W'-W rel-L2 <= 3e-2 against the reference's BF16-autocast path (whose own
BF16 rounding of every gradient accounts for the gap).
"""

import os

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle.numerics import rel_l2
from utttcompanion_b200.model import FastState, UtttB200
from utttcompanion_b200.workloads import CONFIG_TINY, ModelConfig, reference_init_state_dict

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def load(name):
    out = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    out.update(np.load(os.path.join(GOLDEN, "model_shared.npz")))
    return out


def logits_close(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.abs(got - ref) <= LOGIT_TOL + np.abs(ref) / 128


def masked_margin(logits, limit):
    w = np.asarray(logits, np.float64).copy()
    w[:6] = -np.inf
    w[limit:] = -np.inf
    top = np.sort(w)[-2:]
    return float(top[1] - top[0]), int(np.argmax(w))


def small_engine(g):
    cfg = ModelConfig.from_dict(eval(str(g["cfg_json"])))
    sd = {k[3:]: torch.tensor(g[k]) for k in g if k.startswith("W::")}
    eng = UtttB200(sd, cfg, max_personas=2)
    st = eng.init_fast_state(1)
    st.w_up, st.w_gate, st.w_down = (torch.tensor(g["state_" + n]).cuda().contiguous()
                                     for n in ("w_up", "w_gate", "w_down"))
    return eng, cfg, st


def test_small_model_matches_reference_bf16_path():
    g = load("model_bf16")
    eng, cfg, st = small_engine(g)
    prompt = torch.tensor(g["prompt"])
    ids = [int(x) for x in g["ids"]]
    tf = eng.teacher_forced_logits(prompt, ids, st)
    torch.cuda.synchronize()
    for step, (ours, ref) in enumerate(zip(tf, g["logits"])):
        ok = logits_close(ours.cpu().numpy(), ref)
        assert ok.all(), (step, float(np.max(np.abs(ours.cpu().numpy() - ref))))
        margin, ref_id = masked_margin(ref, int(g["active_limit"]))
        got_id = int(np.argmax(_mask(ours.cpu().numpy(), int(g["active_limit"]))))
        if margin > 2 * LOGIT_TOL:
            assert got_id == ref_id, (step, margin)
    new, mean_s, per_layer = eng.test_time_update(torch.tensor(g["inter"]), st, torch.tensor(g["mask"]))
    torch.cuda.synchronize()
    assert new.step == int(g["new_step"])
    for n in ("w_up", "w_gate", "w_down"):
        got = getattr(new, n).cpu().numpy()
        assert rel_l2(got, g["new_" + n]) < 5e-3, n
        assert rel_l2(got - g["state_" + n], g["new_" + n] - g["state_" + n]) < 3e-2, (
            n, rel_l2(got - g["state_" + n], g["new_" + n] - g["state_" + n]))
    for n in ("s_up", "s_down"):
        assert rel_l2(getattr(new, n).cpu().numpy(), g["new_" + n]) < 3e-2, n
    assert abs(mean_s - float(g["mean_surprise"])) < 1e-2 * abs(float(g["mean_surprise"]))
    np.testing.assert_allclose(per_layer, g["layer_surprises"], rtol=1e-2)


def _mask(logits, limit):
    w = np.asarray(logits, np.float64).copy()
    w[:6] = -np.inf
    w[limit:] = -np.inf
    return w


def test_small_model_free_running_greedy_matches_reference_until_a_near_tie():
    g = load("model_bf16")
    eng, cfg, st = small_engine(g)
    ids = [int(x) for x in g["ids"]]
    got, margins, _ = eng.generate_greedy(torch.tensor(g["prompt"]), st, len(ids))
    for step, (a, b) in enumerate(zip(got, ids)):
        if a != b:
            margin, _ = masked_margin(g["logits"][step], int(g["active_limit"]))
            assert margin <= 2 * LOGIT_TOL, (step, margin)
            break


def test_config1_tiny_model_against_oracle():
    """BASELINE config 1 (reference seed-0 init): 256-token prompt, 64 greedy
    steps (teacher-forced on the oracle's ids) and a masked write on
    prompt + reply (5 chunks x 4 layers)."""
    cfg = CONFIG_TINY
    sd = reference_init_state_dict(cfg, seed=0)
    eng = UtttB200(sd, cfg, max_personas=1)
    ocfg = om.ModelConfig(**{k: v for k, v in cfg.to_dict().items() if k in om.ModelConfig.__dataclass_fields__})
    oracle = om.OracleModel({k: v.numpy() for k, v in sd.items()}, ocfg, "bf16",
                            *[t.numpy() for t in (eng.rope_cos.cpu(), eng.rope_sin.cpu())])
    gen = torch.Generator().manual_seed(0)
    prompt = torch.randint(6, cfg.vocab_size, (256,), generator=gen)
    ost = oracle.state_for_forward(1, update=True)
    n_steps = 64
    oid, omargins, olog = oracle.generate_greedy(prompt.numpy(), ost, n_steps)
    st = eng.init_fast_state(1)
    tf = eng.teacher_forced_logits(prompt, oid, st)
    torch.cuda.synchronize()
    flips = 0
    for step in range(n_steps):
        ours = tf[step].cpu().numpy()
        ok = logits_close(ours, olog[step])
        assert ok.all(), (step, float(np.max(np.abs(ours - olog[step]))))
        got = int(np.argmax(_mask(ours, oracle.active_limit)))
        if got != oid[step]:
            flips += 1
            assert omargins[step] <= 2 * LOGIT_TOL, (step, omargins[step])
    # write on prompt + reply padded to a multiple of 64 with a mask (personalizer.py:483-501)
    turn = prompt.tolist() + oid
    C = cfg.chunk_size
    padded = ((len(turn) + C - 1) // C) * C
    inter = np.array(turn + [0] * (padded - len(turn)))
    mask = np.array([1.0] * len(turn) + [0.0] * (padded - len(turn)), np.float32)
    on, oms, opl, _ = oracle.test_time_update(inter[None], ost, mask[None])
    new, ms, pl = eng.test_time_update(torch.tensor(inter), st, torch.tensor(mask))
    torch.cuda.synchronize()
    assert new.step == on.step == 5 * cfg.n_layers
    for n in ("w_up", "w_gate", "w_down"):
        got, ref, base = getattr(new, n).cpu().numpy(), getattr(on, n), getattr(ost, n)
        # W_down starts at std 0.1/sqrt(h) and one turn moves a large part of it
        assert rel_l2(got, ref) < 5e-3, (n, rel_l2(got, ref))
        assert rel_l2(got - base, ref - base) < 3e-2, (n, rel_l2(got - base, ref - base))
    np.testing.assert_allclose(pl, opl, rtol=1e-2)


def test_packed_multi_persona_decode_equals_per_persona_decode():
    """Rows of one packed decode batch (own read copy, KV slot, position) give
    the same logits as each persona decoded alone."""
    cfg = ModelConfig(vocab_size=2048, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff_fast=384,
                      sliding_window_size=32, chunk_size=64, max_seq_len=512)
    sd = reference_init_state_dict(cfg, seed=5)
    P = 4
    eng = UtttB200(sd, cfg, max_personas=P)
    from utttcompanion_b200.workloads import perturbed_persona_states
    w_up, w_gate, w_down = perturbed_persona_states(sd["fast_weight_pool.w_up_init"],
                                                    sd["fast_weight_pool.w_gate_init"],
                                                    sd["fast_weight_pool.w_down_init"], P, std=1e-2, seed=3)
    packed, down = eng.read_copies(w_up, w_gate, w_down)
    gen = torch.Generator().manual_seed(1)
    lens = [5, 40, 17, 33]             # ragged; 40 and 33 wrap the 32-slot ring
    prompts = [torch.randint(6, cfg.vocab_size, (n,), generator=gen) for n in lens]
    first = []
    for p in range(P):
        first.append(eng.prefill(prompts[p], p, packed, down, p))
    toks = torch.stack([eng.greedy(f.unsqueeze(0))[0][0] for f in first])
    pos = torch.tensor(lens, dtype=torch.int32)
    slots = torch.arange(P, dtype=torch.int32)
    # packed step for all personas at once
    k_save = [k.clone() for k in eng.k_ring]
    v_save = [v.clone() for v in eng.v_ring]
    packed_logits = eng.decode_step(toks, pos, slots, packed, down, slots)
    # one persona at a time from the same ring state
    for i in range(cfg.n_layers):
        eng.k_ring[i].copy_(k_save[i])
        eng.v_ring[i].copy_(v_save[i])
    for p in range(P):
        one = eng.decode_step(toks[p:p + 1], pos[p:p + 1], slots[p:p + 1], packed, down, slots[p:p + 1])
        a, b = one[0].cpu().numpy(), packed_logits[p].cpu().numpy()
        assert np.max(np.abs(a - b)) <= 1e-2, p
        assert int(np.argmax(_mask(a, cfg.vocab_size))) == int(np.argmax(_mask(b, cfg.vocab_size)))


def _tiny_cfg():
    return ModelConfig(vocab_size=2048, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff_fast=384,
                       sliding_window_size=32, chunk_size=64, max_seq_len=512)


def test_batched_write_equals_per_persona_writes():
    """test_time_update_batch over ragged personas == each persona's own test_time_update.

    The two runs pack different row counts, so the projection GEMMs pick a
    different split-K and accumulate in a different order; BF16 rounding of
    the activations then differs by a ULP here and there.  Bounds: masters
    rel-L2 <= 1e-4, momentum (the accumulated step) <= 1e-2, surprise 1e-3."""
    cfg = _tiny_cfg()
    sd = reference_init_state_dict(cfg, seed=9)
    eng = UtttB200(sd, cfg)
    from utttcompanion_b200.workloads import perturbed_persona_states
    P = 3
    w = perturbed_persona_states(sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"],
                                 sd["fast_weight_pool.w_down_init"], P, std=1e-2, seed=4)
    st = FastState(*w, *(torch.zeros_like(x) for x in w), eng.ln_w.clone(), eng.ln_b.clone())
    lens = [150, 64, 97]
    Tpad = 192
    gen = torch.Generator().manual_seed(2)
    ids = torch.randint(6, cfg.vocab_size, (P, Tpad), generator=gen)
    mask = torch.zeros(P, Tpad)
    for p, n in enumerate(lens):
        mask[p, :n] = 1
    new, surprises, per_layer = eng.test_time_update_batch(ids, st, mask)
    torch.cuda.synchronize()
    for p in range(P):
        one = FastState(*(x[p:p + 1].clone() for x in (st.w_up, st.w_gate, st.w_down, st.s_up, st.s_gate, st.s_down)),
                        st.ln_weight, st.ln_bias)
        n1, s1, pl1 = eng.test_time_update(ids[p], one, mask[p])
        torch.cuda.synchronize()
        for name in ("w_up", "w_gate", "w_down", "s_up", "s_down"):
            a = getattr(new, name)[p].cpu().numpy()
            b = getattr(n1, name)[0].cpu().numpy()
            bound = 1e-4 if name.startswith("w") else 1e-2
            assert rel_l2(a, b) < bound, (p, name, rel_l2(a, b))
        assert abs(surprises[p] - s1) <= 1e-3 * abs(s1)
        np.testing.assert_allclose(per_layer[p], pl1, rtol=1e-3)


def test_decode_graph_replay_equals_eager_steps():
    from utttcompanion_b200.model import DecodeGraph
    from utttcompanion_b200.workloads import perturbed_persona_states
    cfg = _tiny_cfg()
    sd = reference_init_state_dict(cfg, seed=6)
    P = 3
    eng = UtttB200(sd, cfg, max_personas=P)
    w = perturbed_persona_states(sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"],
                                 sd["fast_weight_pool.w_down_init"], P, std=1e-2, seed=8)
    packed, down = eng.read_copies(*w)
    graph = DecodeGraph(eng, P, packed, down)
    gen = torch.Generator().manual_seed(3)
    lens = [12, 45, 30]
    firsts = [eng.prefill(torch.randint(6, cfg.vocab_size, (n,), generator=gen), p, packed, down, p)
              for p, n in enumerate(lens)]
    toks, _ = eng.greedy(torch.stack(firsts))
    pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
    k_save = [k.clone() for k in eng.k_ring]
    v_save = [v.clone() for v in eng.v_ring]
    t_graph, p_graph = toks.clone(), pos.clone()
    graph_logits = []
    for _ in range(5):
        ids, lg = graph.step(t_graph, p_graph)
        graph_logits.append(lg.clone())
        t_graph = ids.clone()
        p_graph = p_graph + 1
    for i in range(cfg.n_layers):
        eng.k_ring[i].copy_(k_save[i])
        eng.v_ring[i].copy_(v_save[i])
    t_e, p_e = toks.clone(), pos.clone()
    slots = torch.arange(P, dtype=torch.int32, device="cuda")
    for s in range(5):
        lg = eng.decode_step(t_e, p_e, slots, packed, down, slots)
        assert torch.max(torch.abs(lg - graph_logits[s])).item() <= 1e-2, s
        t_e, _ = eng.greedy(lg)
        p_e = p_e + 1


def test_head_dim_128_gqa4_model_against_oracle():
    """The 1.58B configuration's attention shape (head dim 128, 4 query heads per
    KV head) at a small width: a prompt longer than the window, teacher-forced
    decode steps and a masked write, against the oracle's BF16 path."""
    cfg = ModelConfig(vocab_size=1024, d_model=512, n_layers=2, n_heads=4, n_kv_heads=1, d_ff_fast=384,
                      sliding_window_size=32, chunk_size=64, max_seq_len=512)
    assert cfg.head_dim == 128
    sd = reference_init_state_dict(cfg, seed=3)
    eng = UtttB200(sd, cfg, max_personas=1)
    ocfg = om.ModelConfig(**{k: v for k, v in cfg.to_dict().items() if k in om.ModelConfig.__dataclass_fields__})
    oracle = om.OracleModel({k: v.numpy() for k, v in sd.items()}, ocfg, "bf16",
                            *[t.numpy() for t in (eng.rope_cos.cpu(), eng.rope_sin.cpu())])
    gen = torch.Generator().manual_seed(5)
    prompt = torch.randint(6, cfg.vocab_size, (80,), generator=gen)
    ost = oracle.state_for_forward(1, update=True)
    n_steps = 24
    oid, omargins, olog = oracle.generate_greedy(prompt.numpy(), ost, n_steps)
    st = eng.init_fast_state(1)
    tf = eng.teacher_forced_logits(prompt, oid, st)
    torch.cuda.synchronize()
    for step in range(n_steps):
        ours = tf[step].cpu().numpy()
        assert logits_close(ours, olog[step]).all(), (step, float(np.max(np.abs(ours - olog[step]))))
        if int(np.argmax(_mask(ours, oracle.active_limit))) != oid[step]:
            assert omargins[step] <= 2 * LOGIT_TOL, (step, omargins[step])
    turn = prompt.tolist() + oid
    padded = ((len(turn) + 63) // 64) * 64
    inter = np.array(turn + [0] * (padded - len(turn)))
    mask = np.array([1.0] * len(turn) + [0.0] * (padded - len(turn)), np.float32)
    on, _, opl, _ = oracle.test_time_update(inter[None], ost, mask[None])
    new, _, pl = eng.test_time_update(torch.tensor(inter), st, torch.tensor(mask))
    torch.cuda.synchronize()
    for n in ("w_up", "w_gate", "w_down"):
        got, ref, base = getattr(new, n).cpu().numpy(), getattr(on, n), getattr(ost, n)
        assert rel_l2(got, ref) < 5e-3, (n, rel_l2(got, ref))
        assert rel_l2(got - base, ref - base) < 3e-2, (n, rel_l2(got - base, ref - base))
    np.testing.assert_allclose(pl, opl, rtol=1e-2)


def test_decode_graph_survives_workspace_growth():
    """A captured decode graph keeps the workspace pointers it was recorded with;
    a later, larger call that grows those workspaces must not free them under
    the graph (the replays still match eager steps after the freed memory has
    been handed out again)."""
    from utttcompanion_b200.fastweight import workspace
    from utttcompanion_b200.model import DecodeGraph
    from utttcompanion_b200.workloads import perturbed_persona_states
    cfg = _tiny_cfg()
    sd = reference_init_state_dict(cfg, seed=9)
    P = 2
    eng = UtttB200(sd, cfg, max_personas=P)
    w = perturbed_persona_states(sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"],
                                 sd["fast_weight_pool.w_down_init"], P, std=1e-2, seed=4)
    packed, down = eng.read_copies(*w)
    graph = DecodeGraph(eng, P, packed, down)
    dev = torch.device("cuda")
    for slot in range(3):                      # grow every workspace slot the decode step uses
        workspace(workspace(0, dev, slot).numel() * 4, dev, slot)
    junk = [torch.full((1 << 20,), 7.0, device=dev) for _ in range(16)]   # take the allocator's free blocks
    gen = torch.Generator().manual_seed(2)
    lens = [20, 33]
    firsts = [eng.prefill(torch.randint(6, cfg.vocab_size, (n,), generator=gen), p, packed, down, p)
              for p, n in enumerate(lens)]
    toks, _ = eng.greedy(torch.stack(firsts))
    pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
    k_save = [k.clone() for k in eng.k_ring]
    v_save = [v.clone() for v in eng.v_ring]
    t_g, p_g, graph_logits = toks.clone(), pos.clone(), []
    for _ in range(4):
        ids, lg = graph.step(t_g, p_g)
        graph_logits.append(lg.clone())
        t_g, p_g = ids.clone(), p_g + 1
    for i in range(cfg.n_layers):
        eng.k_ring[i].copy_(k_save[i])
        eng.v_ring[i].copy_(v_save[i])
    t_e, p_e = toks.clone(), pos.clone()
    slots = torch.arange(P, dtype=torch.int32, device="cuda")
    for s in range(4):
        lg = eng.decode_step(t_e, p_e, slots, packed, down, slots)
        assert torch.max(torch.abs(lg - graph_logits[s])).item() <= 1e-2, s
        t_e, _ = eng.greedy(lg)
        p_e = p_e + 1
    assert all(float(j[0]) == 7.0 for j in junk)   # the graph wrote into none of them


def test_151m_shape_decode_and_write_against_oracle():
    """BASELINE config 3's model shape (d=768, 12 layers, 12 query heads over 4 KV heads of
    dim 64, window 512, h=2048, V=32000; reference seed-0 init): a 96-token prompt, 8
    teacher-forced decode steps at batch 1 (the cluster-split readout, attention and
    projection finish) and a masked write of prompt + reply (2 chunks x 12 layers).

    At this depth BF16 rounding alone moves the reference's logits by ~5e-2 (its BF16
    path against its own FP32 path), more than the fixed 2e-2 bound the small models
    use.  So each step's bound is calibrated by the oracle: the largest |BF16 - FP32|
    of the oracle's logits at that step, times 1.5 (never below 2e-2)."""
    from utttcompanion_b200.workloads import CONFIG_151M
    cfg = CONFIG_151M
    sd = reference_init_state_dict(cfg, seed=0)
    eng = UtttB200(sd, cfg, max_personas=1)
    ocfg = om.ModelConfig(**{k: v for k, v in cfg.to_dict().items() if k in om.ModelConfig.__dataclass_fields__})
    oracle = om.OracleModel({k: v.numpy() for k, v in sd.items()}, ocfg, "bf16",
                            *[t.numpy() for t in (eng.rope_cos.cpu(), eng.rope_sin.cpu())])
    gen = torch.Generator().manual_seed(3)
    prompt = torch.randint(6, cfg.vocab_size, (96,), generator=gen)
    ost = oracle.state_for_forward(1, update=True)
    n_steps = 8
    oid, omargins, olog = oracle.generate_greedy(prompt.numpy(), ost, n_steps)
    o32 = om.OracleModel({k: v.numpy() for k, v in sd.items()}, ocfg, "f32",
                         *[t.numpy() for t in (eng.rope_cos.cpu(), eng.rope_sin.cpu())])
    olog32 = o32.teacher_forced_logits(prompt.numpy(), oid, o32.state_for_forward(1, update=True))
    st = eng.init_fast_state(1)
    tf = eng.teacher_forced_logits(prompt, oid, st)
    torch.cuda.synchronize()
    for step in range(n_steps):
        ours = tf[step].float().cpu().numpy()
        noise = float(np.max(np.abs(np.asarray(olog[step], np.float64) - olog32[step])))
        bound = max(LOGIT_TOL, 1.5 * noise)
        err = float(np.max(np.abs(ours - olog[step])))
        assert err <= bound, (step, err, noise)
        if int(np.argmax(_mask(ours, oracle.active_limit))) != oid[step]:
            assert omargins[step] <= 2 * bound, (step, omargins[step])
    turn = prompt.tolist() + oid
    C = cfg.chunk_size
    padded = ((len(turn) + C - 1) // C) * C
    inter = np.array(turn + [0] * (padded - len(turn)))
    mask = np.array([1.0] * len(turn) + [0.0] * (padded - len(turn)), np.float32)
    on, oms, opl, _ = oracle.test_time_update(inter[None], ost, mask[None])
    new, ms, pl = eng.test_time_update(torch.tensor(inter), st, torch.tensor(mask))
    torch.cuda.synchronize()
    assert new.step == on.step == (padded // C) * cfg.n_layers
    for n in ("w_up", "w_gate", "w_down"):
        got, ref, base = getattr(new, n).cpu().numpy(), getattr(on, n), getattr(ost, n)
        assert rel_l2(got, ref) < 5e-3, (n, rel_l2(got, ref))
        assert rel_l2(got - base, ref - base) < 3e-2, (n, rel_l2(got - base, ref - base))
    np.testing.assert_allclose(pl, opl, rtol=1e-2)

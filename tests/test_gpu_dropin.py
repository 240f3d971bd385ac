"""GPU: the drop-ins inside the reference's own code, against the unpatched reference on the
same B200.

The reference (installed under baseline/_ref; the test is skipped without it) builds
BASELINE config 1 (seed-0 init, BF16 weights, FP32 fast-weight masters, CUDA autocast as its
personalizer serves).  Unpatched, it gives the expected 64 stop-free greedy ids, their
teacher-forced logits and the written state of prompt + reply.  Then:

  * ``dropin.install(model.uttt_layer, engine.inference)`` swaps the B200 operator drop-ins
    and the B200 ``CUDAGraphDecoder`` into the reference's modules, and the reference's own
    ``stream_generate`` (eager and with ``use_cuda_graph=True``), ``forward`` and
    ``test_time_update`` run again;
  * ``uTTTModelB200.from_reference(model)`` runs the same calls on the B200 engine alone.

Bounds (tests/parity.py): logits 2e-2, or 2x the reference's BF16-vs-FP32 spread at that
step (the FP32 reference runs on the same GPU); greedy ids equal, or a near-tie flip; the
written state 1e-3, or 2x the reference's own BF16-vs-FP32 spread of it.
"""

import os
import sys
from unittest.mock import patch

import numpy as np
import pytest
import torch

from conftest import ROOT, record
from parity import NAMES, check_free_running, check_logits, check_state
from oracle.numerics import rel_l2

REF = os.path.join(ROOT, "baseline", "_ref")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "model")),
                                 reason="the reference is not installed under baseline/_ref")]
N_GEN = 64


def _modules():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import engine.inference as inference
    import model.uttt_layer as uttt_layer
    import model.uttt_model as uttt_model
    return uttt_layer, uttt_model, inference


def _greedy_without_stops(logits, **kwargs):
    """Stop-free greedy, as the reference's tests/test_inference_cuda_graph.py:37-44 patches it."""
    scores = logits.float().clone()
    scores[:, :6] = -torch.inf
    limit = kwargs.get("active_vocab_limit")
    if limit is not None:
        scores[:, limit:] = -torch.inf
    return scores.argmax(dim=-1)


def _reference_model(um, dtype):
    cfg = um.uTTTConfig(vocab_size=8000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=4, d_ff_fast=688,
                        sliding_window_size=128, chunk_size=64)
    torch.manual_seed(0)
    model = um.uTTTModel(cfg).eval().requires_grad_(False)
    w0 = {n: p.detach().clone() for n, p in model.fast_weight_pool.named_parameters()}
    model = model.to(device="cuda", dtype=dtype)
    for n, p in model.fast_weight_pool.named_parameters():      # FP32 fast-weight pool, as served
        p.data = w0[n].to(device="cuda", dtype=torch.float32)
    return model


def _autocast(dtype):
    return torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16)


def _generate(model, state, prompt, graph, dtype):
    with torch.no_grad(), _autocast(dtype), patch.object(model, "_sample_next_token",
                                                         side_effect=_greedy_without_stops):
        return list(model.stream_generate(prompt, fast_state=state, max_new_tokens=N_GEN, temperature=0.0,
                                          eos_token_id=None, speculative_draft_k=0, use_cuda_graph=graph))


def _teacher_forced(model, state, prompt, ids, dtype):
    with torch.no_grad(), _autocast(dtype):
        pre = model(prompt, fast_state=state, update_fast_weights=False, logits_to_keep=1, return_fast_state=False)
        out = [pre.logits[0, -1].float()]
        caches, pos = pre.kv_caches, prompt.shape[1]
        for tok in ids[:-1]:
            step = model(torch.tensor([[tok]], device="cuda"), fast_state=state, kv_caches=caches, start_pos=pos,
                         update_fast_weights=False, return_fast_state=False)
            caches, pos = step.kv_caches, pos + 1
            out.append(step.logits[0, -1].float())
    return torch.stack(out).cpu().numpy()


def _write(model, state, inter, mask, dtype):
    with torch.no_grad(), _autocast(dtype):
        return model.test_time_update(inter, state, mask)


def _turn(prompt, ids, C=64):
    turn = prompt[0].tolist() + list(ids)
    padded = ((len(turn) + C - 1) // C) * C
    inter = torch.tensor([turn + [0] * (padded - len(turn))], device="cuda")
    mask = torch.tensor([[1.0] * len(turn) + [0.0] * (padded - len(turn))], device="cuda")
    return inter, mask


@pytest.fixture(scope="module")
def reference_run():
    ul, um, inf = _modules()
    gen = torch.Generator().manual_seed(0)
    prompt = torch.randint(6, 8000, (1, 256), generator=gen).cuda()
    bf, f32 = torch.bfloat16, torch.float32
    model = _reference_model(um, bf)
    state = model.init_fast_state(batch_size=1, dtype=f32, detach=True)
    ids = _generate(model, state, prompt, False, bf)
    logits = _teacher_forced(model, state, prompt, ids, bf)
    inter, mask = _turn(prompt, ids)
    new, surprise, layers = _write(model, state, inter, mask, bf)
    ref32 = _reference_model(um, f32)
    st32 = ref32.init_fast_state(batch_size=1, dtype=f32, detach=True)
    logits32 = _teacher_forced(ref32, st32, prompt, ids, f32)
    new32, _, _ = _write(ref32, st32, inter, mask, f32)
    del ref32
    spread = [float(np.max(np.abs(a - b))) for a, b in zip(logits, logits32)]
    state_spread = {n: rel_l2(getattr(new, n).float().cpu().numpy(), getattr(new32, n).float().cpu().numpy())
                    for n in NAMES}
    base = {n: getattr(state, n).float().cpu().numpy() for n in NAMES}
    return dict(modules=(ul, um, inf), model=model, state=state, prompt=prompt, ids=ids, logits=logits,
                inter=inter, mask=mask, new={n: getattr(new, n).float().cpu().numpy() for n in NAMES},
                new32={n: getattr(new32, n).float().cpu().numpy() for n in NAMES}, surprise=surprise, layers=layers,
                spread=spread, state_spread=state_spread, base=base, limit=int(model.active_vocab_limit))


def _check_all(name, r, ids_free, logits_tf, new_state, surprise, layers):
    n, _ = check_logits(name, logits_tf, r["logits"], r["spread"], r["ids"], r["limit"])
    assert n == N_GEN
    check_free_running(name, ids_free, r["ids"], r["logits"], r["spread"], r["limit"])
    check_state(name, new_state, r["new"], r["base"], r["state_spread"], extra=r["new32"])
    assert abs(surprise - r["surprise"]) <= 1e-2 * abs(r["surprise"]), (surprise, r["surprise"])
    np.testing.assert_allclose(layers, r["layers"], rtol=1e-2)


def test_reference_model_with_b200_dropins_installed(reference_run):
    """The reference's own uTTTModel with the B200 operator drop-ins and CUDAGraphDecoder swapped
    into its modules: eager and graph greedy decode, teacher-forced logits and the write."""
    from utttcompanion_b200 import dropin
    r = reference_run
    ul, um, inf = r["modules"]
    model, state, prompt = r["model"], r["state"], r["prompt"]
    replaced = dropin.install(ul, inf)
    try:
        assert ul.fused_chunk_ttt_step is not replaced["uttt_layer.fused_chunk_ttt_step"]
        assert inf.CUDAGraphDecoder is dropin.CUDAGraphDecoder
        bf = torch.bfloat16
        ids_eager = _generate(model, state, prompt, False, bf)
        model._cuda_graph_decoder = None
        ids_graph = _generate(model, state, prompt, True, bf)
        assert isinstance(getattr(model, "_cuda_graph_decoder", None), dropin.CUDAGraphDecoder)
        logits = _teacher_forced(model, state, prompt, r["ids"], bf)
        new, surprise, layers = _write(model, state, r["inter"], r["mask"], bf)
    finally:
        dropin.uninstall(replaced, ul, inf)
        model._cuda_graph_decoder = None
    assert ul.fused_chunk_ttt_step is replaced["uttt_layer.fused_chunk_ttt_step"]
    _check_all("dropin_installed", r, ids_eager, logits, new, surprise, layers)
    check_free_running("dropin_installed_graph", ids_graph, r["ids"], r["logits"], r["spread"], r["limit"])
    record("dropin_installed", graph_equals_eager_steps=sum(int(a == b) for a, b in zip(ids_graph, ids_eager)))


def test_uttt_model_b200_surface_against_reference(reference_run):
    """uTTTModelB200 (the B200 engine behind uTTTModel's signatures): stream_generate, forward
    (prefill and KV-cache continuation) and test_time_update."""
    from utttcompanion_b200 import dropin
    r = reference_run
    m = dropin.uTTTModelB200.from_reference(r["model"])
    assert m.active_vocab_limit == r["limit"]
    state = m.init_fast_state(1)
    prompt = r["prompt"]
    with patch.object(m, "_sample_next_token", side_effect=_greedy_without_stops):
        ids = list(m.stream_generate(prompt, state, max_new_tokens=N_GEN, temperature=0.0, eos_token_id=None))
        ids_graph = list(m.stream_generate(prompt, state, max_new_tokens=N_GEN, temperature=0.0, eos_token_id=None,
                                           use_cuda_graph=True))
    # teacher-forced through forward(): prefill, then one-token continuations from the returned caches
    pre = m.forward(prompt, fast_state=state, update_fast_weights=False, logits_to_keep=1)
    out = [pre.logits[0, -1].float()]
    caches, pos = pre.kv_caches, prompt.shape[1]
    assert caches[0][0].shape == (1, 4, 128, 64)
    for tok in r["ids"][:-1]:
        step = m.forward(torch.tensor([[tok]], device="cuda"), fast_state=state, kv_caches=caches, start_pos=pos,
                         update_fast_weights=False)
        caches, pos = step.kv_caches, pos + 1
        out.append(step.logits[0, -1].float())
    logits = torch.stack(out).cpu().numpy()
    new, surprise, layers = m.test_time_update(r["inter"], state, r["mask"])
    assert new.step == 5 * 4
    _check_all("uttt_model_b200", r, ids, logits, new, surprise, layers)
    # the captured step follows the reference as the eager one does (step 0 of this prompt is a
    # one-ULP near-tie, so nondeterministic FP32 summation order may pick either side of it)
    check_free_running("uttt_model_b200_graph", ids_graph, r["ids"], r["logits"], r["spread"], r["limit"])
    # the input state is untouched (the reference publishes a new state object)
    assert torch.equal(state.w_up, m.init_fast_state(1).w_up)


def test_sample_next_token_matches_reference(reference_run):
    """Greedy and nucleus sampling against the reference's own _sample_next_token with the same
    generator seed (same masks, penalty, renormalisation and draw)."""
    from utttcompanion_b200 import dropin
    _, um, _ = reference_run["modules"]
    g = torch.Generator(device="cuda").manual_seed(3)
    logits = torch.randn(4, 8000, device="cuda", generator=g) * 3
    recent = [7, 9, 9, 4000]
    for temp, top_p, pen in ((0.0, 0.9, 1.0), (0.7, 0.9, 1.18), (1.0, 1.0, 1.0), (0.5, 0.3, 1.3)):
        ga = torch.Generator(device="cuda").manual_seed(11)
        gb = torch.Generator(device="cuda").manual_seed(11)
        a = dropin.sample_next_token(logits, temp, top_p, recent, pen, 7000, ga)
        b = um.uTTTModel._sample_next_token(logits, temp, top_p, recent, pen, 7000, gb)
        assert torch.equal(a, b), (temp, top_p, pen)


def test_personalizer_text_turns_with_the_reference_tokenizer(reference_run, tmp_path):
    """uTTTPersonalizerB200 over the serving engine, fed text through the reference's own tokenizer
    and chat-template encoder: the reply is the batch-1 greedy reply of the frozen persona, the
    write runs on the reference's re-tokenised '<|user|> ... <|assistant|> ...' turn, the gate and
    elastic pull follow, the persona file is saved, and the streamed events come in the
    reference's order with text content."""
    from engine.prompting import encode_chat_prompt
    from model.uttt_model import SimpleUTF8Tokenizer
    from utttcompanion_b200 import dropin
    from utttcompanion_b200.model import UtttB200
    from utttcompanion_b200.pool import SharedFastWeightPoolB200
    from utttcompanion_b200.serving import ServingEngine
    from utttcompanion_b200.workloads import CONFIG_TINY, reference_init_state_dict
    tok = SimpleUTF8Tokenizer()
    sd = reference_init_state_dict(CONFIG_TINY, seed=0)
    eng = UtttB200(sd, CONFIG_TINY, max_personas=3)
    srv = ServingEngine(eng, capacity=2, max_batch=2, surprise_threshold=0.0, elastic_anchor_lambda=0.02,
                        max_weight_drift_ratio=0.35)
    p = dropin.uTTTPersonalizerB200(srv, tokenizer=tok, encode_prompt=encode_chat_prompt, persona_dir=str(tmp_path))
    text = "Hello there, how are you today?"
    events = list(p.stream_interact_and_evolve("alice", text, max_new_tokens=16, temperature=0.0))
    assert [e["type"] for e in events[:-1]] == ["token"] * (len(events) - 1)
    assert events[-1]["type"] == "ttt_status"
    res = events[-1]["result"]
    assert res["user_id"] == "alice" and res["prompt"] == text and isinstance(res["reply"], str)
    assert res["persona_saved"] and os.path.exists(res["persona_path"])
    prompt_ids = encode_chat_prompt(tok, text, CONFIG_TINY.max_seq_len - 16)
    assert res["prompt_ids"] == prompt_ids
    # the same turn by hand on a fresh engine: batch-1 greedy with the stop rules, then the write
    # on the re-tokenised turn text, the gate (threshold 0) and the elastic pull
    ref = UtttB200(sd, CONFIG_TINY, max_personas=1)
    st = ref.init_fast_state(1)
    reply, _, _ = ref.generate_greedy(torch.tensor(prompt_ids), st, 16, stop_free=False, eos_token_id=2)
    assert res["reply_ids"] == reply
    reply_text = tok.decode(reply, skip_special_tokens=True).strip() or "[Acknowledged]"
    assert res["reply"] == reply_text
    turn = tok.encode(f"<|user|> {text}\n<|assistant|> {reply_text}", add_bos=True, add_eos=True,
                      max_length=CONFIG_TINY.max_seq_len)
    padded = ((len(turn) + 63) // 64) * 64
    new, s, per_layer = ref.test_time_update(torch.tensor(turn + [0] * (padded - len(turn))), st,
                                             torch.tensor([1.0] * len(turn) + [0.0] * (padded - len(turn))))
    pool = SharedFastWeightPoolB200(*ref.w0, ref.ln_w, ref.ln_b)
    pulled = pool.apply_elastic_pull(new, 0.02, 0.35)
    assert abs(res["surprise_loss"] - s) <= 1e-4 * abs(s)
    assert res["gate_triggered"] and res["step"] == new.step
    exported = srv.arena.export_user("alice")
    for n in NAMES:
        got = torch.as_tensor(exported[n]).reshape(getattr(pulled, n).shape).numpy()
        assert rel_l2(got, getattr(pulled, n).cpu().numpy()) < 1e-3, n
    # a second turn resumes from the committed persona
    res2 = p.interact_and_evolve("alice", "And tomorrow?", max_new_tokens=8, temperature=0.0)
    assert isinstance(res2, dropin.EvolutionResult) and res2.step > res["step"]
    with pytest.raises(ValueError):
        p.interact_and_evolve("alice", "sampled", max_new_tokens=8, temperature=0.7)

"""Generate the golden fixtures that pin the oracle to the reference.

Run on a host where the reference checkout is importable::

    python tests/golden/make_golden.py --reference /path/to/uTTTCompanion

It imports the reference's own ``model.uttt_layer`` / ``model.uttt_model``
(no copy of its code lives in this repository), runs them on CPU on seeded
inputs, and writes ``tests/golden/*.npz``.  The fixtures are small (tiny
dimensions; the algorithms are dimension-agnostic) and are committed, so
the tests never need the reference at run time.

Cases:
  chunk_*    fused_chunk_ttt_step + analytical_swiglu_chunk_grad in FP64,
             FP32 and BF16-activation / FP32-master form, with and without
             token masks, momentum and gradient clipping, q != k and a
             separate read snapshot.
  swiglu_*   swiglu_fast_forward.
  elastic    apply_elastic_pull(+drift clamp) and compute_drift.
  model_*    a small uTTTModel (FP64, FP32, and BF16 params under CPU
             autocast): stop-free greedy decode, teacher-forced logits and
             a masked test_time_update on prompt+reply.
  init_cfg1  checksums of the reference's seed-0 config-1 initialisation.
  config1_reference  BASELINE config 1 (seed-0 init, 256-token prompt, 64 stop-free greedy
             steps, the write on prompt + reply) in FP32 and in BF16 under autocast.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    if t is None:
        return None
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.numpy().copy()


def chunk_case(ul, name, dtype, act_dtype, B, C, d, h, mask, beta, clip, q_is_k, separate_read, seed,
               normalize=True, eps=1e-5):
    g = torch.Generator().manual_seed(seed)
    mdt = dtype

    def rn(*shape, scale=1.0, dt=mdt):
        return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).to(dt)

    def unit_rows():
        x = torch.randn(B, C, d, generator=g, dtype=torch.float64)
        return (x / x.norm(dim=-1, keepdim=True)).to(act_dtype)    # L2-normalised tokens

    k = unit_rows()
    v = unit_rows()
    q = k.clone() if q_is_k else unit_rows()
    eta = (torch.rand(B, C, 1, generator=g, dtype=torch.float64) * 0.05 + 0.005).to(act_dtype)
    alpha = (torch.rand(B, C, 1, generator=g, dtype=torch.float64) * 0.01).to(act_dtype)
    w_up = rn(B, d, h, scale=d ** -0.5)
    w_gate = rn(B, d, h, scale=d ** -0.5)
    w_down = rn(B, h, d, scale=0.3 * h ** -0.5)
    s_up = rn(B, d, h, scale=1e-3)
    s_gate = rn(B, d, h, scale=1e-3)
    s_down = rn(B, h, d, scale=1e-3)
    ln_w = 1.0 + rn(d, scale=0.1)
    ln_b = rn(d, scale=0.1)
    if mask == "ragged":
        m = torch.ones(B, C, dtype=mdt)
        for b in range(B):
            valid = [C, C // 2 + 1, 0, 3][b % 4]
            m[b, valid:] = 0
    else:
        m = None
    if separate_read:
        r_up = w_up + rn(B, d, h, scale=1e-2)
        r_gate = w_gate + rn(B, d, h, scale=1e-2)
        r_down = w_down + rn(B, h, d, scale=1e-2)
    else:
        r_up = r_gate = r_down = None
    with torch.no_grad():
        grads = ul.analytical_swiglu_chunk_grad(k, v, eta, w_up, w_gate, w_down, ln_w, ln_b,
                                                token_mask=m, normalize_by_dim=normalize, eps=eps)
        res = ul.fused_chunk_ttt_step(q, k, v, eta, alpha, w_up, w_gate, w_down, s_up, s_gate, s_down,
                                      ln_w, ln_b, m, beta, clip, normalize, eps, r_up, r_gate, r_down)
    out = dict(q=q, k=k, v=v, eta=eta, alpha=alpha, w_up=w_up, w_gate=w_gate, w_down=w_down,
               s_up=s_up, s_gate=s_gate, s_down=s_down, ln_weight=ln_w, ln_bias=ln_b, mask=m,
               read_w_up=r_up, read_w_gate=r_gate, read_w_down=r_down,
               grad_w_up=grads[0], grad_w_gate=grads[1], grad_w_down=grads[2], grad_surprise=grads[3],
               out=res[0], new_w_up=res[1], new_w_gate=res[2], new_w_down=res[3], new_s_up=res[4],
               new_s_gate=res[5], new_s_down=res[6], surprise=res[7])
    arrays = {key: _np(val) for key, val in out.items() if val is not None}
    arrays["meta"] = np.array([beta, clip, float(normalize), eps], np.float64)
    arrays["act_is_bf16"] = np.array(act_dtype == torch.bfloat16)
    np.savez_compressed(os.path.join(HERE, f"chunk_{name}.npz"), **arrays)


def swiglu_case(ul, name, act_dtype, seed, T=5, B=2, d=256, h=160):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, d, generator=g).to(act_dtype)
    w_up = torch.randn(B, d, h, generator=g) * d ** -0.5
    w_gate = torch.randn(B, d, h, generator=g) * d ** -0.5
    w_down = torch.randn(B, h, d, generator=g) * 0.3 * h ** -0.5
    ln_w = 1 + 0.1 * torch.randn(d, generator=g)
    ln_b = 0.1 * torch.randn(d, generator=g)
    with torch.no_grad():
        y = ul.swiglu_fast_forward(x, w_up, w_gate, w_down, ln_w, ln_b, 1e-5)
        packed = torch.cat((w_up.to(act_dtype), w_gate.to(act_dtype)), dim=-1)
        yp = ul.swiglu_packed_forward(x, packed, w_down.to(act_dtype), ln_w, ln_b, 1e-5)
    np.savez_compressed(os.path.join(HERE, f"swiglu_{name}.npz"), x=_np(x), w_up=_np(w_up), w_gate=_np(w_gate),
                        w_down=_np(w_down), ln_weight=_np(ln_w), ln_bias=_np(ln_b), out=_np(y),
                        out_packed=_np(yp), act_is_bf16=np.array(act_dtype == torch.bfloat16))


def elastic_case(ul):
    torch.manual_seed(11)
    pool = ul.SharedFastWeightPool(16, 24)
    state = pool.init_state(batch_size=2, detach=True)
    g = torch.Generator().manual_seed(12)
    state.w_up = state.w_up + 0.5 * torch.randn(state.w_up.shape, generator=g)
    state.w_gate = state.w_gate + 0.05 * torch.randn(state.w_gate.shape, generator=g)
    state.w_down = state.w_down + 0.2 * torch.randn(state.w_down.shape, generator=g)
    pulled = pool.apply_elastic_pull(state, anchor_lambda=0.02, max_drift_ratio=0.35)
    pulled_nc = pool.apply_elastic_pull(state, anchor_lambda=0.05, max_drift_ratio=None)
    one = ul.FastWeightState(state.w_up[:1], state.w_gate[:1], state.w_down[:1], state.s_up[:1],
                             state.s_gate[:1], state.s_down[:1], state.ln_weight, state.ln_bias)
    drift = pool.compute_drift(one)
    keys = sorted(k for k, v in drift.items() if isinstance(v, float) and k not in ("last_surprise_loss",))
    np.savez_compressed(
        os.path.join(HERE, "elastic.npz"),
        w_up0=_np(pool.w_up_init), w_gate0=_np(pool.w_gate_init), w_down0=_np(pool.w_down_init),
        w_up=_np(state.w_up), w_gate=_np(state.w_gate), w_down=_np(state.w_down),
        p_up=_np(pulled.w_up), p_gate=_np(pulled.w_gate), p_down=_np(pulled.w_down),
        n_up=_np(pulled_nc.w_up), n_gate=_np(pulled_nc.w_gate), n_down=_np(pulled_nc.w_down),
        drift_keys=np.array(keys), drift_vals=np.array([drift[k] for k in keys], np.float64))


SMALL = dict(vocab_size=512, d_model=128, n_layers=2, n_heads=4, n_kv_heads=2, d_ff_fast=160,
             sliding_window_size=16, max_seq_len=256, chunk_size=16, gradient_checkpointing=False,
             dropout=0.0)


def greedy_without_stops(logits, **kwargs):
    """Same stop-free greedy as the reference's tests/test_inference_cuda_graph.py:37-44."""
    scores = logits.float().clone()
    scores[:, :6] = -torch.inf
    limit = kwargs.get("active_vocab_limit")
    if limit is not None:
        scores[:, limit:] = -torch.inf
    return scores.argmax(dim=-1)


def model_case(um, name, dtype, autocast_bf16, seed=2024, n_prompt=37, n_gen=20):
    torch.manual_seed(seed)
    cfg = um.uTTTConfig(**SMALL)
    model = um.uTTTModel(cfg).eval().requires_grad_(False)
    with torch.no_grad():
        for block in model.layers:          # make positions visible above rounding noise
            block.attn.wq.weight.mul_(3)
            block.attn.wk.weight.mul_(3)
        # non-trivial eta/alpha routers and LN so every term of the write is exercised
        for block in model.layers:
            block.uttt.w_eta.weight.normal_(0, 0.05)
            block.uttt.w_alpha.weight.normal_(0, 0.05)
        model.fast_weight_pool.ln_weight.add_(0.1 * torch.randn(cfg.d_model))
        model.fast_weight_pool.ln_bias.add_(0.1 * torch.randn(cfg.d_model))
    weights = {k: _np(v.float() if v.dtype != torch.float64 else v) for k, v in model.state_dict().items()}
    if dtype == torch.float64:
        model = model.double()
    elif autocast_bf16:
        model = model.to(torch.bfloat16)
        # FP32 fast-weight masters (W_0 unrounded), as the persona path keeps them
        for n, p in model.fast_weight_pool.named_parameters():
            p.data = torch.tensor(weights["fast_weight_pool." + n], dtype=torch.float32)
    gen = torch.Generator().manual_seed(seed + 1)
    prompt = torch.randint(6, cfg.vocab_size, (1, n_prompt), generator=gen)
    state_dtype = torch.float64 if dtype == torch.float64 else torch.float32
    state = model.init_fast_state(batch_size=1, dtype=state_dtype, detach=True)
    # perturb the persona away from W_0 as BASELINE config 3 does
    pg = torch.Generator().manual_seed(seed + 2)
    for nm in ("w_up", "w_gate", "w_down"):
        t = getattr(state, nm)
        delta = (1e-2 * torch.randn(t.shape, generator=pg, dtype=torch.float64)).float()
        setattr(state, nm, (t.float() + delta).to(t.dtype))
    ctx = torch.autocast("cpu", dtype=torch.bfloat16) if autocast_bf16 else torch.autocast("cpu", enabled=False)
    out = {}
    with torch.no_grad(), ctx:
        from unittest.mock import patch
        with patch.object(model, "_sample_next_token", side_effect=greedy_without_stops):
            ids = list(model.stream_generate(prompt, fast_state=state, max_new_tokens=n_gen, temperature=0.0,
                                             eos_token_id=None, speculative_draft_k=0, use_cuda_graph=False))
        # teacher-forced logits along the generated ids
        pre = model(prompt, fast_state=state, update_fast_weights=False, logits_to_keep=1, return_fast_state=False)
        logits = [pre.logits[0, -1].float()]
        caches, pos = pre.kv_caches, prompt.shape[1]
        for tok in ids[:-1]:
            step = model(torch.tensor([[tok]]), fast_state=state, kv_caches=caches, start_pos=pos,
                         update_fast_weights=False, return_fast_state=False)
            caches, pos = step.kv_caches, pos + 1
            logits.append(step.logits[0, -1].float())
        # write on prompt + reply, right-padded to a multiple of chunk_size with a mask
        turn = prompt[0].tolist() + ids
        C = cfg.chunk_size
        padded = ((len(turn) + C - 1) // C) * C
        inter = torch.tensor([turn + [0] * (padded - len(turn))])
        mask = torch.tensor([[1.0] * len(turn) + [0.0] * (padded - len(turn))])
        new_state, mean_surprise, layer_surprises = model.test_time_update(inter, state, mask)
    out.update(weights={}, prompt=prompt[0].numpy(), ids=np.array(ids), logits=np.stack([_np(x) for x in logits]),
               inter=inter[0].numpy(), mask=mask[0].numpy(),
               state_w_up=_np(state.w_up), state_w_gate=_np(state.w_gate), state_w_down=_np(state.w_down),
               new_w_up=_np(new_state.w_up), new_w_gate=_np(new_state.w_gate), new_w_down=_np(new_state.w_down),
               new_s_up=_np(new_state.s_up), new_s_gate=_np(new_state.s_gate), new_s_down=_np(new_state.s_down),
               new_step=np.array(new_state.step), mean_surprise=np.array(mean_surprise),
               layer_surprises=np.array(layer_surprises), active_limit=np.array(model.active_vocab_limit),
               rope_cos=_np(model.layers[0].attn.rope.cos_cached.float()),
               rope_sin=_np(model.layers[0].attn.rope.sin_cached.float()))
    out.pop("weights")
    arrays = dict(out)
    # weights and the starting persona state are identical for every dtype case: stored once
    shared = {"W::" + k: v for k, v in weights.items()}
    shared.update(cfg_json=np.array(repr(SMALL)), prompt=arrays["prompt"], rope_cos=arrays.pop("rope_cos"),
                  rope_sin=arrays.pop("rope_sin"), active_limit=arrays["active_limit"],
                  state_w_up=arrays.pop("state_w_up").astype(np.float32),
                  state_w_gate=arrays.pop("state_w_gate").astype(np.float32),
                  state_w_down=arrays.pop("state_w_down").astype(np.float32))
    path = os.path.join(HERE, "model_shared.npz")
    if name == "f32":
        np.savez_compressed(path, **shared)
    np.savez_compressed(os.path.join(HERE, f"model_{name}.npz"), **arrays)


def config1_case(um, n_prompt=256, n_gen=64):
    """BASELINE config 1 run by the reference itself: seed-0 init, a 256-token prompt of ids
    uniform in [6, 8000) from Generator seed 0, 64 stop-free greedy steps with their
    teacher-forced logits, then test_time_update on prompt + reply (T = 320: 5 chunks x 4 layers).

    Two dtype flows of the same model: FP32 (BASELINE's own spec) and BF16 parameters under CPU
    autocast with FP32 fast-weight masters (the serving flow).  Both write the SAME interaction
    (prompt + the BF16 run's reply), so their states can be compared with each other: the
    distance between them is the reference's own BF16 rounding spread.  Logits of the BF16 run
    are BF16 and are stored as their bit patterns."""
    cfg = um.uTTTConfig(vocab_size=8000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=4, d_ff_fast=688,
                        sliding_window_size=128, chunk_size=64)
    gen = torch.Generator().manual_seed(0)
    prompt = torch.randint(6, cfg.vocab_size, (1, n_prompt), generator=gen)
    runs = {}
    for name in ("bf16", "f32"):
        torch.manual_seed(0)
        model = um.uTTTModel(cfg).eval().requires_grad_(False)
        autocast_bf16 = name == "bf16"
        if autocast_bf16:
            w0 = {n: p.detach().clone() for n, p in model.fast_weight_pool.named_parameters()}
            model = model.to(torch.bfloat16)
            for n, p in model.fast_weight_pool.named_parameters():
                p.data = w0[n].float()
        state = model.init_fast_state(batch_size=1, dtype=torch.float32, detach=True)
        ctx = torch.autocast("cpu", dtype=torch.bfloat16) if autocast_bf16 else torch.autocast("cpu", enabled=False)
        from unittest.mock import patch
        with torch.no_grad(), ctx:
            with patch.object(model, "_sample_next_token", side_effect=greedy_without_stops):
                ids = list(model.stream_generate(prompt, fast_state=state, max_new_tokens=n_gen, temperature=0.0,
                                                 eos_token_id=None, speculative_draft_k=0, use_cuda_graph=False))
            pre = model(prompt, fast_state=state, update_fast_weights=False, logits_to_keep=1,
                        return_fast_state=False)
            logits = [pre.logits[0, -1]]
            caches, pos = pre.kv_caches, prompt.shape[1]
            for tok in ids[:-1]:
                step = model(torch.tensor([[tok]]), fast_state=state, kv_caches=caches, start_pos=pos,
                             update_fast_weights=False, return_fast_state=False)
                caches, pos = step.kv_caches, pos + 1
                logits.append(step.logits[0, -1])
        runs[name] = dict(model=model, state=state, ids=ids, logits=torch.stack(logits), ctx=autocast_bf16)
    turn = prompt[0].tolist() + runs["bf16"]["ids"]
    C = cfg.chunk_size
    padded = ((len(turn) + C - 1) // C) * C
    inter = torch.tensor([turn + [0] * (padded - len(turn))])
    mask = torch.tensor([[1.0] * len(turn) + [0.0] * (padded - len(turn))])
    arrays = dict(prompt=prompt[0].numpy(), inter=inter[0].numpy(), mask=mask[0].numpy())
    for name, r in runs.items():
        ctx = torch.autocast("cpu", dtype=torch.bfloat16) if r["ctx"] else torch.autocast("cpu", enabled=False)
        with torch.no_grad(), ctx:
            new_state, mean_surprise, layer_surprises = r["model"].test_time_update(inter, r["state"], mask)
        lg = r["logits"]
        if name == "bf16":
            assert lg.dtype == torch.bfloat16
            arrays["bf16_logits_bits"] = lg.view(torch.int16).numpy().view(np.uint16)
        else:
            arrays["f32_logits"] = _np(lg.float())
        arrays[name + "_ids"] = np.array(r["ids"])
        for nm in ("w_up", "w_gate", "w_down"):
            arrays[f"{name}_new_{nm}"] = _np(getattr(new_state, nm)).astype(np.float32)
        arrays[name + "_new_step"] = np.array(new_state.step)
        arrays[name + "_mean_surprise"] = np.array(mean_surprise)
        arrays[name + "_layer_surprises"] = np.array(layer_surprises)
    arrays["active_limit"] = np.array(runs["f32"]["model"].active_vocab_limit)
    np.savez_compressed(os.path.join(HERE, "config1_reference.npz"), **arrays)


def init_checksums(um):
    """Checksums of the reference's config-1 (tiny) seed-0 init, for the synthetic weight generator."""
    torch.manual_seed(0)
    cfg = um.uTTTConfig(vocab_size=8000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=4, d_ff_fast=688,
                        sliding_window_size=128, chunk_size=64)
    model = um.uTTTModel(cfg)
    sd = model.state_dict()
    names = sorted(sd)
    sums = np.array([float(sd[n].double().sum()) for n in names])
    sq = np.array([float(sd[n].double().square().sum()) for n in names])
    first = np.stack([np.pad(sd[n].reshape(-1)[:4].double().numpy(), (0, 4 - min(4, sd[n].numel())))
                      for n in names])
    np.savez_compressed(os.path.join(HERE, "init_cfg1.npz"), names=np.array(names), sums=sums, sq=sq, first=first,
                        active_limit=np.array(um.SimpleUTF8Tokenizer.ACTIVE_VOCAB_LIMIT))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default="", help="comma-separated case groups to write (chunk, swiglu, elastic, "
                                               "model, init, config1); default all")
    args = ap.parse_args()
    only = set(filter(None, args.only.split(",")))

    def want(group):
        return not only or group in only
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    import model.uttt_layer as ul
    import model.uttt_model as um

    f64, f32, bf = torch.float64, torch.float32, torch.bfloat16
    if want("chunk"):
        _chunk_cases(ul, f64, f32, bf)
    if want("swiglu"):
        swiglu_case(ul, "f32", f32, 21, d=32, h=48)
        swiglu_case(ul, "bf16", bf, 22)
        swiglu_case(ul, "bf16_t1", bf, 23, T=1)
        swiglu_case(ul, "bf16_t70", bf, 24, T=70)
    if want("elastic"):
        elastic_case(ul)
    if want("model"):
        model_case(um, "f32", f32, False)
        model_case(um, "f64", f64, False)
        model_case(um, "bf16", f32, True)
    if want("init"):
        init_checksums(um)
    if want("config1"):
        config1_case(um)
    print("golden fixtures written to", HERE)


def _chunk_cases(ul, f64, f32, bf):
    chunk_case(ul, "f64_plain", f64, f64, 2, 8, 16, 24, None, 0.0, 0.0, True, False, 1)
    chunk_case(ul, "f64_full", f64, f64, 4, 8, 16, 24, "ragged", 0.9, 0.05, False, True, 2)
    chunk_case(ul, "f32_plain", f32, f32, 2, 16, 32, 48, None, 0.0, 0.0, True, False, 3)
    chunk_case(ul, "f32_full", f32, f32, 4, 16, 32, 48, "ragged", 0.9, 0.5, False, True, 4)
    chunk_case(ul, "bf16_plain", f32, bf, 2, 64, 128, 160, None, 0.0, 0.0, True, False, 5)
    chunk_case(ul, "bf16_full", f32, bf, 3, 64, 128, 160, "ragged", 0.9, 1.0, False, True, 6)
    chunk_case(ul, "bf16_clipbite", f32, bf, 2, 64, 128, 160, None, 0.5, 0.02, False, False, 7)


if __name__ == "__main__":
    main()

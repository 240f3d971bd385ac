"""Oracle restatement of the uTTT model forward, greedy decode and TTT write.

Reference: ``model/uttt_model.py`` and ``model/uttt_layer.py`` of
Phova/uTTTCompanion.  Weights use the reference's state-dict names
(``layers.{i}.attn.wq.weight`` ...), so a reference checkpoint's tensors can
be fed in directly (as numpy arrays).

This is test infrastructure (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import fastweight as fw
from .numerics import Precision, round_bf16, sigmoid

PAD_ID, BOS_ID, EOS_ID, UNK_ID, USER_ID, ASSISTANT_ID = 0, 1, 2, 3, 4, 5  # model/uttt_model.py:130-254


@dataclass
class ModelConfig:
    """Subset of ``uTTTConfig`` (``model/uttt_model.py:44-111``) used on the hot path."""
    vocab_size: int = 32000
    d_model: int = 1024
    n_layers: int = 16
    n_heads: int = 16
    n_kv_heads: int = 4
    d_ff_fast: int = 2816
    sliding_window_size: int = 512
    max_seq_len: int = 4096
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    chunk_size: int = 64
    base_inner_lr: float = 0.015
    base_weight_decay: float = 0.005
    momentum_beta: float = 0.90
    max_inner_grad_norm: float = 1.0
    normalize_loss_by_dim: bool = True

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


# SimpleUTF8Tokenizer.ACTIVE_VOCAB_LIMIT (model/uttt_model.py:151); the golden
# script records the reference's value and tests/test_oracle_golden.py compares.
_SIMPLE_ACTIVE_LIMIT = 21478


def active_vocab_limit(cfg: ModelConfig) -> int:
    """``uTTTModel.__init__`` (``model/uttt_model.py:294-297``) without an embedded tokenizer."""
    return _SIMPLE_ACTIVE_LIMIT if cfg.vocab_size >= 24000 else cfg.vocab_size


def rope_tables(head_dim: int, n_pos: int, theta: float = 10000.0):
    """FP32 cos/sin tables (``RotaryEmbedding._build_cache``, ``model/uttt_layer.py:910-933``)."""
    inv_freq = (np.float32(1.0) / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                                         / np.float32(head_dim)))).astype(np.float32)
    t = np.arange(0, n_pos, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


class OracleModel:
    """Numpy uTTT model over reference-named weights."""

    def __init__(self, weights: Dict[str, np.ndarray], cfg: ModelConfig, prec: str = "f32",
                 rope_cos: Optional[np.ndarray] = None, rope_sin: Optional[np.ndarray] = None):
        self.cfg = cfg
        self.prec = Precision(prec)
        self.autocast = prec == "bf16"
        p = self.prec
        # Slow weights live in the activation dtype (BF16 params in the bf16 path).
        self.w = {k: (p.act(v) if not k.startswith("fast_weight_pool.") else np.asarray(v, p.stat_dtype))
                  for k, v in weights.items()}
        n_pos = max(cfg.max_seq_len, 1)
        if rope_cos is None:
            rope_cos, rope_sin = rope_tables(cfg.head_dim, n_pos, cfg.rope_theta)
        self.cos = rope_cos
        self.sin = rope_sin
        self.active_limit = active_vocab_limit(cfg)

    # -- small ops -------------------------------------------------------------
    def linear(self, x, name):
        """``F.linear(x, W)`` with activation-dtype output."""
        return self.prec.mm(x, np.swapaxes(self.w[name], -1, -2))

    def rmsnorm(self, x, weight=None):
        """``F.rms_norm`` (``model/uttt_layer.py:881-896``): FP32 statistics, activation output."""
        p = self.prec
        xf = np.asarray(x, p.stat_dtype)
        var = np.square(xf).mean(axis=-1, keepdims=True)
        y = xf / np.sqrt(var + p.stat_dtype(self.cfg.rms_norm_eps))
        if weight is not None:
            y = y * np.asarray(p.act(weight), p.stat_dtype)
        return p.act(y)

    def state_for_forward(self, batch: int, update: bool) -> fw.OracleState:
        """Fresh state from W_0 (``model/uttt_model.py:782-795``)."""
        dt = np.float64 if self.prec.mode == "f64" else np.float32
        if not update and self.prec.mode == "bf16":
            dt = np.float32
        return fw.init_state(self.w["fast_weight_pool.w_up_init"], self.w["fast_weight_pool.w_gate_init"],
                             self.w["fast_weight_pool.w_down_init"], self.w["fast_weight_pool.ln_weight"],
                             self.w["fast_weight_pool.ln_bias"], batch, dt)

    # -- attention -------------------------------------------------------------
    def _rope(self, x, start_pos):
        """``apply_rope`` with tables cast to the activation dtype (``model/uttt_layer.py:935-958``)."""
        p = self.prec
        t = x.shape[2]
        cos = p.act(self.cos[start_pos:start_pos + t])[None, None]
        sin = p.act(self.sin[start_pos:start_pos + t])[None, None]
        half = x.shape[-1] // 2
        rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
        return p.act(p.act(x * cos) + p.act(rot * sin))

    def attention(self, i: int, x, cache=None, start_pos: int = 0):
        """``SlidingWindowAttention.forward`` in eval/no-grad (``model/uttt_layer.py:1058-1168``)."""
        cfg, p = self.cfg, self.prec
        b, t, _ = x.shape
        nh, nkv, hd, win = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.sliding_window_size
        pre = f"layers.{i}.attn."
        q = self.linear(x, pre + "wq.weight").reshape(b, t, nh, hd).transpose(0, 2, 1, 3)
        k = self.linear(x, pre + "wk.weight").reshape(b, t, nkv, hd).transpose(0, 2, 1, 3)
        v = self.linear(x, pre + "wv.weight").reshape(b, t, nkv, hd).transpose(0, 2, 1, 3)
        q = self._rope(q, start_pos)
        k = self._rope(k, start_pos)
        if cache is not None:                                          # :1082-1103
            kp, vp = cache
            hist = win - 1
            if kp.shape[2] > hist:
                kp, vp = kp[:, :, kp.shape[2] - hist:], vp[:, :, vp.shape[2] - hist:]
            k = np.concatenate([kp, k], axis=2)
            v = np.concatenate([vp, v], axis=2)
            needed = win - 1 + t
            if k.shape[2] > needed:
                k, v = k[:, :, -needed:], v[:, :, -needed:]
        new_cache = (k[:, :, -win:], v[:, :, -win:]) if k.shape[2] > win else (k, v)   # :1105-1114
        kv_len = k.shape[2]
        qpos = np.arange(kv_len - t, kv_len)[:, None]
        kpos = np.arange(kv_len)[None, :]
        allowed = (qpos >= kpos) & ((qpos - kpos) < win)
        if t == 1:
            allowed = np.ones((1, kv_len), bool)                       # :1119-1124 (no mask)
        rep = nh // nkv
        kk = np.repeat(k, rep, axis=1) if rep > 1 else k
        vv = np.repeat(v, rep, axis=1) if rep > 1 else v
        sdt = p.stat_dtype
        scores = np.matmul(np.asarray(q, sdt), np.swapaxes(np.asarray(kk, sdt), -1, -2)) * sdt(1.0 / math.sqrt(hd))
        scores = np.where(allowed[None, None], scores, -np.inf)
        scores = scores - scores.max(axis=-1, keepdims=True)
        pr = np.exp(scores)
        pr = pr / pr.sum(axis=-1, keepdims=True)
        o = p.act(np.matmul(pr, np.asarray(vv, sdt)))
        o = o.transpose(0, 2, 1, 3).reshape(b, t, cfg.d_model)
        return self.linear(o, pre + "wo.weight"), new_cache

    # -- frozen forward ----------------------------------------------------------
    def fast_q_proj(self, i: int, x):
        """``fused_fast_q_proj`` (``model/uttt_layer.py:1175-1190``)."""
        q_raw = self.linear(x, f"layers.{i}.uttt.w_q.weight")
        return self.rmsnorm(q_raw, self.w[f"layers.{i}.uttt.q_norm.weight"])

    def readout(self, q, state: fw.OracleState):
        """``SharedFastWeightPool.forward_readout`` (``model/uttt_layer.py:670-695``)."""
        return fw.swiglu_fast_forward(q, state.w_up, state.w_gate, state.w_down, state.ln_weight,
                                      state.ln_bias, self.cfg.rms_norm_eps, self.prec, self.autocast)

    def forward_frozen(self, ids, state: fw.OracleState, caches=None, start_pos: int = 0,
                       logits_to_keep: int = 0):
        """``uTTTModel.forward(update_fast_weights=False)`` (``model/uttt_model.py:813-830,944-950``)."""
        p = self.prec
        ids = np.asarray(ids)
        h = p.act(self.w["tok_embeddings.weight"][ids])
        new_caches = []
        for i in range(self.cfg.n_layers):
            a, c = self.attention(i, self.rmsnorm(h, self.w[f"layers.{i}.attn_norm.weight"]),
                                  None if caches is None else caches[i], start_pos)
            new_caches.append(c)
            h = p.act(h + a)
            x2 = self.rmsnorm(h, self.w[f"layers.{i}.uttt_norm.weight"])
            r = self.readout(self.fast_q_proj(i, x2), state)
            h = p.act(h + self.linear(p.act(r), f"layers.{i}.uttt.w_o.weight"))
        if logits_to_keep > 0 and h.shape[1] > logits_to_keep:
            h = h[:, -logits_to_keep:]
        logits = self.prec.mm(self.rmsnorm(h, self.w["norm.weight"]),
                              np.swapaxes(self.w["tok_embeddings.weight"], 0, 1))
        return logits, new_caches

    def greedy_pick(self, logits, stop_free: bool = True) -> Tuple[int, float]:
        """``_sample_next_token`` at temperature 0 (``model/uttt_model.py:1204-1221``).

        ``stop_free`` also masks the EOS/role ids 2, 4, 5 as the reference's
        own graph-vs-eager greedy test does (``tests/test_inference_cuda_graph.py:37-44``),
        so every step is compared.  Returns (id, top-1 minus top-2 margin).
        """
        work = np.asarray(logits, np.float64).reshape(-1).copy()
        work[[PAD_ID, BOS_ID, UNK_ID]] = -np.inf
        if stop_free:
            work[:6] = -np.inf
        if self.active_limit < work.shape[0]:
            work[self.active_limit:] = -np.inf
        idx = int(np.argmax(work))
        top = work[idx]
        work[idx] = -np.inf
        return idx, float(top - work.max())

    def generate_greedy(self, prompt, state: fw.OracleState, n_tokens: int, stop_on_role=False):
        """Greedy ``stream_generate`` (``model/uttt_model.py:966-1179``) without stop tokens.

        Role/EOS stops are disabled (as ``tests/test_inference_cuda_graph.py:169-176``
        does) so every step is compared.  Returns ids, margins and per-step logits.
        """
        logits, caches = self.forward_frozen(np.asarray(prompt)[None], state, None, 0, 1)
        pos = len(prompt)
        ids, margins, all_logits = [], [], []
        for _ in range(n_tokens):
            lg = logits[0, -1]
            all_logits.append(np.asarray(lg, np.float32))
            tok, margin = self.greedy_pick(lg)
            if stop_on_role and tok in (USER_ID, ASSISTANT_ID):
                break
            ids.append(tok)
            margins.append(margin)
            if len(ids) == n_tokens:
                break
            logits, caches = self.forward_frozen(np.array([[tok]]), state, caches, pos, 0)
            pos += 1
        return ids, margins, all_logits

    def teacher_forced_logits(self, prompt, forced_ids, state: fw.OracleState):
        """Last-token logits after the prompt and after each forced token."""
        logits, caches = self.forward_frozen(np.asarray(prompt)[None], state, None, 0, 1)
        out = [np.asarray(logits[0, -1], np.float32)]
        pos = len(prompt)
        for tok in forced_ids[:-1]:
            logits, caches = self.forward_frozen(np.array([[tok]]), state, caches, pos, 0)
            out.append(np.asarray(logits[0, -1], np.float32))
            pos += 1
        return out

    # -- update path -------------------------------------------------------------
    def slow_projections(self, i: int, x):
        """``fused_slow_projections`` (``model/uttt_layer.py:1193-1231``)."""
        cfg, p = self.cfg, self.prec
        pre = f"layers.{i}.uttt."
        q = self.rmsnorm(self.linear(x, pre + "w_q.weight"), self.w[pre + "q_norm.weight"])
        k = self.rmsnorm(self.linear(x, pre + "w_k.weight"), self.w[pre + "k_norm.weight"])
        v = self.rmsnorm(self.linear(x, pre + "w_v.weight"), None)
        eta_lin = p.act(self.prec.mm(x, np.swapaxes(self.w[pre + "w_eta.weight"], 0, 1)) + self.w[pre + "w_eta.bias"])
        alpha_lin = p.act(self.prec.mm(x, np.swapaxes(self.w[pre + "w_alpha.weight"], 0, 1)) + self.w[pre + "w_alpha.bias"])
        eta = p.act(p.stat_dtype(cfg.base_inner_lr) * p.act(sigmoid(np.asarray(eta_lin, p.stat_dtype))))
        alpha = p.act(p.stat_dtype(cfg.base_weight_decay) * p.act(sigmoid(np.asarray(alpha_lin, p.stat_dtype))))
        return q, k, v, eta, alpha

    def test_time_update(self, ids, state: fw.OracleState, mask=None):
        """``uTTTModel.test_time_update`` with the chunk-first shared schedule.

        Follows ``model/uttt_model.py:1237-1271`` -> ``forward`` (``:776-838``)
        -> ``_forward_shared_chunks`` (``:576-608``) -> ``_run_shared_chunk`` /
        ``_run_shared_layer_segment`` (``:453-530``).  Every layer of a chunk
        reads the chunk-start snapshot; its writes advance one cursor.
        Returns (new_state, mean_surprise, per_layer_surprises, chunk_outputs).
        """
        cfg, p = self.cfg, self.prec
        ids = np.asarray(ids)
        bsz, seq = ids.shape
        h_all = p.act(self.w["tok_embeddings.weight"][ids])
        cur = state.copy()
        caches: List[Optional[tuple]] = [None] * cfg.n_layers
        losses, counts, pieces = [], [], []
        step = cur.step
        C = cfg.chunk_size
        for off in range(0, seq, C):
            end = min(off + C, seq)
            m = None if mask is None else np.asarray(mask, np.float32)[:, off:end]
            hidden = h_all[:, off:end]
            read = cur.copy()                                          # chunk-start snapshot
            layer_losses = []
            for i in range(cfg.n_layers):
                a, c = self.attention(i, self.rmsnorm(hidden, self.w[f"layers.{i}.attn_norm.weight"]),
                                      caches[i], off)
                caches[i] = tuple(x[:, :, -cfg.sliding_window_size:] for x in c)
                hh = p.act(hidden + a)
                x2 = self.rmsnorm(hh, self.w[f"layers.{i}.uttt_norm.weight"])
                q, k, v, eta, alpha = self.slow_projections(i, x2)
                res = fw.fused_chunk_ttt_step(
                    q, k, v, eta, alpha, cur.w_up, cur.w_gate, cur.w_down, cur.s_up, cur.s_gate,
                    cur.s_down, cur.ln_weight, cur.ln_bias, m, cfg.momentum_beta,
                    float(cfg.max_inner_grad_norm or 0.0), cfg.normalize_loss_by_dim, cfg.rms_norm_eps,
                    read.w_up, read.w_gate, read.w_down, prec=p, autocast=self.autocast)
                cur.w_up, cur.w_gate, cur.w_down = res.w_up, res.w_gate, res.w_down
                cur.s_up, cur.s_gate, cur.s_down = res.s_up, res.s_gate, res.s_down
                out = self.linear(p.act(res.out), f"layers.{i}.uttt.w_o.weight")
                hidden = p.act(hh + out)
                layer_losses.append(res.surprise)
            pieces.append(hidden)
            losses.append(layer_losses)
            counts.append(float(m.sum()) if m is not None else float(bsz * (end - off)))
            step += cfg.n_layers
        L = np.asarray(losses, np.float64)
        cnt = np.asarray(counts, np.float64)
        per_layer = (L * cnt[:, None]).sum(axis=0) / max(cnt.sum(), 1.0)
        per_layer = [float(np.float32(x)) for x in per_layer]
        cur.step = step
        cur.last_surprise_loss = sum(per_layer) / max(len(per_layer), 1)
        cur.surprise_history = (list(state.surprise_history) + per_layer)[-100:]
        return cur, cur.last_surprise_loss, per_layer, pieces

"""B200 uTTT model engine behind the reference's model API.

``UtttB200`` holds a reference state dict (``uTTTModel`` parameter names) on
the GPU and runs the hot path with this package's kernels only:

* ``forward_frozen`` / ``prefill`` -- ``uTTTModel.forward(update_fast_weights=False)``
  (``model/uttt_model.py:813-830,944-950``): embedding, per block RMSNorm ->
  packed QKV -> RoPE + sliding-window attention -> wo + residual -> RMSNorm ->
  q projection + RMSNorm (``fused_fast_q_proj``) -> fast-weight readout through
  the persona's frozen weights -> w_o + residual; final RMSNorm, tied lm_head.
* ``decode_step`` -- one token for each of B personas in ONE packed batch,
  each row with its own fast-weight read copy (``state_index``) and its own
  KV ring slot and position (the multi-persona decode the reference, which is
  batch-1, serialises per persona).
* ``generate_greedy`` -- ``stream_generate`` at temperature 0.
* ``test_time_update`` -- ``uTTTModel.test_time_update`` with the chunk-first
  shared schedule (``model/uttt_model.py:453-608``): all layers of a chunk read
  the chunk-start snapshot; their writes advance one cursor.

Activations are BF16 and masters FP32, the reference's serving dtypes.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib
from .fastweight import _stream, chunk_write, check_status, workspace
from .readout import fast_readout
from .workloads import ModelConfig

PAD_ID, BOS_ID, EOS_ID, UNK_ID, USER_ID, ASSISTANT_ID = 0, 1, 2, 3, 4, 5
SIMPLE_ACTIVE_VOCAB_LIMIT = 21478          # SimpleUTF8Tokenizer.ACTIVE_VOCAB_LIMIT, model/uttt_model.py:151


@dataclass
class FastState:
    """Device mirror of ``FastWeightState`` (``model/uttt_layer.py:59-204``): FP32 masters."""
    w_up: torch.Tensor
    w_gate: torch.Tensor
    w_down: torch.Tensor
    s_up: torch.Tensor
    s_gate: torch.Tensor
    s_down: torch.Tensor
    ln_weight: torch.Tensor
    ln_bias: torch.Tensor
    step: int = 0
    last_surprise_loss: float = 0.0
    surprise_history: List[float] = field(default_factory=list)

    def clone(self) -> "FastState":
        return FastState(*(t.clone() for t in (self.w_up, self.w_gate, self.w_down, self.s_up, self.s_gate,
                                                self.s_down, self.ln_weight, self.ln_bias)),
                         int(self.step), float(self.last_surprise_loss), list(self.surprise_history[-100:]))

    def to_state_dict(self) -> Dict[str, object]:
        """Persona checkpoint payload in the reference's format (``:170-184``)."""
        d = {k: getattr(self, k).detach().cpu() for k in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down",
                                                         "ln_weight", "ln_bias")}
        d.update(step=self.step, last_surprise_loss=self.last_surprise_loss,
                 surprise_history=list(self.surprise_history[-100:]))
        return d

    @classmethod
    def from_state_dict(cls, sd: Dict[str, object], device="cuda") -> "FastState":
        t = [torch.as_tensor(sd[k]).to(device=device, dtype=torch.float32).contiguous()
             for k in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down", "ln_weight", "ln_bias")]
        for i in range(6):
            if t[i].dim() == 2:
                t[i] = t[i].unsqueeze(0)
        return cls(*t, int(sd.get("step", 0)), float(sd.get("last_surprise_loss", 0.0)),
                   list(sd.get("surprise_history", [])))


def rope_tables(head_dim: int, n_pos: int, theta: float):
    """FP32 cos/sin exactly as ``RotaryEmbedding._build_cache`` (``model/uttt_layer.py:910-933``)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(0, n_pos, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()



def _host_list(values, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A small host-side list as a device tensor without stalling the host: staged in pinned
    memory and copied asynchronously on the current stream (a plain ``torch.tensor(...,
    device=...)`` copies from pageable memory and waits for the stream to drain)."""
    if torch.device(device).type != "cuda":
        return torch.tensor(values, dtype=dtype, device=device)
    return torch.tensor(values, dtype=dtype).pin_memory().to(device, non_blocking=True)

def _seg(start, length, op, out, out_ld, aux=None, aux_ld=0, scale=0.0, out_f32=False, aux2=None):
    return _lib.Segment(start, length, op, int(out_f32), out.data_ptr(), out_ld,
                        None if aux is None else aux.data_ptr(), aux_ld, scale,
                        None if aux2 is None else aux2.data_ptr())


class UtttB200:
    def __init__(self, state_dict: Dict[str, torch.Tensor], cfg: ModelConfig, device="cuda",
                 max_personas: int = 1, max_positions: Optional[int] = None, hsplit=None):
        """``hsplit``: a ``hsplit.HiddenSplit``; persona states and read copies are then
        this rank's slices of the hidden units and every readout sums its z across
        the group (decode and prefill; the batched write needs unsplit states)."""
        self.cfg = cfg
        self.hsplit = hsplit
        self.device = torch.device(device)
        dev = self.device
        self.lib = _lib.load()
        d, hd = cfg.d_model, cfg.head_dim
        if d % 128 != 0 or cfg.d_ff_fast % 8 != 0:
            raise ValueError("B200 kernels need d_model % 128 == 0 and d_ff_fast % 8 == 0")

        def bf(t):
            return t.detach().to(device=dev, dtype=torch.bfloat16).contiguous()

        def f32(t):
            return t.detach().to(device=dev, dtype=torch.float32).contiguous()

        sd = state_dict
        self.emb = bf(sd["tok_embeddings.weight"])
        head = sd.get("lm_head.weight")
        self.lm_head = self.emb if head is None or head is sd["tok_embeddings.weight"] else bf(head)
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"layers.{i}."
            self.layers.append(SimpleNamespace(
                attn_norm=f32(sd[p + "attn_norm.weight"]),
                wqkv=bf(torch.cat([sd[p + "attn.wq.weight"], sd[p + "attn.wk.weight"], sd[p + "attn.wv.weight"]])),
                wo=bf(sd[p + "attn.wo.weight"]),
                uttt_norm=f32(sd[p + "uttt_norm.weight"]),
                w_q=bf(sd[p + "uttt.w_q.weight"]),
                slow=bf(torch.cat([sd[p + "uttt.w_q.weight"], sd[p + "uttt.w_k.weight"], sd[p + "uttt.w_v.weight"],
                                   sd[p + "uttt.w_eta.weight"], sd[p + "uttt.w_alpha.weight"]])),
                w_o=bf(sd[p + "uttt.w_o.weight"]),
                q_norm=f32(sd[p + "uttt.q_norm.weight"]),
                k_norm=f32(sd[p + "uttt.k_norm.weight"]),
                b_eta=f32(sd[p + "uttt.w_eta.bias"]),
                b_alpha=f32(sd[p + "uttt.w_alpha.bias"]),
            ))
        self.norm = f32(sd["norm.weight"])
        self.w0 = tuple(f32(sd["fast_weight_pool." + n]) for n in ("w_up_init", "w_gate_init", "w_down_init"))
        self.ln_w = f32(sd["fast_weight_pool.ln_weight"])
        self.ln_b = f32(sd["fast_weight_pool.ln_bias"])
        # readout LayerNorm affine as the BF16 path applies it (ln.to(x.dtype), model/uttt_layer.py:253-257)
        self.ln_w_act = self.ln_w.to(torch.bfloat16).float().contiguous()
        self.ln_b_act = self.ln_b.to(torch.bfloat16).float().contiguous()
        n_pos = max_positions or (cfg.max_seq_len + 1024)
        cos, sin = rope_tables(hd, n_pos, cfg.rope_theta)
        self.rope_cos, self.rope_sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
        self.n_pos = n_pos
        self.active_limit = SIMPLE_ACTIVE_VOCAB_LIMIT if cfg.vocab_size >= 24000 else cfg.vocab_size
        self.qkv_dim = (cfg.n_heads + 2 * cfg.n_kv_heads) * hd
        self.max_personas = max_personas
        shape = (max_personas, cfg.n_kv_heads, cfg.sliding_window_size, hd)
        self.k_ring = [torch.zeros(shape, dtype=torch.bfloat16, device=dev) for _ in range(cfg.n_layers)]
        self.v_ring = [torch.zeros(shape, dtype=torch.bfloat16, device=dev) for _ in range(cfg.n_layers)]

    # ------------------------------------------------------------------ launch helpers
    def _st(self) -> int:
        return _stream(self.device)

    def _linear(self, x: torch.Tensor, w: torch.Tensor, segs: Sequence[_lib.Segment]) -> None:
        M, K = x.shape
        N = w.shape[0]
        arr = (_lib.Segment * len(segs))(*segs)
        ws = workspace(self.lib.uttt_linear_workspace(M, N), self.device, slot=2)
        _lib.check(self.lib.uttt_linear(M, N, K, x.data_ptr(), w.data_ptr(), len(segs), arr, self.cfg.rms_norm_eps,
                                        ws.data_ptr(), ws.numel(), self._st()), "uttt_linear")

    def _rmsnorm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(x)
        rows, d = x.shape
        _lib.check(self.lib.uttt_rmsnorm(rows, d, x.data_ptr(), x.stride(0), w.data_ptr(), self.cfg.rms_norm_eps,
                                         out.data_ptr(), d, self._st()), "uttt_rmsnorm")
        return out

    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        if not ids.is_cuda and ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.emb.shape[0]):
            raise ValueError("token id outside the vocabulary")       # nn.Embedding raises as well
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous().reshape(-1)
        out = torch.empty(ids.numel(), self.cfg.d_model, dtype=torch.bfloat16, device=self.device)
        _lib.check(self.lib.uttt_embed(ids.numel(), self.cfg.d_model, self.emb.shape[0], ids.data_ptr(),
                                       self.emb.data_ptr(), out.data_ptr(), self._st()), "uttt_embed")
        return out

    def _resid_linear(self, h: torch.Tensor, x: torch.Tensor, w: torch.Tensor,
                      norm: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """h += bf16(x W^T), in place (block residual adds, model/uttt_layer.py:1544-1554);
        with ``norm`` (an RMSNorm weight) also returns rms_norm(h) * norm from the same launch."""
        d = w.shape[0]
        segs = [_seg(0, d, _lib.SEG_RESID, h, h.stride(0), h, h.stride(0))]
        out = None
        if norm is not None:
            out = torch.empty(h.shape[0], d, dtype=torch.bfloat16, device=self.device)
            segs.append(_seg(0, d, _lib.SEG_NORM, out, d, h, h.stride(0), aux2=norm))
        self._linear(x, w, segs)
        return out

    def _readout(self, q: torch.Tensor, packed: torch.Tensor, down: torch.Tensor, sidx: torch.Tensor,
                 ln: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
        """Frozen readout f_W(q) of (B, T, d) BF16 queries through BF16 read copies, with the
        engine's LayerNorm affine or a state's own ``ln`` (weight, bias)."""
        if ln is None:
            lw, lb = self.ln_w_act, self.ln_b_act
        else:   # as the BF16 path applies it (ln.to(x.dtype), model/uttt_layer.py:253-257)
            lw, lb = (t.to(torch.bfloat16).float().contiguous() for t in ln)
        if self.hsplit is not None:
            return self.hsplit.readout(q, packed, down, sidx, lw, lb, self.cfg.rms_norm_eps)
        return fast_readout(q, packed, None, down, lw, lb, self.cfg.rms_norm_eps, state_index=sidx, packed=True,
                            ln_prepared=True)

    def _q_proj(self, layer, x2: torch.Tensor) -> torch.Tensor:
        """``fused_fast_q_proj`` (model/uttt_layer.py:1175-1190)."""
        d = self.cfg.d_model
        q = torch.empty(x2.shape[0], d, dtype=torch.bfloat16, device=self.device)
        self._linear(x2, layer.w_q, [_seg(0, d, _lib.SEG_RMSNORM, q, d, layer.q_norm)])
        return q

    def logits(self, h_last: torch.Tensor) -> torch.Tensor:
        """Final RMSNorm + tied lm_head (BF16 output, as under autocast), returned as FP32."""
        return self._lm_head(self._rmsnorm(h_last, self.norm))

    def _lm_head(self, x: torch.Tensor) -> torch.Tensor:
        """Tied lm_head of final-normalised rows (BF16 output), returned as FP32."""
        V = self.lm_head.shape[0]
        out = torch.empty(x.shape[0], V, dtype=torch.bfloat16, device=self.device)
        self._linear(x, self.lm_head, [_seg(0, V, _lib.SEG_STORE, out, V)])
        return out.float()

    def greedy(self, logits: torch.Tensor, stop_free: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
        """Device greedy pick; returns (ids int32 (B,), top-1/top-2 values (B, 2))."""
        B, V = logits.shape
        logits = logits.contiguous()
        ids = torch.empty(B, dtype=torch.int32, device=self.device)
        top2 = torch.empty(B, 2, dtype=torch.float32, device=self.device)
        _lib.check(self.lib.uttt_greedy_argmax(B, V, logits.data_ptr(), 1, V, self.active_limit, int(stop_free),
                                               ids.data_ptr(), top2.data_ptr(), self._st()), "uttt_greedy_argmax")
        return ids, top2

    def read_copies(self, w_up, w_gate, w_down) -> Tuple[torch.Tensor, torch.Tensor]:
        """BF16 read copies of FP32 states (S, d, h) (``inference_read_weights``)."""
        S, d, h = w_up.shape
        packed = torch.empty(S, d, 2 * h, dtype=torch.bfloat16, device=self.device)
        down = torch.empty(S, h, d, dtype=torch.bfloat16, device=self.device)
        _lib.check(self.lib.uttt_pack_read_copies(S, d, h, w_up.data_ptr(), w_gate.data_ptr(), w_down.data_ptr(),
                                                  packed.data_ptr(), down.data_ptr(), self._st()),
                   "uttt_pack_read_copies")
        return packed, down

    def init_fast_state(self, batch_size: int = 1) -> FastState:
        """``SharedFastWeightPool.init_state`` (detach=True), FP32 masters (this rank's
        hidden-unit slices when the engine splits them)."""
        w0 = self.w0 if self.hsplit is None else self.hsplit.shard(*(w.unsqueeze(0) for w in self.w0))
        rep = [w.reshape(w.shape[-2:]).unsqueeze(0).expand(batch_size, *w.shape[-2:]).contiguous() for w in w0]
        return FastState(*rep, *(torch.zeros_like(t) for t in rep), self.ln_w.clone(), self.ln_b.clone())

    # ------------------------------------------------------------------ frozen path
    def prefill(self, ids: torch.Tensor, slot: int, read_packed: torch.Tensor, read_down: torch.Tensor,
                state_index: int = 0) -> torch.Tensor:
        """Frozen forward of one persona's prompt; fills its KV ring; returns last-token logits (V,)."""
        return self._lm_head(self._prefill_hidden(ids, slot, read_packed, read_down, state_index)[-1:])[0]

    def prefill_logits(self, ids: torch.Tensor, slot: int, read_packed: torch.Tensor, read_down: torch.Tensor,
                       state_index: int = 0, keep: int = 1) -> torch.Tensor:
        """``prefill`` returning the logits of the last ``keep`` positions (0: every position),
        (keep, V) FP32 of BF16 values (``uTTTModel.forward``'s ``logits_to_keep``)."""
        x = self._prefill_hidden(ids, slot, read_packed, read_down, state_index)
        return self._lm_head(x if keep <= 0 else x[-keep:].contiguous())

    def _prefill_hidden(self, ids: torch.Tensor, slot: int, read_packed: torch.Tensor, read_down: torch.Tensor,
                        state_index: int = 0) -> torch.Tensor:
        """The prompt's final-normalised hidden rows (T, d) BF16; fills the persona's KV ring."""
        cfg = self.cfg
        ids = ids.reshape(-1)
        T = ids.numel()
        d, hd, nh, nkv = cfg.d_model, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        if T + 1 >= self.n_pos:
            raise ValueError("prompt longer than the RoPE table")
        dev = self.device
        h = self._embed(ids)
        slot_t = _host_list([slot], torch.int32, dev)
        sidx = _host_list([state_index], torch.int32, dev)
        qkv = torch.empty(T, self.qkv_dim, dtype=torch.bfloat16, device=dev)
        qs = torch.empty(T, nh * hd, dtype=torch.bfloat16, device=dev)
        kb = torch.empty(1, nkv, T, hd, dtype=torch.bfloat16, device=dev)
        vb = torch.empty_like(kb)
        att = torch.empty(T, d, dtype=torch.bfloat16, device=dev)
        x = self._rmsnorm(h, self.layers[0].attn_norm)
        L = len(self.layers)
        for i, lay in enumerate(self.layers):
            self._linear(x, lay.wqkv, [_seg(0, self.qkv_dim, _lib.SEG_STORE, qkv, self.qkv_dim)])
            _lib.check(self.lib.uttt_attn_prefill(1, T, 0, 0, nh, nkv, hd, cfg.sliding_window_size, qkv.data_ptr(),
                                                  self.qkv_dim, self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
                                                  qs.data_ptr(), kb.data_ptr(), vb.data_ptr(), att.data_ptr(),
                                                  self._st()), "uttt_attn_prefill")
            _lib.check(self.lib.uttt_kv_ring_fill(1, T, T, nkv, hd, cfg.sliding_window_size, kb.data_ptr(),
                                                  vb.data_ptr(), slot_t.data_ptr(), self.k_ring[i].data_ptr(),
                                                  self.v_ring[i].data_ptr(), self._st()), "uttt_kv_ring_fill")
            x2 = self._resid_linear(h, att, lay.wo, lay.uttt_norm)
            q = self._q_proj(lay, x2)
            r = self._readout(q.unsqueeze(0), read_packed, read_down, sidx)
            x = self._resid_linear(h, r.reshape(T, d), lay.w_o, self.layers[i + 1].attn_norm if i + 1 < L else self.norm)
        return x

    def prefill_batch(self, prompts: Sequence[torch.Tensor], slots: Sequence[int], read_packed: torch.Tensor,
                      read_down: torch.Tensor, state_index: Sequence[int]) -> torch.Tensor:
        """Frozen forward of several personas' prompts of any lengths at once; fills each persona's KV
        ring; returns the last-token logits (n, V) FP32 of BF16 values.

        The prompts are packed one after another, each padded to a multiple of 64 tokens, so every
        projection GEMM and the fast-weight readout (one 64-token tile per state row) run once per
        layer for all of them; attention and the ring fill run per prompt on its own rows.  Padding
        rows never reach a prompt's rows (causal attention, row-wise everything else)."""
        cfg = self.cfg
        n = len(prompts)
        if n == 0 or len(slots) != n or len(state_index) != n:
            raise ValueError("one slot and one state index per prompt")
        lens = [int(p.numel()) for p in prompts]
        if min(lens) < 1 or max(lens) + 1 >= self.n_pos:
            raise ValueError("prompt empty or longer than the RoPE table")
        d, hd, nh, nkv, W = cfg.d_model, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.sliding_window_size
        dev = self.device
        spans = [(T + 63) // 64 * 64 for T in lens]
        offs = [0]
        for sp in spans:
            offs.append(offs[-1] + sp)
        R = offs[-1]
        ids = torch.zeros(R, dtype=torch.long)
        tile_state = []
        for p, T, o, sp, si in zip(prompts, lens, offs, spans, state_index):
            ids[o:o + T] = p.reshape(-1).to(torch.long).cpu()
            tile_state += [int(si)] * (sp // 64)
        if int(ids.min()) < 0 or int(ids.max()) >= self.emb.shape[0]:
            raise ValueError("token id outside the vocabulary")
        h = self._embed(ids.pin_memory().to(dev, non_blocking=True))
        tiles = _host_list(tile_state, torch.int32, dev)
        slot_all = _host_list([int(s_) for s_ in slots], torch.int32, dev)
        slot_t = [slot_all[j:j + 1] for j in range(len(slots))]
        qkv = torch.empty(R, self.qkv_dim, dtype=torch.bfloat16, device=dev)
        qs = torch.empty(R, nh * hd, dtype=torch.bfloat16, device=dev)
        kv_off = [0]
        for T in lens:
            kv_off.append(kv_off[-1] + nkv * T * hd)
        kflat = torch.empty(kv_off[-1], dtype=torch.bfloat16, device=dev)
        vflat = torch.empty_like(kflat)
        att = torch.zeros(R, d, dtype=torch.bfloat16, device=dev)      # padding rows stay finite
        esz = kflat.element_size()
        x = self._rmsnorm(h, self.layers[0].attn_norm)
        L = len(self.layers)
        for i, lay in enumerate(self.layers):
            self._linear(x, lay.wqkv, [_seg(0, self.qkv_dim, _lib.SEG_STORE, qkv, self.qkv_dim)])
            for j, T in enumerate(lens):
                o = offs[j]
                kb = kflat.data_ptr() + kv_off[j] * esz
                vb = vflat.data_ptr() + kv_off[j] * esz
                _lib.check(self.lib.uttt_attn_prefill(1, T, 0, 0, nh, nkv, hd, W, qkv[o].data_ptr(), self.qkv_dim,
                                                      self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
                                                      qs[o].data_ptr(), kb, vb, att[o].data_ptr(), self._st()),
                           "uttt_attn_prefill")
                _lib.check(self.lib.uttt_kv_ring_fill(1, T, T, nkv, hd, W, kb, vb, slot_t[j].data_ptr(),
                                                      self.k_ring[i].data_ptr(), self.v_ring[i].data_ptr(),
                                                      self._st()), "uttt_kv_ring_fill")
            x2 = self._resid_linear(h, att, lay.wo, lay.uttt_norm)
            q = self._q_proj(lay, x2)
            r = self._readout(q.reshape(R // 64, 64, d), read_packed, read_down, tiles)
            x = self._resid_linear(h, r.reshape(R, d), lay.w_o, self.layers[i + 1].attn_norm if i + 1 < L else self.norm)
        last = _host_list([o + T - 1 for o, T in zip(offs, lens)], torch.long, dev)
        return self._lm_head(x.index_select(0, last).contiguous())

    # ------------------------------------------------------------------ KV rings <-> chronological caches
    def export_kv(self, slot: int, end_pos: int) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """The persona's KV history as the reference's per-layer caches: (1, n_kv, L, hd) BF16 in
        position order, L = min(end_pos, W), the keys RoPE'd (``SlidingWindowAttention.forward``,
        model/uttt_layer.py:1080-1114; ``CUDAGraphDecoder.export_kv_caches``, engine/inference.py:295-302)."""
        W = self.cfg.sliding_window_size
        n = min(end_pos, W)
        idx = torch.arange(end_pos - n, end_pos, device=self.device).remainder(W)
        return [(k[slot:slot + 1].index_select(2, idx), v[slot:slot + 1].index_select(2, idx))
                for k, v in zip(self.k_ring, self.v_ring)]

    def import_kv(self, slot: int, caches, end_pos: int) -> None:
        """Load the reference's chronological per-layer caches (positions end_pos - L .. end_pos - 1)
        into the persona's rings at slot pos % W (``CUDAGraphDecoder.reset``, engine/inference.py:205-222)."""
        W = self.cfg.sliding_window_size
        if len(caches) != len(self.k_ring):
            raise ValueError("one (key, value) cache per layer is required")
        for (k, v), kr, vr in zip(caches, self.k_ring, self.v_ring):
            n = k.shape[2]
            if n > W or n > end_pos or k.shape != v.shape or k.shape[0] != 1:
                raise ValueError("KV cache longer than the window or than its positions")
            idx = torch.arange(end_pos - n, end_pos, device=self.device).remainder(W)
            kr[slot].zero_()
            vr[slot].zero_()
            kr[slot].index_copy_(1, idx, k[0].to(device=self.device, dtype=torch.bfloat16))
            vr[slot].index_copy_(1, idx, v[0].to(device=self.device, dtype=torch.bfloat16))

    def use_state_ln(self, ln_weight: torch.Tensor, ln_bias: torch.Tensor) -> None:
        """Make a persona state's readout LayerNorm affine the one the frozen path applies (in place,
        so captured decode graphs see it), rounded as the BF16 path applies it (:253-257)."""
        self.ln_w_act.copy_(ln_weight.to(torch.bfloat16).float())
        self.ln_b_act.copy_(ln_bias.to(torch.bfloat16).float())

    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor, read_packed: torch.Tensor,
                    read_down: torch.Tensor, state_index: torch.Tensor) -> torch.Tensor:
        """One new token for each of B rows (packed multi-persona decode); returns logits (B, V) FP32."""
        cfg = self.cfg
        B = tokens.numel()
        d, hd, nh, nkv = cfg.d_model, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        dev = self.device
        pos = pos.to(device=dev, dtype=torch.int32).contiguous()
        slots = slots.to(device=dev, dtype=torch.int32).contiguous()
        sidx = state_index.to(device=dev, dtype=torch.int32).contiguous()
        h = self._embed(tokens)
        qkv = torch.empty(B, self.qkv_dim, dtype=torch.bfloat16, device=dev)
        att = torch.empty(B, d, dtype=torch.bfloat16, device=dev)
        L = len(self.layers)
        x = self._rmsnorm(h, self.layers[0].attn_norm)
        for i, lay in enumerate(self.layers):
            self._linear(x, lay.wqkv, [_seg(0, self.qkv_dim, _lib.SEG_STORE, qkv, self.qkv_dim)])
            _lib.check(self.lib.uttt_attn_decode(B, nh, nkv, hd, cfg.sliding_window_size, qkv.data_ptr(),
                                                 self.qkv_dim, pos.data_ptr(), slots.data_ptr(),
                                                 self.k_ring[i].data_ptr(), self.v_ring[i].data_ptr(),
                                                 self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), att.data_ptr(),
                                                 d, self._st()), "uttt_attn_decode")
            x2 = self._resid_linear(h, att, lay.wo, lay.uttt_norm)
            q = self._q_proj(lay, x2)
            r = self._readout(q.unsqueeze(1), read_packed, read_down, sidx)
            x = self._resid_linear(h, r.reshape(B, d), lay.w_o, self.layers[i + 1].attn_norm if i + 1 < L else self.norm)
        return self._lm_head(x)

    def generate_greedy(self, prompt: torch.Tensor, state: FastState, n_tokens: int, slot: int = 0,
                        stop_free: bool = True, eos_token_id: Optional[int] = None
                        ) -> Tuple[List[int], List[float], List[torch.Tensor]]:
        """``stream_generate`` at temperature 0 for one persona (stop-free greedy by default;
        otherwise the reference's stops: role ids end the reply unyielded, EOS is yielded last,
        model/uttt_model.py:1036-1050)."""
        packed, down = self.read_copies(state.w_up, state.w_gate, state.w_down)
        logits = self.prefill(prompt, slot, packed, down, 0).unsqueeze(0)
        pos = prompt.numel()
        ids, margins, all_logits = [], [], []
        zero = torch.zeros(1, dtype=torch.int32, device=self.device)
        slot_t = torch.full((1,), slot, dtype=torch.int32, device=self.device)
        for _ in range(n_tokens):
            all_logits.append(logits[0])
            tok, top2 = self.greedy(logits, stop_free)
            t = int(tok.item())
            if not stop_free and t in (USER_ID, ASSISTANT_ID):
                break
            ids.append(t)
            tv = top2[0].tolist()
            margins.append(tv[0] - tv[1])
            if len(ids) == n_tokens or (not stop_free and eos_token_id is not None and t == eos_token_id):
                break
            logits = self.decode_step(tok, torch.full((1,), pos, dtype=torch.int32, device=self.device), slot_t,
                                      packed, down, zero)
            pos += 1
        return ids, margins, all_logits

    def teacher_forced_logits(self, prompt: torch.Tensor, forced: Sequence[int], state: FastState,
                              slot: int = 0) -> List[torch.Tensor]:
        packed, down = self.read_copies(state.w_up, state.w_gate, state.w_down)
        out = [self.prefill(prompt, slot, packed, down, 0)]
        pos = prompt.numel()
        zero = torch.zeros(1, dtype=torch.int32, device=self.device)
        slot_t = torch.full((1,), slot, dtype=torch.int32, device=self.device)
        for tok in list(forced)[:-1]:
            lg = self.decode_step(torch.tensor([tok], dtype=torch.int32, device=self.device),
                                  torch.full((1,), pos, dtype=torch.int32, device=self.device), slot_t, packed, down,
                                  zero)
            out.append(lg[0])
            pos += 1
        return out

    # ------------------------------------------------------------------ write path
    def test_time_update(self, interaction_ids: torch.Tensor, fast_state: FastState,
                         attention_mask: Optional[torch.Tensor] = None) -> Tuple[FastState, float, List[float]]:
        """``uTTTModel.test_time_update`` (model/uttt_model.py:1237-1271) for one persona."""
        new, surprises, per_layer = self.test_time_update_batch(interaction_ids.reshape(1, -1), fast_state,
                                                                None if attention_mask is None
                                                                else attention_mask.reshape(1, -1))
        return new, surprises[0], per_layer[0]

    def test_time_update_batch(self, interaction_ids: torch.Tensor, fast_state: FastState,
                               attention_mask: Optional[torch.Tensor] = None, return_logits: bool = False,
                               guard: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor, float]] = None):
        """The write of B personas at once: rows of ``interaction_ids`` (B, T) with
        masks; ``fast_state`` holds B stacked states.  Every chunk of every layer is
        one packed launch sequence over the rows still in the batch: a row leaves
        it once no valid token is left (its state is final, since a chunk without
        valid tokens keeps W and S exactly, model/uttt_layer.py:513-520), so a
        ragged batch costs what its rows' own lengths cost.
        Returns (new stacked state, per-row mean surprise, per-row per-layer surprise), and with
        ``return_logits`` also the logits (B, T, V) FP32 of every position as the writing forward
        reads them (every row then stays in the batch to its end, padding included).
        Per-row statistics follow the reference's single-persona definitions
        (model/uttt_model.py:598-607, 833-838).
        ``guard`` = (w_up0, w_gate0, w_down0, anchor_lambda): the elastic pull of the stability guard
        (``apply_elastic_pull``, model/uttt_layer.py:773-832) runs inside each row's last update, and
        the per-row sums ||W_m - W0_m||^2 of the pulled state (B, 4) FP32 come back as the last output.
        A row whose turn is gated off is simply not committed, so the pull can always run."""
        cfg = self.cfg
        dev = self.device
        ids = interaction_ids if interaction_ids.is_cuda else interaction_ids.pin_memory()
        ids = ids.to(device=dev, non_blocking=True)
        B, T = ids.shape
        C, W = cfg.chunk_size, cfg.sliding_window_size
        d, hd, nh, nkv = cfg.d_model, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        L = cfg.n_layers
        if C > 64:
            raise ValueError("chunk_size > 64 is not supported by the B200 write kernels")
        if fast_state.w_up.shape[0] != B:
            raise ValueError(f"fast_state holds {fast_state.w_up.shape[0]} states for {B} rows")
        if guard is not None and self.hsplit is not None:
            raise ValueError("the guarded write needs whole (unsplit) states")
        cur = fast_state.clone()
        if attention_mask is None:
            mask_all, last = None, [T - 1] * B
        else:
            m_host = attention_mask.reshape(B, T).to(dtype=torch.float32).cpu()
            pos_idx = torch.arange(T).expand(B, T)
            last = torch.where(m_host != 0, pos_idx, torch.full_like(pos_idx, -1)).max(dim=1).values.tolist()
            mask_all = m_host.contiguous().pin_memory().to(device=dev, non_blocking=True)
        h_all = self._embed(ids).reshape(B, T, d)
        hist_k: List[Optional[torch.Tensor]] = [None] * L
        hist_v: List[Optional[torch.Tensor]] = [None] * L
        alive = list(range(B))
        rows = torch.arange(B, dtype=torch.int32, device=dev)
        chunk_losses, counts = [], []
        final = torch.empty(B, T, d, dtype=torch.bfloat16, device=dev) if return_logits else None
        drift = torch.zeros(B, 4, dtype=torch.float32, device=dev) if guard is not None else None
        for off in range(0, T, C):
            Cc = min(C, T - off)
            keep_rows = list(alive) if return_logits else [r for r in alive if last[r] >= off]
            if not keep_rows:
                cur.step += L                      # the reference still steps through padded chunks
                continue
            if len(keep_rows) < len(alive):        # compact: rows with nothing left leave the batch
                sel = _host_list([alive.index(r) for r in keep_rows], torch.long, dev)
                for i in range(L):
                    if hist_k[i] is not None:
                        hist_k[i] = hist_k[i].index_select(0, sel)
                        hist_v[i] = hist_v[i].index_select(0, sel)
                alive = keep_rows
                rows = _host_list(alive, torch.int32, dev)
            Bc = len(alive)
            R = Bc * Cc
            rows_l = rows.long()
            rp, rd = self.read_copies(cur.w_up, cur.w_gate, cur.w_down)      # chunk-start snapshot
            hidden = h_all[rows_l, off:off + Cc].reshape(R, d).contiguous()
            m = None if mask_all is None else mask_all[rows_l, off:off + Cc].contiguous()
            # Every layer reads the chunk-start snapshot, so the slow forward of all L
            # layers runs first and produces each layer's write inputs (layer-major) ...
            K = torch.empty(L, R, d, dtype=torch.bfloat16, device=dev)
            V = torch.empty_like(K)
            ETA = torch.empty(L, R, dtype=torch.float32, device=dev)
            ALPHA = torch.empty_like(ETA)
            x = self._rmsnorm(hidden, self.layers[0].attn_norm)
            for i, lay in enumerate(self.layers):
                qkv = torch.empty(R, self.qkv_dim, dtype=torch.bfloat16, device=dev)
                self._linear(x, lay.wqkv, [_seg(0, self.qkv_dim, _lib.SEG_STORE, qkv, self.qkv_dim)])
                hist = 0 if hist_k[i] is None else hist_k[i].shape[2]
                kb = torch.empty(Bc, nkv, hist + Cc, hd, dtype=torch.bfloat16, device=dev)
                vb = torch.empty_like(kb)
                if hist:
                    kb[:, :, :hist].copy_(hist_k[i])
                    vb[:, :, :hist].copy_(hist_v[i])
                qs = torch.empty(R, nh * hd, dtype=torch.bfloat16, device=dev)
                att = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
                _lib.check(self.lib.uttt_attn_prefill(Bc, Cc, off, hist, nh, nkv, hd, W, qkv.data_ptr(), self.qkv_dim,
                                                      self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
                                                      qs.data_ptr(), kb.data_ptr(), vb.data_ptr(), att.data_ptr(),
                                                      self._st()), "uttt_attn_prefill")
                keep = min(W - 1, hist + Cc)
                hist_k[i] = kb[:, :, hist + Cc - keep:].contiguous()
                hist_v[i] = vb[:, :, hist + Cc - keep:].contiguous()
                hh = hidden.clone()
                x2 = self._resid_linear(hh, att, lay.wo, lay.uttt_norm)
                q = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
                self._linear(x2, lay.slow, [                       # fused_slow_projections, :1193-1231
                    _seg(0, d, _lib.SEG_RMSNORM, q, d, lay.q_norm),
                    _seg(d, d, _lib.SEG_RMSNORM, K[i], d, lay.k_norm),
                    _seg(2 * d, d, _lib.SEG_RMSNORM, V[i], d),
                    _seg(3 * d, 1, _lib.SEG_SIGMOID, ETA[i], 1, lay.b_eta, 0, cfg.base_inner_lr, out_f32=True),
                    _seg(3 * d + 1, 1, _lib.SEG_SIGMOID, ALPHA[i], 1, lay.b_alpha, 0, cfg.base_weight_decay,
                         out_f32=True),
                ])
                out = self._readout(q.reshape(Bc, Cc, d), rp, rd, rows, (cur.ln_weight, cur.ln_bias))
                if i + 1 < L:
                    x = self._resid_linear(hh, out.reshape(R, d), lay.w_o, self.layers[i + 1].attn_norm)
                else:
                    normed = self._resid_linear(hh, out.reshape(R, d), lay.w_o,
                                                self.norm if final is not None else None)
                    if final is not None:
                        final[rows_l, off:off + Cc] = normed.reshape(Bc, Cc, d)
                hidden = hh
            # ... then the L writes chain through the state as ONE call whose chunks are the
            # layers (row b's tokens: layer 0's chunk, layer 1's chunk, ...), so every write
            # after the first reuses the previous one's freshly updated tiles for its forward.
            Kr = K.reshape(L, Bc, Cc, d).permute(1, 0, 2, 3).reshape(Bc, L * Cc, d).contiguous()
            Vr = V.reshape(L, Bc, Cc, d).permute(1, 0, 2, 3).reshape(Bc, L * Cc, d).contiguous()
            Er = ETA.reshape(L, Bc, Cc).permute(1, 0, 2).reshape(Bc, L * Cc).contiguous()
            Ar = ALPHA.reshape(L, Bc, Cc).permute(1, 0, 2).reshape(Bc, L * Cc).contiguous()
            Mr = None if m is None else m.repeat(1, L).contiguous()
            loss = torch.empty(Bc, L * Cc, dtype=torch.float32, device=dev)
            g = None
            if guard is not None:
                # the rows whose last valid token is in this chunk take their final update here
                fin = _host_list([1 if off <= last[r] < off + Cc else 0 for r in alive], torch.int32, dev)
                sums = torch.zeros(Bc, 4, dtype=torch.float32, device=dev)
                g = (*guard, fin, sums)
            chunk_write(Kr, Vr, Er, Ar, cur.w_up, cur.w_gate, cur.w_down, cur.s_up, cur.s_gate, cur.s_down,
                        cur.ln_weight, cur.ln_bias, Mr, cfg.momentum_beta, float(cfg.max_inner_grad_norm or 0.0),
                        cfg.normalize_loss_by_dim, cfg.rms_norm_eps, chunk_size=Cc, token_loss=loss,
                        state_rows=rows, partial_sum=None if self.hsplit is None else self.hsplit.all_reduce,
                        guard=g)
            if g is not None:
                drift.index_add_(0, rows_l, sums)
            lz = loss.reshape(Bc, L, Cc)
            if m is None:
                layer_loss = lz.mean(dim=2)                                        # (Bc, L)
            else:
                layer_loss = (lz * m[:, None, :]).sum(dim=2) / m.sum(dim=1, keepdim=True).clamp_min(1.0)
            chunk_loss = torch.zeros(B, L, dtype=torch.float32, device=dev)
            chunk_loss[rows_l] = layer_loss                                     # (B, L), zero off the batch
            count = torch.zeros(B, dtype=torch.float32, device=dev)
            count[rows_l] = m.sum(dim=1) if m is not None else float(Cc)
            chunk_losses.append(chunk_loss)
            counts.append(count)
            cur.step += L
        check_status(workspace(0, dev), "test_time_update")
        if not chunk_losses:
            per_layer = [[0.0] * L for _ in range(B)]
        else:
            cnt = torch.stack(counts, dim=1).to(torch.float64)                      # (B, n_chunks)
            losses = torch.stack(chunk_losses, dim=1).to(torch.float64)            # (B, n_chunks, L)
            per_layer_t = (losses * cnt[:, :, None]).sum(1) / cnt.sum(1, keepdim=True).clamp_min(1.0)
            per_layer = [[float(x) for x in row] for row in per_layer_t.float().tolist()]   # single sync
        means = [sum(r) / max(len(r), 1) for r in per_layer]
        cur.last_surprise_loss = means[0] if B == 1 else float(sum(means) / B)
        cur.surprise_history = (list(fast_state.surprise_history) + (per_layer[0] if B == 1 else []))[-100:]
        out = (cur, means, per_layer)
        if final is not None:
            out += (self._lm_head(final.reshape(B * T, d)).reshape(B, T, -1),)
        if drift is not None:
            out += (drift,)
        return out


class DecodeTable:
    """The rows of a packed decode batch, resident in device memory (the descriptor arrays of
    ``uttt_engine_step`` / ``uttt_engine_admit``): next token, position, KV slot, fast-weight state,
    reply length, limits, status and a ring of the last ``ENGINE_RING`` reply tokens per row.

    The captured decode step advances the rows on the device after its greedy pick
    (``advance``), so steps run back to back without the host.  The host starts a row with
    ``admit`` (after the turn's prefill) and reads the rows back asynchronously with
    ``snapshot`` / ``read``, one step behind, to stream tokens and retire finished turns.
    Idle and finished rows are padding rows: KV slot ``pad_slot``, state -1."""

    def __init__(self, device: torch.device, rows: int, pad_slot: int, stop_free: bool):
        self.device = device
        self.rows = rows
        self.pad_slot = int(pad_slot)
        self.stop_free = bool(stop_free)
        i32 = dict(dtype=torch.int32, device=device)
        self.tokens = torch.zeros(rows, **i32)
        self.pos = torch.zeros(rows, **i32)
        self.slots = torch.full((rows,), self.pad_slot, **i32)
        self.state = torch.full((rows,), -1, **i32)
        self.produced = torch.zeros(rows, **i32)
        self.max_new = torch.ones(rows, **i32)
        self.eos = torch.full((rows,), -1, **i32)
        self.status = torch.full((rows,), _lib.ROW_IDLE, **i32)
        self.ring = torch.zeros(rows, _lib.ENGINE_RING, **i32)
        self.lib = _lib.load()
        # two pinned host copies of (produced, status, ring), written alternately
        self._host = [(torch.empty(rows, dtype=torch.int32).pin_memory(),
                       torch.empty(rows, dtype=torch.int32).pin_memory(),
                       torch.empty(rows, _lib.ENGINE_RING, dtype=torch.int32).pin_memory()) for _ in range(2)]
        self._ready = [torch.cuda.Event(), torch.cuda.Event()]

    def _ptrs(self):
        return (self.tokens.data_ptr(), self.pos.data_ptr(), self.slots.data_ptr(), self.state.data_ptr(),
                self.produced.data_ptr(), self.max_new.data_ptr(), self.eos.data_ptr(), self.status.data_ptr(),
                self.ring.data_ptr())

    def advance(self, ids: torch.Tensor, n: int) -> None:
        """Apply the stop rules to rows 0..n-1 after a step's greedy pick ``ids`` (device int32)."""
        _lib.check(self.lib.uttt_engine_step(n, ids.data_ptr(), *self._ptrs(), int(self.stop_free), self.pad_slot,
                                             _stream(self.device)), "uttt_engine_step")

    def admit(self, row: int, first_id: torch.Tensor, pos: int, slot: int, state: int, max_new: int,
              eos: Optional[int]) -> None:
        """Start ``row`` for a turn whose prefill picked ``first_id`` (device int32, one element)."""
        if not 0 <= row < self.rows:
            raise ValueError("row outside the table")
        _lib.check(self.lib.uttt_engine_admit(row, first_id.data_ptr(), int(pos), int(slot), int(state),
                                              int(max_new), -1 if eos is None else int(eos), *self._ptrs(),
                                              int(self.stop_free), self.pad_slot, _stream(self.device)),
                   "uttt_engine_admit")

    def snapshot(self, k: int) -> None:
        """Queue copies of (produced, status, ring) into host buffer ``k`` (0 or 1) on the current stream."""
        hp, hs, hr = self._host[k]
        hp.copy_(self.produced, non_blocking=True)
        hs.copy_(self.status, non_blocking=True)
        hr.copy_(self.ring, non_blocking=True)
        self._ready[k].record(torch.cuda.current_stream(self.device))

    def read(self, k: int):
        """Wait for snapshot ``k`` and return (produced, status, ring) as host tensors."""
        self._ready[k].synchronize()
        return self._host[k]


class DecodeGraph:
    """A packed decode step (+ greedy pick) captured once in a CUDA graph.

    The B200 counterpart of ``CUDAGraphDecoder`` (``engine/inference.py:71-302``)
    for a packed batch: static device buffers hold each row's token, position,
    KV slot and fast-weight state index; ``step`` copies the new inputs in,
    replays, and returns (greedy ids, logits) from static outputs that stay
    valid until the next replay.  The read copies and KV rings it captured
    must stay allocated.
    """

    def __init__(self, engine: "UtttB200", batch: int, read_packed: torch.Tensor, read_down: torch.Tensor,
                 stop_free: bool = True, pad_slot: Optional[int] = None, table: Optional["DecodeTable"] = None):
        """``table``: the rows live in a device-resident ``DecodeTable`` (its first ``batch`` rows) and the
        captured step ends with ``uttt_engine_step``, which advances them on the device: ``step()`` then
        takes no inputs.  The table's rows must be idle (padding) while the graph is captured."""
        self.engine = engine
        dev = engine.device
        self.batch = batch
        self.table = table
        if table is not None:
            self.tokens, self.pos = table.tokens[:batch], table.pos[:batch]
            self.slots, self.sidx = table.slots[:batch], table.state[:batch]
        else:
            self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
            self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
            if pad_slot is None:
                if batch > min(engine.max_personas, read_packed.shape[0]):
                    raise ValueError("batch exceeds the persona slots; pass pad_slot")
                self.slots = torch.arange(batch, dtype=torch.int32, device=dev)
            else:
                self.slots = torch.full((batch,), pad_slot, dtype=torch.int32, device=dev)
            self.sidx = self.slots.clone()
        self.read_packed, self.read_down = read_packed, read_down
        self.stop_free = stop_free
        # warm up (workspaces, kernel attributes) on a side stream, then capture;
        # the warm-up writes ring slot 0 of every row's persona, which the
        # caller's next step overwrites before any read (positions start >= 0).
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self.logits, self.ids, self.top2 = self._body()
        torch.cuda.synchronize(dev)

    def _body(self):
        lg = self.engine.decode_step(self.tokens, self.pos, self.slots, self.read_packed, self.read_down, self.sidx)
        ids, top2 = self.engine.greedy(lg, self.stop_free)
        if self.table is not None:
            self.table.advance(ids, self.batch)
        return lg, ids, top2

    def step(self, tokens: Optional[torch.Tensor] = None, pos: Optional[torch.Tensor] = None,
             slots: Optional[torch.Tensor] = None, state_index: Optional[torch.Tensor] = None):
        """Replay with new row inputs (or, with a ``table``, with the rows the device holds)."""
        if self.table is not None:
            self.graph.replay()
            return self.ids, self.logits
        self.tokens.copy_(tokens, non_blocking=True)
        self.pos.copy_(pos, non_blocking=True)
        if slots is not None:
            self.slots.copy_(slots, non_blocking=True)
        if state_index is not None:
            self.sidx.copy_(state_index, non_blocking=True)
        self.graph.replay()
        return self.ids, self.logits

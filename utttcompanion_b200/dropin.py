"""Model- and personalizer-level drop-ins: the reference's Python surface above the kernels.

Three faces of the same B200 engine, each keeping the reference's names, signatures, return
types and error classes (``ValueError`` for bad arguments, ``RuntimeError`` for device
failures):

* ``uTTTModelB200`` -- ``uTTTModel``'s serving surface (``model/uttt_model.py``):
  ``forward`` (:714-729), ``stream_generate`` (:966-979, an iterator of token ids),
  ``test_time_update`` (:1237-1271), ``init_fast_state`` and ``_sample_next_token``
  (:1181-1235), run entirely on the sm_100a kernels.
* ``CUDAGraphDecoder`` -- the protocol the reference's ``stream_generate`` imports lazily from
  ``engine.inference`` (``engine/inference.py:71-302``: ``is_supported``, the constructor,
  ``matches``, ``reset``, ``step``, ``export_kv_caches``).  ``install(inference_module=...)``
  swaps it in, so the reference's own generation loop decodes through a captured B200 step.
* ``uTTTPersonalizerB200`` -- ``interact_and_evolve`` / ``stream_interact_and_evolve``
  (``engine/personalizer.py:369-595``) returning ``EvolutionResult`` (:44-66), over the
  continuous-batching ``ServingEngine``.

``install(uttt_layer_module, inference_module)`` is the reference's own plug-in mechanism
(``setattr`` on its modules, ``engine/personalizer.py:221-233``) applied to the operator
drop-ins of ``pool.DROP_INS`` and to the decoder.
"""

from __future__ import annotations

import math
import os
import weakref
from dataclasses import asdict, dataclass, field
from typing import Any, Callable, Dict, Generator, Iterator, List, Optional, Sequence, Tuple

import torch

from .model import ASSISTANT_ID, BOS_ID, EOS_ID, PAD_ID, UNK_ID, USER_ID, DecodeGraph, FastState, UtttB200
from .workloads import ModelConfig


# ------------------------------------------------------------------------------------------------
# configuration and state adapters
# ------------------------------------------------------------------------------------------------
def config_from(config) -> ModelConfig:
    """``ModelConfig`` from the reference's ``uTTTConfig`` (a dataclass), a dict or a ModelConfig."""
    if isinstance(config, ModelConfig):
        return config
    if isinstance(config, dict):
        return ModelConfig.from_dict(config)
    fields = ModelConfig.__dataclass_fields__
    return ModelConfig(**{k: getattr(config, k) for k in fields if hasattr(config, k)})


def as_fast_state(state, device) -> FastState:
    """A ``FastState`` (FP32 masters on ``device``) from the reference's ``FastWeightState`` or a
    ``FastState``; tensors already FP32 on the device are used as they are."""
    if isinstance(state, FastState):
        return state

    def f32(t):
        return t.detach().to(device=device, dtype=torch.float32).contiguous()
    return FastState(*(f32(getattr(state, n)) for n in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down",
                                                        "ln_weight", "ln_bias")),
                     int(getattr(state, "step", 0)), float(getattr(state, "last_surprise_loss", 0.0)),
                     list(getattr(state, "surprise_history", [])))


@dataclass
class uTTTModelOutput:
    """Same fields as the reference's ``uTTTModelOutput`` (``model/uttt_model.py:114-123``)."""
    logits: torch.Tensor
    fast_state: Optional[FastState]
    loss: Optional[torch.Tensor] = None
    ce_loss: Optional[torch.Tensor] = None
    surprise_loss: Optional[torch.Tensor] = None
    layer_surprise_losses: List[float] = field(default_factory=list)
    kv_caches: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None


def sample_next_token(logits: torch.Tensor, temperature: float = 0.7, top_p: float = 0.9,
                      recent_tokens: Optional[List[int]] = None, repetition_penalty: float = 1.18,
                      active_vocab_limit: Optional[int] = None,
                      generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """``uTTTModel._sample_next_token`` (``model/uttt_model.py:1181-1235``): PAD/BOS/UNK and ids at
    or above the active limit are excluded, recent ids are penalised, then greedy at
    temperature <= 1e-5, else nucleus sampling (the smallest set of most probable ids whose
    probability reaches ``top_p``, renormalised) with the given generator."""
    if not math.isfinite(temperature) or temperature < 0:
        raise ValueError("temperature must be finite and nonnegative")
    if not math.isfinite(top_p) or not 0 < top_p <= 1:
        raise ValueError("top_p must be finite and in (0, 1]")
    if not math.isfinite(repetition_penalty):
        raise ValueError("repetition_penalty must be finite")
    if logits.ndim != 2 or logits.shape[-1] <= UNK_ID:
        raise ValueError("Sampling logits must have batch and vocabulary dimensions")
    if active_vocab_limit is not None and active_vocab_limit <= EOS_ID:
        raise ValueError("Active vocabulary must include EOS")
    scores = logits.to(dtype=torch.float32, copy=True)
    scores[:, [PAD_ID, BOS_ID, UNK_ID]] = -torch.inf
    if active_vocab_limit is not None and active_vocab_limit < scores.shape[-1]:
        scores[:, active_vocab_limit:] = -torch.inf
    if recent_tokens and repetition_penalty > 1.0:
        ids = torch.tensor(sorted(set(recent_tokens[-48:])), dtype=torch.long, device=scores.device)
        picked = scores[:, ids]
        scores[:, ids] = torch.where(picked < 0, picked * repetition_penalty, picked / repetition_penalty)
    if temperature <= 1e-5:
        return torch.argmax(scores, dim=-1)
    probs = torch.softmax(scores / temperature, dim=-1)
    if top_p < 1.0:
        p_sorted, order = torch.sort(probs, dim=-1, descending=True)
        before = torch.cumsum(p_sorted, dim=-1) - p_sorted        # mass of the ids ranked above each id
        p_sorted = torch.where(before > top_p, torch.zeros_like(p_sorted), p_sorted)
        p_sorted = p_sorted / p_sorted.sum(dim=-1, keepdim=True).clamp_min(1e-8)
        choice = torch.multinomial(p_sorted, 1, generator=generator)
        return order.gather(-1, choice).squeeze(-1)
    return torch.multinomial(probs, 1, generator=generator).squeeze(-1)


# ------------------------------------------------------------------------------------------------
# uTTTModel surface
# ------------------------------------------------------------------------------------------------
class uTTTModelB200:
    """``uTTTModel``'s serving surface on the B200 engine (module docstring).

    Persona slots 0 .. ``max_personas`` - 1 of the engine's KV rings hold the rows of a call;
    weights are BF16 copies of the given state dict (reference parameter names), fast-weight
    W_0 and LayerNorm FP32.  Outer-loop training (``labels``) is not part of the serving path
    and is rejected with ``ValueError``."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], config, device="cuda", max_personas: int = 1,
                 active_vocab_limit: Optional[int] = None):
        self.config = config_from(config)
        self.engine = UtttB200(state_dict, self.config, device=device, max_personas=max_personas)
        self.device = self.engine.device
        self.active_vocab_limit = int(active_vocab_limit or self.engine.active_limit)
        self.engine.active_limit = self.active_vocab_limit
        self.repetition_penalty = float(getattr(config, "repetition_penalty", 1.0))
        self._graph: Optional[DecodeGraph] = None
        self._graph_key = None

    @classmethod
    def from_reference(cls, model, device=None, max_personas: int = 1) -> "uTTTModelB200":
        """Build from a reference ``uTTTModel`` instance (its weights, config and vocabulary limit)."""
        dev = device or next(model.parameters()).device
        out = cls({k: v.detach() for k, v in model.state_dict().items()}, model.config, device=dev,
                  max_personas=max_personas, active_vocab_limit=getattr(model, "active_vocab_limit", None))
        out.repetition_penalty = float(getattr(model.config, "repetition_penalty", 1.0))
        return out

    # -------------------------------------------------------------------------------- state
    def init_fast_state(self, batch_size: int = 1, device=None, dtype: torch.dtype = torch.float32,
                        detach: bool = True) -> FastState:
        """``uTTTModel.init_fast_state``: W_0 repeated over the batch, zero momentum (FP32 masters;
        the kernels keep FP32 state whatever ``dtype`` asks)."""
        if batch_size < 1:
            raise ValueError("batch_size must be positive")
        return self.engine.init_fast_state(batch_size)

    def _reads(self, st: FastState) -> Tuple[torch.Tensor, torch.Tensor]:
        self.engine.use_state_ln(st.ln_weight[0] if st.ln_weight.dim() > 1 else st.ln_weight,
                                 st.ln_bias[0] if st.ln_bias.dim() > 1 else st.ln_bias)
        return self.engine.read_copies(st.w_up, st.w_gate, st.w_down)

    # -------------------------------------------------------------------------------- forward
    def forward(self, input_ids: torch.Tensor, fast_state=None, labels: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                kv_caches: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None, start_pos: int = 0,
                update_fast_weights: bool = True, surprise_aux_weight: float = 0.10, logits_to_keep: int = 0,
                return_fast_state: bool = True, ce_reduction: str = "token_mean",
                ce_token_indices: Optional[torch.Tensor] = None,
                detach_returned_fast_state: bool = True) -> uTTTModelOutput:
        """``uTTTModel.forward`` (``model/uttt_model.py:714-960``) for the serving path: the frozen
        read (prefill, or continuation from ``kv_caches`` at ``start_pos``) and the writing forward
        (chunk-first schedule over every layer).  ``logits_to_keep``: 0 every position, k > 0 the
        last k, -1 none (as ``test_time_update`` asks)."""
        if type(detach_returned_fast_state) is not bool:
            raise ValueError("detach_returned_fast_state must be boolean")
        if ce_reduction not in ("token_mean", "sequence_mean"):
            raise ValueError("ce_reduction must be token_mean or sequence_mean")
        if labels is not None or ce_token_indices is not None:
            raise ValueError("outer-loop training (labels / CE) is not part of the B200 serving path")
        if input_ids.dim() != 2 or input_ids.shape[1] == 0:
            raise ValueError("input_ids must be a non-empty (B, T) tensor")
        B, T = input_ids.shape
        V = self.config.vocab_size
        eng = self.engine
        if B > eng.max_personas:
            raise ValueError(f"batch {B} exceeds the engine's {eng.max_personas} persona slots")
        st = self.init_fast_state(B) if fast_state is None else as_fast_state(fast_state, self.device)
        if st.w_up.shape[0] == 1 and B > 1:
            st = FastState(*(t.expand(B, *t.shape[1:]).contiguous() for t in
                             (st.w_up, st.w_gate, st.w_down, st.s_up, st.s_gate, st.s_down)),
                           st.ln_weight, st.ln_bias, st.step, st.last_surprise_loss, list(st.surprise_history))
        if st.w_up.shape[0] != B:
            raise ValueError(f"fast_state holds {st.w_up.shape[0]} states for batch {B}")
        if update_fast_weights:
            if kv_caches is not None or start_pos != 0:
                raise ValueError("the B200 writing forward starts a turn: kv_caches must be None and start_pos 0")
            want = logits_to_keep != -1
            res = eng.test_time_update_batch(input_ids, st, attention_mask, return_logits=want)
            new, means, per_layer = res[:3]
            if attention_mask is None:
                n_valid = [float(T)] * B
            else:
                n_valid = attention_mask.reshape(B, T).float().sum(dim=1).tolist()
            tot = max(sum(n_valid), 1.0)
            layer = [sum(per_layer[b][i] * n_valid[b] for b in range(B)) / tot for i in range(self.config.n_layers)]
            if want:
                logits = (res[3] if logits_to_keep == 0 else res[3][:, -logits_to_keep:]).to(torch.bfloat16)
            else:
                logits = torch.empty(B, 0, V, device=self.device)
            surprise = torch.tensor(sum(layer) / max(len(layer), 1), device=self.device)
            return uTTTModelOutput(logits, new if return_fast_state else None, surprise_loss=surprise,
                                   layer_surprise_losses=layer)
        # frozen read
        packed, down = self._reads(st)
        rows, caches_out = [], []
        for b in range(B):
            ids = input_ids[b]
            if kv_caches is None and start_pos == 0:
                lg = eng.prefill_logits(ids, b, packed, down, b, keep=max(logits_to_keep, 0) if logits_to_keep >= 0
                                        else 1)
                if logits_to_keep < 0:
                    lg = lg[:0]
            else:
                if kv_caches is None:
                    raise ValueError("start_pos > 0 needs the kv_caches of the earlier positions")
                eng.import_kv(b, [(k[b:b + 1], v[b:b + 1]) for k, v in kv_caches], start_pos)
                outs = []
                sidx = torch.tensor([b], dtype=torch.int32, device=self.device)
                for t in range(T):
                    outs.append(eng.decode_step(ids[t:t + 1].to(self.device),
                                                torch.tensor([start_pos + t], dtype=torch.int32,
                                                             device=self.device), sidx, packed, down, sidx))
                lg = torch.cat(outs)
                if logits_to_keep > 0:
                    lg = lg[-logits_to_keep:]
                elif logits_to_keep < 0:
                    lg = lg[:0]
            rows.append(lg)
            caches_out.append(eng.export_kv(b, start_pos + T))
        logits = torch.stack(rows)
        kv = [(torch.cat([c[i][0] for c in caches_out]), torch.cat([c[i][1] for c in caches_out]))
              for i in range(self.config.n_layers)]
        return uTTTModelOutput(logits.to(torch.bfloat16), st if return_fast_state else None,
                               surprise_loss=torch.zeros((), device=self.device),
                               layer_surprise_losses=[0.0] * self.config.n_layers, kv_caches=kv)

    __call__ = forward

    # -------------------------------------------------------------------------------- write
    @torch.no_grad()
    def test_time_update(self, interaction_ids: torch.Tensor, fast_state,
                         attention_mask: Optional[torch.Tensor] = None) -> Tuple[FastState, float, List[float]]:
        """``uTTTModel.test_time_update`` (``model/uttt_model.py:1237-1271``): a new state (the input
        is not modified), the mean surprise and the per-layer surprises."""
        ids = interaction_ids.reshape(1, -1) if interaction_ids.dim() == 1 else interaction_ids
        out = self.forward(ids, fast_state=as_fast_state(fast_state, self.device).clone(),
                           attention_mask=attention_mask, update_fast_weights=True, logits_to_keep=-1)
        st = out.fast_state
        st.last_surprise_loss = float(sum(out.layer_surprise_losses) / max(len(out.layer_surprise_losses), 1))
        return st, st.last_surprise_loss, out.layer_surprise_losses

    # -------------------------------------------------------------------------------- generate
    _sample_next_token = staticmethod(sample_next_token)

    @torch.no_grad()
    def stream_generate(self, input_ids: torch.Tensor, fast_state, max_new_tokens: int = 128,
                        temperature: float = 0.7, top_p: float = 0.9, eos_token_id: Optional[int] = EOS_ID,
                        speculative_draft_k: Optional[int] = None, dspark_conf_threshold: Optional[float] = None,
                        use_cuda_graph: bool = False, generator: Optional[torch.Generator] = None) -> Iterator[int]:
        """``uTTTModel.stream_generate`` (``model/uttt_model.py:966-1179``): prefill with the frozen
        persona, then one token at a time; role ids end the reply unyielded, EOS is yielded last.
        Each decode step runs on the B200 kernels (captured in a CUDA graph with ``use_cuda_graph``).
        Self-speculative drafting is not part of the path: ``speculative_draft_k`` must be 0 or None."""
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens must be nonnegative")
        if max_new_tokens == 0:
            return
        if input_ids.ndim != 2 or input_ids.shape[0] != 1 or input_ids.shape[1] == 0:
            raise ValueError("Streaming generation requires one non-empty prompt")
        if speculative_draft_k:
            raise ValueError("self-speculative drafting is not part of the B200 serving path")
        eng = self.engine
        st = as_fast_state(fast_state, self.device)
        packed, down = self._reads(st)
        logits = eng.prefill(input_ids[0], 0, packed, down, 0).unsqueeze(0)
        pos = input_ids.shape[1]
        zero = torch.zeros(1, dtype=torch.int32, device=self.device)
        graph = None
        if use_cuda_graph:
            key = (packed.data_ptr(), down.data_ptr())
            if self._graph is None or self._graph_key != key:
                self._graph = DecodeGraph(eng, 1, packed, down)
                self._graph_key = key
            graph = self._graph
        recent: List[int] = []
        produced = 0
        while produced < max_new_tokens:
            tok = self._sample_next_token(logits, temperature=temperature, top_p=top_p, recent_tokens=recent,
                                          active_vocab_limit=self.active_vocab_limit,
                                          repetition_penalty=self.repetition_penalty, generator=generator)
            tid = int(tok.item())
            if tid in (USER_ID, ASSISTANT_ID):
                break
            recent.append(tid)
            yield tid
            produced += 1
            if (eos_token_id is not None and tid == eos_token_id) or produced >= max_new_tokens:
                break
            t32 = tok.to(torch.int32).reshape(1)
            p32 = torch.full((1,), pos, dtype=torch.int32, device=self.device)
            if graph is not None:
                _, logits = graph.step(t32, p32)
            else:
                logits = eng.decode_step(t32, p32, zero, packed, down, zero)
            pos += 1


# ------------------------------------------------------------------------------------------------
# CUDAGraphDecoder protocol
# ------------------------------------------------------------------------------------------------
def _tensor_key(t: torch.Tensor):
    return (id(t), t.data_ptr(), t._version, t.dtype, t.device, tuple(t.shape))


_ENGINES: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()


class CUDAGraphDecoder:
    """Drop-in for ``engine.inference.CUDAGraphDecoder`` (``engine/inference.py:71-302``).

    Frozen batch-1 decode of a reference ``uTTTModel`` through the B200 engine: one captured
    packed step (embedding, projections, ring attention, fast-weight readout, LM head) per
    token, KV history in the engine's ring (slot = position mod window).  The engine (BF16
    copies of the model's weights) is built once per model and rebuilt when any parameter
    changes; the persona's BF16 read copies are made from ``fast_state`` at construction.
    ``step`` returns logits (1, V) in the model's dtype from a static buffer that stays valid
    until the next step.  Callers serialise access and ``reset`` at every turn, as with the
    reference's decoder."""

    _FAST_NAMES = ("w_up", "w_gate", "w_down", "ln_weight", "ln_bias")

    @staticmethod
    def _state_key(state):
        return tuple(_tensor_key(getattr(state, n)) for n in CUDAGraphDecoder._FAST_NAMES)

    @staticmethod
    def _model_key(model):
        return (model.training, tuple(_tensor_key(p) for p in model.parameters()))

    @classmethod
    def is_supported(cls, model, fast_state, prefill_kv_caches, start_pos) -> bool:
        """The reference's conditions (frozen CUDA FP16/BF16 weights, FP32 fast-weight pool allowed,
        batch one, caches of min(start_pos, W) positions) plus the kernels' shape limits."""
        if model.training or torch.is_inference_mode_enabled() or not isinstance(start_pos, int) or start_pos < 1:
            return False
        named = list(model.named_parameters())
        if not named:
            return False
        first = named[0][1]
        if first.device.type != "cuda" or first.dtype not in (torch.float16, torch.bfloat16):
            return False
        if any(p.requires_grad or p.device != first.device
               or (p.dtype != first.dtype and not (n.startswith("fast_weight_pool.") and p.dtype == torch.float32))
               for n, p in named):
            return False
        cfg = config_from(model.config)
        if cfg.d_model % 128 or cfg.d_ff_fast % 8 or cfg.head_dim not in (32, 64, 128) \
                or cfg.n_heads % cfg.n_kv_heads or cfg.n_heads // cfg.n_kv_heads > 8 \
                or cfg.sliding_window_size > 1024:
            return False
        if prefill_kv_caches is None or len(prefill_kv_caches) != cfg.n_layers:
            return False
        want = (1, cfg.n_kv_heads, min(start_pos, cfg.sliding_window_size), cfg.head_dim)
        if any(tuple(t.shape) != want or t.device != first.device for pair in prefill_kv_caches for t in pair):
            return False
        for n in cls._FAST_NAMES:
            t = getattr(fast_state, n)
            if t.device != first.device or t.dtype not in (first.dtype, torch.float32) or t.requires_grad:
                return False
        return fast_state.w_up.shape[0] == 1 and fast_state.w_down.shape[0] == 1

    @staticmethod
    def _engine_for(model) -> UtttB200:
        key = CUDAGraphDecoder._model_key(model)
        hit = _ENGINES.get(model)
        if hit is not None and hit[0] == key:
            return hit[1]
        dev = next(model.parameters()).device
        eng = UtttB200({k: v.detach() for k, v in model.state_dict().items()}, config_from(model.config),
                       device=dev, max_personas=1,
                       max_positions=max(int(getattr(model.config, "max_seq_len", 4096)) + 1024, 2048))
        eng.active_limit = int(getattr(model, "active_vocab_limit", eng.active_limit))
        _ENGINES[model] = (key, eng)
        return eng

    @torch.no_grad()
    def __init__(self, model, fast_state, prefill_kv_caches, start_pos):
        if not self.is_supported(model, fast_state, prefill_kv_caches, start_pos):
            raise ValueError("CUDA graph decode requires frozen CUDA FP16/BF16 weights, batch one and supported "
                             "KV caches")
        self.model = model
        self.fast_state = fast_state
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        self.engine = self._engine_for(model)
        masters = [getattr(fast_state, n).detach().to(torch.float32).contiguous() for n in ("w_up", "w_gate",
                                                                                            "w_down")]
        self._packed, self._down = self.engine.read_copies(*masters)
        self.engine.use_state_ln(fast_state.ln_weight.detach().reshape(-1), fast_state.ln_bias.detach().reshape(-1))
        self._captured_model_key = self._model_key(model)
        self._captured_state_key = self._state_key(fast_state)
        self._position_limit = self.engine.n_pos - 1
        self._token = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._pos = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.reset(prefill_kv_caches, start_pos)
        self._graph = DecodeGraph(self.engine, 1, self._packed, self._down)
        self.reset(prefill_kv_caches, start_pos)      # the capture's warm-up wrote ring slot 0

    def matches(self, model, fast_state) -> bool:
        """Validate a cached decoder at a turn boundary (identity and version of the weights)."""
        return (model is self.model and fast_state is self.fast_state
                and self._captured_state_key == self._state_key(fast_state)
                and self._captured_model_key == self._model_key(model))

    @torch.no_grad()
    def reset(self, prefill_kv_caches, start_pos) -> None:
        if not self.matches(self.model, self.fast_state):
            raise ValueError("Model or persona weights changed; create a new CUDA graph decoder")
        if not self.is_supported(self.model, self.fast_state, prefill_kv_caches, start_pos):
            raise ValueError("Unsupported prefill state or RoPE position for CUDA graph decode")
        self.engine.use_state_ln(self.fast_state.ln_weight.detach().reshape(-1),
                                 self.fast_state.ln_bias.detach().reshape(-1))
        self.engine.import_kv(0, prefill_kv_caches, start_pos)
        self.next_position = start_pos

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor) -> torch.Tensor:
        if self.model.training or self._captured_state_key != self._state_key(self.fast_state):
            raise ValueError("Persona weights changed during graph decoding")
        if self.next_position >= self._position_limit:
            raise ValueError("CUDA graph reached its captured RoPE table limit")
        if tuple(input_ids.shape) != (1, 1) or input_ids.device != self.device or input_ids.dtype != torch.long:
            raise ValueError("CUDA graph input must be a CUDA int64 tensor of shape (1, 1)")
        self._token.copy_(input_ids.reshape(1))
        self._pos.fill_(self.next_position)
        _, logits = self._graph.step(self._token, self._pos)
        self.next_position += 1
        return logits.to(self.dtype)

    @torch.no_grad()
    def export_kv_caches(self) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """Chronological KV history for a mid-turn eager fallback."""
        return [(k.to(self.dtype), v.to(self.dtype)) for k, v in self.engine.export_kv(0, self.next_position)]


def install(uttt_layer_module=None, inference_module=None) -> Dict[str, object]:
    """Swap the B200 drop-ins into the reference's modules with ``setattr`` (its own plug-in
    mechanism): the operator functions of ``pool.DROP_INS`` into ``model.uttt_layer`` and this
    ``CUDAGraphDecoder`` into ``engine.inference``.  Returns the replaced originals, keyed
    ``"uttt_layer.<name>"`` / ``"inference.CUDAGraphDecoder"``."""
    from . import pool
    replaced: Dict[str, object] = {}
    if uttt_layer_module is not None:
        replaced.update({"uttt_layer." + k: v for k, v in pool.install(uttt_layer_module).items()})
    if inference_module is not None:
        if hasattr(inference_module, "CUDAGraphDecoder"):
            replaced["inference.CUDAGraphDecoder"] = inference_module.CUDAGraphDecoder
        inference_module.CUDAGraphDecoder = CUDAGraphDecoder
    return replaced


def uninstall(replaced: Dict[str, object], uttt_layer_module=None, inference_module=None) -> None:
    """Put back what ``install`` replaced."""
    for key, fn in replaced.items():
        mod, name = key.split(".", 1)
        target = uttt_layer_module if mod == "uttt_layer" else inference_module
        if target is not None:
            setattr(target, name, fn)


# ------------------------------------------------------------------------------------------------
# personalizer surface
# ------------------------------------------------------------------------------------------------
@dataclass
class EvolutionResult:
    """Same fields as the reference's ``EvolutionResult`` (``engine/personalizer.py:44-66``), plus
    the turn's token ids."""
    user_id: str
    prompt: Any
    reply: str
    surprise_loss: float
    surprise_threshold: float
    gate_triggered: bool
    weight_drift_frobenius: float
    weight_drift_pct: float
    persona_saved: bool
    persona_path: str
    step: int
    status_bar: str
    layer_surprise_losses: List[float] = field(default_factory=list)
    is_command: bool = False
    command_name: Optional[str] = None
    drift_details: Optional[Dict[str, Any]] = None
    seed: Optional[int] = None
    prompt_ids: List[int] = field(default_factory=list)
    reply_ids: List[int] = field(default_factory=list)

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


def status_bar(surprise_loss: float, weight_drift_pct: float, persona_saved: bool, gate_triggered: bool) -> str:
    """One-line TTT status for a turn (the information of ``format_ttt_status_bar``,
    ``engine/personalizer.py:69-82``)."""
    state = "updated" if gate_triggered else "gated off"
    saved = "saved" if persona_saved else "not saved"
    return (f"[TTT Status] Surprise: {surprise_loss:.4f} | Fast weights {state} | "
            f"Drift: {weight_drift_pct:.3f}% | Persona {saved}")


class uTTTPersonalizerB200:
    """``uTTTPersonalizer``'s turn API over the continuous-batching ``ServingEngine``.

    ``prompt`` is text when a ``tokenizer`` is given (an object with the reference tokenizer's
    ``encode(text, add_bos, add_eos, max_length)`` / ``decode(ids, skip_special_tokens)`` and
    ``EOS_ID`` / ``PAD_ID``) together with ``encode_prompt(tokenizer, prompt, max_len, history)``
    (the reference's ``engine.prompting.encode_chat_prompt``); the turn is then written on the
    reference's re-tokenised ``<|user|> ... <|assistant|> ...`` text (``personalizer.py:480-489``).
    Without a tokenizer ``prompt`` is a list of token ids and the write runs on prompt + reply ids.
    Decoding is greedy (the north star's contract): ``temperature`` must be 0 or None.
    With ``persona_dir`` every gated write is saved in the reference's persona-file format."""

    def __init__(self, serving, tokenizer=None, encode_prompt: Optional[Callable] = None,
                 persona_dir: Optional[str] = None, auto_save_every_turn: bool = True,
                 default_max_new_tokens: int = 128):
        self.serving = serving
        self.tokenizer = tokenizer
        self.encode_prompt = encode_prompt
        self.persona_dir = persona_dir
        self.auto_save_every_turn = auto_save_every_turn
        self.default_max_new_tokens = default_max_new_tokens
        self.surprise_threshold = serving.surprise_threshold
        if tokenizer is not None and encode_prompt is None:
            raise ValueError("a text tokenizer needs encode_prompt (the chat-template encoder)")

    def _ids(self, prompt, max_tokens: int, history) -> Tuple[List[int], Optional[Callable]]:
        cfg = self.serving.engine.cfg
        if self.tokenizer is None:
            if isinstance(prompt, str) or not len(prompt):
                raise ValueError("without a tokenizer the prompt must be a non-empty list of token ids")
            return [int(x) for x in prompt], None
        if not isinstance(prompt, str) or not prompt.strip():
            raise ValueError("Prompt must not be blank")
        ids = list(self.encode_prompt(self.tokenizer, prompt, cfg.max_seq_len - max_tokens, history=history))
        tok = self.tokenizer

        def write_ids(prompt_ids, reply_ids):
            reply = tok.decode(list(reply_ids), skip_special_tokens=True).strip() or "[Acknowledged]"
            text = f"<|user|> {prompt.strip()}\n<|assistant|> {reply}"
            return tok.encode(text, add_bos=True, add_eos=True, max_length=cfg.max_seq_len)
        return ids, write_ids

    def _check(self, max_new_tokens, temperature, top_p, seed) -> int:
        cfg = self.serving.engine.cfg
        max_tokens = self.default_max_new_tokens if max_new_tokens is None else max_new_tokens
        if type(max_tokens) is not int or not 1 <= max_tokens < cfg.max_seq_len:
            raise ValueError(f"max_new_tokens must be between 1 and {cfg.max_seq_len - 1}")
        if temperature is not None and (not math.isfinite(temperature) or temperature > 1e-5 or temperature < 0):
            raise ValueError("the B200 serving path decodes greedily: temperature must be 0")
        if top_p is not None and (not math.isfinite(top_p) or not 0.0 < top_p <= 1.0):
            raise ValueError("top_p must be finite and in (0, 1]")
        if seed is not None and (type(seed) is not int or not 0 <= seed < 2 ** 63):
            raise ValueError("seed must be an integer between 0 and 2**63 - 1")
        return max_tokens

    def _result(self, user_id, prompt, seed, raw: dict) -> EvolutionResult:
        saved, path = False, ""
        if self.persona_dir is not None:
            path = os.path.join(self.persona_dir, f"{user_id}_state.pt")
            if raw["gate_triggered"] and self.auto_save_every_turn:
                self.serving.arena.save_user(user_id, self.persona_dir)
                saved = True
        reply_ids = list(raw["reply_ids"])
        if self.tokenizer is not None:
            reply = self.tokenizer.decode(reply_ids, skip_special_tokens=True).strip() or "[Acknowledged]"
        else:
            reply = " ".join(str(i) for i in reply_ids)
        s = float(raw["surprise_loss"]) if raw["surprise_loss"] is not None else 0.0
        return EvolutionResult(
            user_id=user_id, prompt=prompt, reply=reply, surprise_loss=s,
            surprise_threshold=float(raw["surprise_threshold"]), gate_triggered=bool(raw["gate_triggered"]),
            weight_drift_frobenius=float(raw["weight_drift_frobenius"]),
            weight_drift_pct=float(raw["weight_drift_pct"]), persona_saved=saved, persona_path=path,
            step=int(raw["step"]), status_bar=status_bar(s, float(raw["weight_drift_pct"]), saved,
                                                          bool(raw["gate_triggered"])),
            layer_surprise_losses=[float(x) for x in raw["layer_surprise_losses"]],
            drift_details=raw["drift_details"], seed=seed, prompt_ids=list(raw["prompt_ids"]), reply_ids=reply_ids)

    def stream_interact_and_evolve(self, user_id: str, prompt, max_new_tokens: Optional[int] = None,
                                   temperature: Optional[float] = None, top_p: Optional[float] = None,
                                   seed: Optional[int] = None, history: Optional[List[Dict[str, str]]] = None
                                   ) -> Generator[Dict[str, Any], None, EvolutionResult]:
        """Yields ``{"type": "token", "content": ..., "token_id": ...}`` per reply token as it is
        decoded, then ``{"type": "ttt_status", "result": ...}``; returns the ``EvolutionResult``."""
        max_tokens = self._check(max_new_tokens, temperature, top_p, seed)
        ids, write_ids = self._ids(prompt, max_tokens, history)
        events: List[dict] = []
        t = self.serving.submit(user_id, ids, max_tokens, eos_token_id=EOS_ID, on_event=events.append,
                                write_ids=write_ids)
        emitted: List[int] = []
        text_len = 0
        while True:
            while events:
                ev = events.pop(0)
                if ev["type"] == "token":
                    emitted.append(ev["token_id"])
                    piece = str(ev["token_id"])
                    if self.tokenizer is not None:
                        full = self.tokenizer.decode(emitted, skip_special_tokens=True)
                        piece, text_len = full[text_len:], len(full)
                    yield {"type": "token", "content": piece, "token_id": ev["token_id"]}
                else:
                    result = self._result(user_id, prompt, seed, ev["result"])
                    yield {"type": "ttt_status", "result": result.to_dict()}
                    return result
            if t.done and not events:
                result = self._result(user_id, prompt, seed, t.result)
                yield {"type": "ttt_status", "result": result.to_dict()}
                return result
            self.serving.step()

    def interact_and_evolve(self, user_id: str, prompt, max_new_tokens: Optional[int] = None,
                            temperature: Optional[float] = None, top_p: Optional[float] = None,
                            seed: Optional[int] = None,
                            history: Optional[List[Dict[str, str]]] = None) -> EvolutionResult:
        """One full turn: decode with the frozen persona, chunk-TTT write of the turn, surprise gate,
        elastic pull + drift clamp, commit (``engine/personalizer.py:586-595``)."""
        gen = self.stream_interact_and_evolve(user_id, prompt, max_new_tokens, temperature, top_p, seed, history)
        while True:
            try:
                next(gen)
            except StopIteration as stop:
                return stop.value

"""HF transformers integration: ``patch_aoh_model`` over the CUDA runtime.

Counterpart of the reference's ``patch_aoh_model`` / ``make_aoh_forward``
(eval/efficiency/benchmark_llama31.py:187-275, benchmark_qwen.py:196-292):
every decoder layer's attention forward is replaced by one that projects
q/k/v, applies Qwen3's QK-norm when the module has one and the rotary
embedding (benchmark_qwen.py:216-226) -- for bf16 caches in one kernel
(``rope_qk``), otherwise with the model's own torch functions --, runs the
head-mixed attention (``aoh_attention``: retrieval heads over every cached token,
streaming heads over sink + window, then the append) and ``o_proj``.

Differences kept on purpose: the library is label-driven, so the attention
weights are not permuted into retrieval-first order (reorder_weights.py:19-60)
and the output is already in original head order; ``make_cache`` takes the
paged cache's sizing (batch, max_context, dtype, device) as keyword arguments;
``backend="flash"`` is the reference's decoding-simulation protocol
(attention_utils.py:45-89) on this library's kernels, not on FlashAttention-2:
the prompt in one forward with every head causal over it, then decode steps.

    make_cache, n_ret, n_str = patch_aoh_model(model, labels, 128, 256)
    cache = make_cache(max_context=65536)
    logits = model(input_ids=chunk, past_key_values=cache, use_cache=True).logits
"""
from __future__ import annotations

import sys
import types

import numpy as np
import torch

from .attention import aoh_attention, rope_qk
from .cache import AoHKVCache

try:  # the Cache base class the model's forward expects (the reference subclasses it too)
    from transformers.cache_utils import Cache
    try:
        from transformers.cache_utils import DynamicLayer
    except ImportError:  # older transformers without per-layer cache objects
        DynamicLayer = None
except ImportError:  # transformers absent: the adapter is unavailable, the runtime is not
    Cache = object
    DynamicLayer = None


class AoHModelCache(Cache):
    """The paged cache as a transformers ``Cache``, with the reference's hooks
    (benchmark_llama31.py:155-166): ``update`` is a no-op (the patched forward
    appends), sequence length and mask sizes come from ``kv_seq_len``."""

    def __init__(self, paged: AoHKVCache):
        if Cache is object:
            raise ImportError("transformers is required for the HF cache adapter")
        if DynamicLayer is None:
            super().__init__()
        else:
            super().__init__(layers=[DynamicLayer() for _ in range(paged.num_layers)])
        self.paged = paged

    @property
    def kv_seq_len(self) -> int:
        return self.paged.kv_seq_len

    @kv_seq_len.setter
    def kv_seq_len(self, n: int) -> None:
        self.paged.kv_seq_len = n

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None, **kwargs):
        return key_states, value_states

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.paged.kv_seq_len

    def get_max_cache_shape(self):
        return None

    def get_mask_sizes(self, cache_position, layer_idx: int = 0):
        # newer transformers pass the query length, older ones cache_position
        if cache_position is None:
            q_len = 1
        elif isinstance(cache_position, int):
            q_len = cache_position
        else:
            q_len = int(cache_position.numel())
        return self.paged.kv_seq_len + q_len, 0


def make_aoh_forward(layer_idx: int, num_q: int, num_kv: int, head_dim: int):
    """The patched attention forward of one layer (same signature as the
    reference's, benchmark_llama31.py:191-192); other caches fall through to
    the module's original forward."""

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None,
                cache_position=None, **kwargs):
        if not isinstance(past_key_values, AoHModelCache):
            return self._orig_forward(hidden_states=hidden_states, position_embeddings=position_embeddings,
                                      attention_mask=attention_mask, past_key_values=past_key_values,
                                      cache_position=cache_position, **kwargs)
        bsz, q_len, _ = hidden_states.shape
        cache = past_key_values.paged
        dt = cache.dtype
        q = self.q_proj(hidden_states).view(bsz, q_len, num_q, head_dim)
        k = self.k_proj(hidden_states).view(bsz, q_len, num_kv, head_dim)
        v = self.v_proj(hidden_states).view(bsz, q_len, num_kv, head_dim)
        qn, kn = getattr(self, "q_norm", None), getattr(self, "k_norm", None)
        if (position_embeddings is not None and dt == torch.bfloat16 and q.dtype == torch.bfloat16
                and head_dim == 128):
            # QK-norm (Qwen3) and RoPE in one kernel, straight into the layout the attention takes
            cos, sin = position_embeddings
            q, k = rope_qk(q.contiguous(), k.contiguous(), cos.to(torch.bfloat16).contiguous(),
                           sin.to(torch.bfloat16).contiguous(), None if qn is None else qn.weight,
                           None if kn is None else kn.weight, getattr(qn, "variance_epsilon", 1e-6))
        else:
            q, k = q.transpose(1, 2), k.transpose(1, 2)
            if qn is not None:
                q = qn(q)
            if kn is not None:
                k = kn(k)
            if position_embeddings is not None:
                cos, sin = position_embeddings
                rope = getattr(sys.modules[type(self).__module__], "apply_rotary_pos_emb")  # the model's own RoPE
                q, k = rope(q, k, cos, sin)
            q = q.transpose(1, 2).to(dt).contiguous()
            k = k.transpose(1, 2).to(dt).contiguous()
        v = v.to(dt).contiguous()
        out = aoh_attention(cache, layer_idx, q, k, v)  # attend, append, advance after the last layer
        out = out.reshape(bsz, q_len, num_q * head_dim).to(hidden_states.dtype)
        return self.o_proj(out), None

    return forward


def patch_aoh_model(model, labels: np.ndarray, sink_size: int, recent_size: int):
    """Patch every decoder layer of a Llama / Qwen2 / Qwen3 HF model; returns
    ``(make_cache, n_ret, n_str)`` like the reference (benchmark_llama31.py:
    256-275).  ``make_cache(backend="eager", *, batch=1, max_context=None,
    dtype=None, device=None)`` builds the paged cache (default: the model's
    max_position_embeddings, dtype and device); backend is "eager" or "flash"."""
    if sink_size < 0 or recent_size < 0:
        raise ValueError("sink_size and recent_size must be non-negative")
    cfg = model.config
    layers = model.model.layers
    num_q = cfg.num_attention_heads
    num_kv = cfg.num_key_value_heads
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // num_q
    labels = np.asarray(labels, dtype=np.float64)
    if labels.shape != (len(layers), num_kv):
        raise ValueError(f"head labels shape {labels.shape} != {(len(layers), num_kv)}")
    n_ret, n_str = [], []
    for i, layer in enumerate(layers):
        attn = layer.self_attn
        if not hasattr(attn, "_orig_forward"):
            attn._orig_forward = attn.forward
        attn.forward = types.MethodType(make_aoh_forward(i, num_q, num_kv, head_dim), attn)
        nr = int((labels[i] >= 0.5).sum())
        n_ret.append(nr)
        n_str.append(num_kv - nr)

    def make_cache(backend: str = "eager", *, batch: int = 1, max_context: int | None = None, dtype=None,
                   device=None) -> AoHModelCache:
        p = next(model.parameters())
        paged = AoHKVCache(labels, num_q, batch=batch, sink_size=sink_size, recent_size=recent_size,
                           max_context=int(max_context or cfg.max_position_embeddings),
                           dtype=dtype or p.dtype, device=device or p.device, head_dim=head_dim,
                           backend=backend)
        return AoHModelCache(paged)

    return make_cache, n_ret, n_str


class ModelDecodeGraph:
    """One decode step of a patched model -- every layer's projections,
    QK-norm/RoPE, head-mixed attention and MLP, and the logits -- captured once
    as a CUDA graph and replayed per token.

    The reference decodes with eager Python over the layers
    (eval/efficiency/benchmark_llama31.py:319-338); on the GPU that is mostly
    launch overhead.  Captured here: the attention reads the cache's
    device-resident length (``AoHKVCache.device_length``), a final kernel
    advances it (the reference's ``kv_seq_len += 1``, :249-250), and the token
    and its position are fixed tensors written before each replay.  Pages for
    ``max_steps`` tokens are reserved up front.  ``step(token_ids)`` returns the
    step's logits (B, 1, vocab) -- a tensor the next step overwrites.
    """

    def __init__(self, model, cache: AoHModelCache, max_steps: int):
        import ctypes as C

        from . import _lib

        paged = cache.paged
        if paged.dtype != torch.bfloat16:
            raise ValueError("a captured decode step needs a bfloat16 cache")
        if paged.backend != "eager" and paged.kv_seq_len == 0:
            raise ValueError("prefill the prompt before capturing decode steps")
        self.model, self.cache, self.paged = model, cache, paged
        dev = paged.device
        B = paged.batch
        self.ids = torch.zeros((B, 1), dtype=torch.long, device=dev)
        self.pos = torch.zeros((B, 1), dtype=torch.long, device=dev)
        self.cpos = torch.zeros((1,), dtype=torch.long, device=dev)
        paged.reserve(paged.kv_seq_len + max_steps + 1)
        self._L, self._C = paged._L, C
        self._set_length(paged.kv_seq_len)
        self._inputs(torch.zeros((B, 1), dtype=torch.long, device=dev))
        paged.device_length = True
        try:
            # the first launches configure kernels and workspaces (not capturable):
            # one eager step at the current length as a dry run -- attend, no
            # append (an append at this position would already overwrite a
            # streaming head's ring slot whose row the first replay still attends)
            _lib.check(self._L.aoh_kv_set_decode_append(paged._h, 0), "aoh_kv_set_decode_append")
            try:
                with torch.no_grad():
                    self._forward()
            finally:
                _lib.check(self._L.aoh_kv_set_decode_append(paged._h, 1), "aoh_kv_set_decode_append")
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.no_grad(), torch.cuda.graph(self.graph):
                self.logits = self._forward()
                _lib.check(self._L.aoh_kv_advance(paged._h, 1, C.c_void_p(_lib.stream_handle())), "aoh_kv_advance")
        finally:
            paged.device_length = False
        self._set_length(paged.kv_seq_len)  # capture does not execute: the device length is the host's again

    def _set_length(self, n: int) -> None:
        from . import _lib

        _lib.check(self._L.aoh_kv_set_length(self.paged._h, n, self._C.c_void_p(_lib.stream_handle())),
                   "aoh_kv_set_length")

    def _inputs(self, token_ids: torch.Tensor) -> None:
        t = self.paged.kv_seq_len
        self.ids.copy_(token_ids.view(self.ids.shape), non_blocking=True)
        self.pos.fill_(t)
        self.cpos.fill_(t)

    def _forward(self) -> torch.Tensor:
        return self.model(input_ids=self.ids, position_ids=self.pos, cache_position=self.cpos,
                          past_key_values=self.cache, use_cache=True).logits

    def step(self, token_ids: torch.Tensor) -> torch.Tensor:
        """Decode one token per sequence (token_ids: (B,) or (B, 1)) and advance."""
        self._inputs(token_ids)
        self.graph.replay()
        self.paged.kv_seq_len += 1
        return self.logits

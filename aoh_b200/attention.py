"""Per-layer head-mixed attention op over the paged cache.

``aoh_attention(cache, layer_idx, q, k, v)`` is the attention core of the
reference's patched forward (make_aoh_forward, eval/efficiency/
benchmark_llama31.py:218-250 and benchmark_qwen.py:235-267), from post-RoPE
q/k/v to the attention output, in ORIGINAL head order:

* retrieval KV heads (label 1) -> ``eager_attention`` over every cached key
  plus this call's keys, causal when q_len > 1 (:123-132);
* streaming KV heads (label 0) -> ``streaming_attention`` over the sink +
  recent window (attention_utils.py:92-119);
* then ``AoHKVCache.append_layer`` (:171-184), and ``kv_seq_len += q_len``
  after the last layer (:249-250).

q_len == 1 runs the split-KV decode kernel; longer chunks run the prefill
kernel.  Both are CUDA kernels in libaoh.so; there is no other path.  A cache
made with ``backend="flash"`` follows the reference's decoding-simulation
protocol (attention_utils.py:45-89): its prompt goes in one call over the empty
cache, every head attending causally to all of it, then decode steps as above.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .cache import AoHKVCache, _check_kv


def _check_q(cache: AoHKVCache, q: torch.Tensor, q_len: int) -> None:
    want = (cache.batch, q_len, cache.num_q_heads, cache.head_dim)
    if tuple(q.shape) != want:
        raise ValueError(f"q must have shape (batch, q_len, num_q_heads, head_dim) = {want}, got {tuple(q.shape)}")
    if q.dtype != cache.dtype or q.device != cache.device or not q.is_contiguous():
        raise ValueError("q must be a contiguous tensor of the cache's dtype on the cache's device")


def aoh_attention(cache: AoHKVCache, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  out: torch.Tensor | None = None, advance: bool = True) -> torch.Tensor:
    """Attend (retrieval: full, streaming: sink + window), then append k/v.

    q (B, C, Hq, D), k/v (B, C, G, D): contiguous, post-RoPE, original head
    order, dtype = cache dtype.  Returns (B, C, Hq, D).  With ``advance`` the
    cache's ``kv_seq_len`` moves by C after the last layer, as the reference
    does.
    """
    if not 0 <= layer_idx < cache.num_layers:
        raise ValueError(f"layer_idx {layer_idx} out of range")
    q_len = k.shape[1]
    _check_kv(cache, k, v)
    _check_q(cache, q, q_len)
    if out is None:
        out = torch.empty_like(q)
    if cache.device_length:
        # a captured decode step: the kernel reads the device-resident length,
        # whose pages were reserved when the capture was set up
        if q_len != 1:
            raise ValueError("a cache in device-length mode takes decode steps (q_len 1) only")
        past = _lib.PAST_LEN_DEVICE
    else:
        past = cache.kv_seq_len
        cache.reserve(past + q_len)
    L = cache._L
    st = C.c_void_p(_lib.stream_handle())
    if q_len == 1:
        ws = cache.decode_workspace()
        rc = L.aoh_attn_decode(cache._h, layer_idx, past, C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                               C.c_void_p(v.data_ptr()), C.c_void_p(out.data_ptr()),
                               C.c_void_p(ws.data_ptr()), ws.numel(), st)
        _lib.check(rc, "aoh_attn_decode")
    else:
        # the decoding-simulation protocol prefills the prompt in one call with
        # every head causal over it (attention_utils.py:45-89); a later
        # multi-token call of that protocol raises NotImplementedError
        fn = L.aoh_attn_prefill_flash if cache.backend == "flash" else L.aoh_attn_prefill
        rc = fn(cache._h, layer_idx, past, q_len, C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                C.c_void_p(v.data_ptr()), C.c_void_p(out.data_ptr()), st)
        _lib.check(rc, "aoh_attn_prefill_flash" if cache.backend == "flash" else "aoh_attn_prefill")
    if advance and layer_idx == cache.num_layers - 1 and not cache.device_length:
        cache.kv_seq_len += q_len
    return out


def rope_qk(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
            q_norm_weight: torch.Tensor | None = None, k_norm_weight: torch.Tensor | None = None,
            eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """q_norm / k_norm (when weights are given) and the rotate-half RoPE of the
    patched forward (benchmark_qwen.py:216-226) in one kernel.

    q (B, C, Hq, D), k (B, C, G, D): bf16, contiguous (the projections'
    views); cos / sin (B, C, D) bf16 from the model's rotary embedding.
    Returns contiguous (q, k) ready for :func:`aoh_attention`."""
    for name, t in (("q", q), ("k", k), ("cos", cos), ("sin", sin)):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or not t.is_cuda:
            raise ValueError(f"{name} must be a contiguous bfloat16 CUDA tensor")
    B, n, Hq, D = q.shape
    G = k.shape[2]
    if tuple(k.shape) != (B, n, G, D) or tuple(cos.shape) != (B, n, D) or tuple(sin.shape) != (B, n, D):
        raise ValueError("q (B, C, Hq, D), k (B, C, G, D) and cos / sin (B, C, D) must agree")
    if (q_norm_weight is None) != (k_norm_weight is None):
        raise ValueError("give both norm weights or neither")
    ws = []
    for w in (q_norm_weight, k_norm_weight):
        if w is not None:
            w = w.to(torch.bfloat16).contiguous()
            if tuple(w.shape) != (D,):
                raise ValueError(f"norm weights must be ({D},)")
        ws.append(w)
    q_out, k_out = torch.empty_like(q), torch.empty_like(k)
    ptr = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    _lib.check(_lib.lib().aoh_rope_qk(ptr(q), ptr(k), ptr(cos), ptr(sin), ptr(ws[0]), ptr(ws[1]), float(eps), B, n,
                                      Hq, G, D, ptr(q_out), ptr(k_out), C.c_void_p(_lib.stream_handle())),
               "aoh_rope_qk")
    return q_out, k_out

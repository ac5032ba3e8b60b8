"""A decode step through every layer, captured once as a CUDA graph.

The reference runs decode as an eager Python loop over layers
(eval/efficiency/benchmark_llama31.py:319-338); each layer's attention here is
one kernel launch, so on the host side a step is only launch overhead.
``DecodeStepGraph`` captures the whole step -- one decode kernel per layer,
then one tiny kernel that advances the device-resident sequence length (the
reference's ``kv_seq_len += q_len`` after the last layer, :249-250) -- and
replays it.  Consecutive layer kernels are launched with programmatic
dependent launch, so a layer's page streaming starts while the previous
layer's kernel finishes.

Inputs and outputs are the fixed tensors given at construction; write a
step's q/k/v into them before ``replay()`` (or let producing kernels do so).

With a ``PeerGather`` (multi-GPU, one process per GPU) each layer's decode
kernel also stores its units' outputs into every rank's output region, and
the graph waits for all ranks' units after each layer (the layer boundary).
With ``overlap_gather=True`` each layer's wait runs on a second stream
instead, beside the next layers' decode kernels, and the step ends after all
of them: for a step whose layers do not consume one another's attention
output (q, k, v of every layer given up front, as in an attention-only
benchmark), the ranks then meet once per step instead of once per layer.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .cache import AoHKVCache


class DecodeStepGraph:
    """Decode step over ``layers`` of ``cache`` as one CUDA graph.

    q: (L, B, 1, Hq, D), k/v: (L, B, 1, G, D), out: (L, B, 1, Hq, D) -- bf16,
    contiguous, on the cache's device, L = number of layers in the step.
    ``max_steps``: replays this graph will be used for (pages are reserved
    for all of them up front; the graph itself never allocates).
    """

    def __init__(self, cache: AoHKVCache, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 out: torch.Tensor, max_steps: int, layers=None, gather=None, overlap_gather: bool = False):
        if cache.dtype != torch.bfloat16:
            raise ValueError("graph decode needs a bfloat16 cache")
        self.cache = cache
        self.layers = list(range(cache.num_layers)) if layers is None else list(layers)
        if q.shape[0] != len(self.layers):
            raise ValueError("q/k/v/out must have one leading entry per captured layer")
        for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
            if not t.is_contiguous() or t.dtype != torch.bfloat16 or t.device != cache.device:
                raise ValueError(f"{name} must be a contiguous bf16 tensor on {cache.device}")
        self.q, self.k, self.v, self.out = q, k, v, out
        self.gather = gather
        self.overlap_gather = bool(overlap_gather) and gather is not None
        self._side = torch.cuda.Stream(device=cache.device) if self.overlap_gather else None
        cache.reserve(cache.kv_seq_len + max_steps + 1)
        self._L = cache._L
        self._ws = cache.decode_workspace()
        self._set_length(cache.kv_seq_len)
        # the first launch configures kernel attributes (not capturable): run the
        # step once eagerly as a dry run -- attend, no append (an append at the
        # current position would already overwrite a streaming head's ring slot
        # whose row the first replay, at the same position, still attends).
        # A gather is detached meanwhile: the eager step must publish no flags
        # the first replay (same position) would then find already set.
        if gather is not None:
            gather.detach()
        _lib.check(self._L.aoh_kv_set_decode_append(cache._h, 0), "aoh_kv_set_decode_append")
        try:
            self._launch_layers(with_gather=False)
        finally:
            _lib.check(self._L.aoh_kv_set_decode_append(cache._h, 1), "aoh_kv_set_decode_append")
        torch.cuda.synchronize(cache.device)
        if gather is not None:
            gather.attach()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._launch_layers()
            # the waits read the device length: they end before it advances
            _lib.check(self._L.aoh_kv_advance(cache._h, 1, C.c_void_p(_lib.stream_handle())),
                       "aoh_kv_advance")
        # capture does not execute: put the device length back to the host's
        self._set_length(cache.kv_seq_len)

    def _set_length(self, n: int) -> None:
        _lib.check(self._L.aoh_kv_set_length(self.cache._h, n, C.c_void_p(_lib.stream_handle())),
                   "aoh_kv_set_length")

    def _launch_layers(self, with_gather: bool = True) -> None:
        main = torch.cuda.current_stream(self.cache.device)
        st = C.c_void_p(_lib.stream_handle())
        h = self.cache._h
        overlap = with_gather and self.overlap_gather
        for i, layer in enumerate(self.layers):
            rc = self._L.aoh_attn_decode(h, layer, _lib.PAST_LEN_DEVICE, C.c_void_p(self.q[i].data_ptr()),
                                         C.c_void_p(self.k[i].data_ptr()), C.c_void_p(self.v[i].data_ptr()),
                                         C.c_void_p(self.out[i].data_ptr()), C.c_void_p(self._ws.data_ptr()),
                                         self._ws.numel(), st)
            _lib.check(rc, "aoh_attn_decode")
            if overlap:
                # the layer's wait starts when this layer's decode has finished
                self._side.wait_stream(main)
                side = C.c_void_p(_lib.stream_handle(self._side))
                _lib.check(self._L.aoh_gather_wait(h, layer, _lib.PAST_LEN_DEVICE, side), "aoh_gather_wait")
            elif with_gather and self.gather is not None:
                _lib.check(self._L.aoh_gather_wait(h, layer, _lib.PAST_LEN_DEVICE, st), "aoh_gather_wait")
        if overlap:
            main.wait_stream(self._side)

    def replay(self) -> None:
        """Run one decode step (all captured layers) and advance the length."""
        self.graph.replay()
        self.cache.kv_seq_len += 1

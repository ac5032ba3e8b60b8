"""Timed CPU baselines: the reference's own eager code, driven on the host cores.

MEASUREMENT INFRASTRUCTURE ONLY.  bench.py's CPU-baseline legs and its
reference arm call this module; the product path never does.  It runs the
unmodified reference package installed under ``baseline/_ref`` (a
``pip install --target`` of the reference project).  When that install is
absent or does not import, the callers fall back to the numpy restatement in
``aoh_oracle`` and report ``kind: "port"`` instead of ``"reference"``.

The reference is driven the way ``tests/golden/make_golden.py`` drives it to
make the parity fixtures:

* attention: ``make_aoh_forward`` (eval/efficiency/benchmark_llama31.py:187-253,
  benchmark_qwen.py:196-270) bound to a stub attention module whose q/k/v
  projections return the step's post-RoPE tensors in the reference's
  retrieval-first head order (eval/efficiency/reorder_weights.py:40-48) and
  whose o_proj is the identity, over the reference's own ``AoHKVCache``
  (:135-184) pre-filled with the state a long prefill leaves (full retrieval
  KV, compressed streaming KV);
* classifier: ``AoHClassifier.classify`` (aoh/classifier.py:78-135) on a stub
  model exposing ``model.model.layers[i].self_attn.{q_proj,k_proj}.weight`` in
  bf16 and a config namespace (aoh/weight_extract.py:40-77 reads exactly those).
"""
from __future__ import annotations

import os
import sys
import time
import types
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
REF_DIR = ROOT / "baseline" / "_ref"
D = 128


def load():
    """The reference's modules from ``baseline/_ref``; raises ImportError
    (with the reason) when the install is missing or does not import."""
    if not (REF_DIR / "eval" / "efficiency" / "benchmark_llama31.py").exists():
        raise ImportError(f"reference not installed under {REF_DIR}")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    from eval.efficiency import benchmark_llama31, benchmark_qwen  # noqa: E402
    from aoh.classifier import AoHClassifier  # noqa: E402
    from aoh.weight_extract import get_model_info  # noqa: E402
    return dict(bench_llama=benchmark_llama31, bench_qwen=benchmark_qwen, AoHClassifier=AoHClassifier,
                get_model_info=get_model_info)


def use_all_cores():
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def _stub(q, k, v):
    return types.SimpleNamespace(q_proj=lambda h: q, k_proj=lambda h: k, v_proj=lambda h: v, o_proj=lambda x: x)


def decode_layer_call(ref, *, num_q=32, num_kv=8, n_stream=6, context=131072, sink=128, recent=256,
                      kv_scale=0.5, seed=0):
    """A callable running one decode step of one layer through the reference's
    patched forward (Llama module), over an AoHKVCache holding ``context``
    tokens: each call attends, appends (torch.cat of the full KV) and advances
    the sequence by one token, exactly the reference's per-layer decode work."""
    import torch
    mod = ref["bench_llama"]
    nr, ns = num_kv - n_stream, n_stream
    bf = torch.bfloat16
    cache = mod.AoHKVCache(1, [nr], [ns], sink, recent)
    g = torch.Generator().manual_seed(seed)
    if nr:
        cache.full_k[0] = (torch.randn((1, nr, context, D), generator=g) * kv_scale).to(bf)
        cache.full_v[0] = (torch.randn((1, nr, context, D), generator=g) * kv_scale).to(bf)
    if ns:
        keep = min(context, sink + recent)
        cache.stream_k[0] = (torch.randn((1, ns, keep, D), generator=g) * kv_scale).to(bf)
        cache.stream_v[0] = (torch.randn((1, ns, keep, D), generator=g) * kv_scale).to(bf)
    cache.kv_seq_len = context
    q = torch.randn((1, 1, num_q * D), generator=g).to(bf)
    k = (torch.randn((1, 1, num_kv * D), generator=g) * kv_scale).to(bf)
    v = (torch.randn((1, 1, num_kv * D), generator=g) * kv_scale).to(bf)
    stub = _stub(q, k, v)
    fwd = mod.make_aoh_forward(0, nr, ns, num_q, num_kv, D)
    h = torch.zeros(1, 1, 1, dtype=bf)

    def call():
        with torch.no_grad():
            fwd(stub, h, position_embeddings=None, past_key_values=cache)

    return call


def prefill_chunk_calls(ref, *, past, chunk, n_chunks, num_q=28, num_kv=4, n_ret=2, sink=128, recent=256, seed=0):
    """Callables for ``n_chunks`` consecutive prefill chunks of one layer
    through the reference's patched forward (Qwen2 module), starting over an
    AoHKVCache that already holds ``past`` tokens."""
    import torch
    mod = ref["bench_qwen"]
    ns = num_kv - n_ret
    bf = torch.bfloat16
    cache = mod.AoHKVCache(1, [n_ret], [ns], sink, recent)
    g = torch.Generator().manual_seed(seed)
    if n_ret and past:
        cache.full_k[0] = torch.randn((1, n_ret, past, D), generator=g).to(bf)
        cache.full_v[0] = torch.randn((1, n_ret, past, D), generator=g).to(bf)
    if ns and past:
        keep = min(past, sink + recent)
        cache.stream_k[0] = torch.randn((1, ns, keep, D), generator=g).to(bf)
        cache.stream_v[0] = torch.randn((1, ns, keep, D), generator=g).to(bf)
    cache.kv_seq_len = past
    fwd = mod.make_aoh_forward(0, n_ret, ns, num_q, num_kv, D)
    h = torch.zeros(1, chunk, 1, dtype=bf)
    calls = []
    for _ in range(n_chunks):
        q = torch.randn((1, chunk, num_q * D), generator=g).to(bf)
        k = torch.randn((1, chunk, num_kv * D), generator=g).to(bf)
        v = torch.randn((1, chunk, num_kv * D), generator=g).to(bf)
        stub = _stub(q, k, v)

        def call(stub=stub):
            with torch.no_grad():
                fwd(stub, h, position_embeddings=None, past_key_values=cache)

        calls.append(call)
    return calls


class _Cfg:
    def __init__(self, L, Hq, G, d_model):
        self.num_hidden_layers = L
        self.num_attention_heads = Hq
        self.num_key_value_heads = G
        self.hidden_size = d_model
        self.head_dim = D


def classify_seconds(ref, wq_bits, wk_bits, num_q, num_kv, d_model, binary, agg="mean", sparsity=0.5):
    """Seconds of one AoHClassifier.classify over the given per-layer bf16
    weights (uint16 bit patterns, (Hq*D, d_model) and (G*D, d_model)), and
    the labels it returns."""
    import torch
    layers = []
    for wq, wk in zip(wq_bits, wk_bits):
        q = torch.from_numpy(np.ascontiguousarray(wq).astype(np.int16)).view(torch.bfloat16)
        k = torch.from_numpy(np.ascontiguousarray(wk).astype(np.int16)).view(torch.bfloat16)
        attn = types.SimpleNamespace(q_proj=types.SimpleNamespace(weight=q), k_proj=types.SimpleNamespace(weight=k))
        layers.append(types.SimpleNamespace(self_attn=attn))
    model = types.SimpleNamespace(model=types.SimpleNamespace(layers=layers))
    cfg = _Cfg(len(layers), num_q, num_kv, d_model)
    clf = ref["AoHClassifier"]("stub", torch_dtype=torch.bfloat16, device="cpu", binary=binary, agg=agg)
    clf._model, clf._config = model, cfg
    clf._info = ref["get_model_info"](cfg)
    t0 = time.perf_counter()
    labels = clf.classify(sparsity=sparsity)
    return time.perf_counter() - t0, labels

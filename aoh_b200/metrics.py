"""Work and memory accounting for the head-mixed runtime.

* ``attention_flops``: 4 * head_dim flops per masked-in (query, key) pair -- the
  algorithmic work of QK^T and P.V, used for TFLOP/s and the tensor roofline.
* ``kv_storage_gb_full`` / ``kv_storage_gb_aoh``: the reference's analytical KV
  storage (eval/efficiency/benchmark_llama31.py:341-351), the "KV GB" columns
  of its efficiency table.
* ``kv_pool_gb``: what the paged cache actually holds (pages x page bytes).
"""
from __future__ import annotations

import numpy as np


def attention_flops(q_len: int, past_len: int, retrieval: bool, sink: int, recent: int,
                    head_dim: int = 128) -> int:
    """Flops of one query head over a chunk of ``q_len`` queries at positions
    past_len.., counting only the (query, key) pairs the mask allows:
    retrieval p <= q; streaming p <= q and (p < sink or p >= q - recent)."""
    qp = np.arange(past_len, past_len + q_len, dtype=np.int64)
    if retrieval:
        pairs = (qp + 1).sum()
    else:
        pairs = (np.minimum(qp + 1, sink) + np.maximum(0, qp + 1 - np.maximum(sink, qp - recent))).sum()
    return int(pairs) * 4 * head_dim


def kv_storage_gb_full(num_layers: int, num_kv_heads: int, head_dim: int, total_len: int,
                       dtype_bytes: int = 2) -> float:
    return num_layers * 2 * num_kv_heads * total_len * head_dim * dtype_bytes / 1e9


def kv_storage_gb_aoh(n_ret, n_str, head_dim: int, total_len: int, sink_size: int, recent_size: int,
                      dtype_bytes: int = 2) -> float:
    stream_len = min(total_len, sink_size + recent_size)
    elems = 0
    for nr, ns in zip(n_ret, n_str):
        elems += 2 * (nr * total_len + ns * stream_len) * head_dim
    return elems * dtype_bytes / 1e9


def kv_pool_gb(cache) -> float:
    """Bytes of pages granted in a paged AoHKVCache (GB)."""
    used = cache.num_pages - cache.free_pages()
    return used * 2 * 16 * cache.head_dim * cache.pool_view().element_size() / 1e9

"""Seeded synthetic inputs for the head-mixed attention runtime and the classifier.

There are no checkpoints or datasets on the machines this runs on, so every
workload is generated from a seed.  Small and medium inputs come from numpy's
PCG64 generator, which gives the same values on every machine with the same
numpy; the multi-GB decode caches used for timing are filled on the device
(``torch.randn`` with a seeded CUDA generator) and are never compared value by
value with stored fixtures, only with the oracle on the same device-side data.

Shapes follow the model families the reference benchmarks:

* Llama-3.1-8B attention: 32 query heads, 8 KV heads, head_dim 128, RoPE theta 5e5.
* Qwen2.5-7B attention: 28 query heads, 4 KV heads, head_dim 128.
* Qwen3-8B attention: 32 query heads, 8 KV heads, head_dim 128.
* Qwen2.5-7B projections for the classifier: hidden 3584, 28 layers.

q/k passed to the attention op are post-RoPE (the op boundary of the
reference's ``eager_attention``/``streaming_attention``,
eval/efficiency/benchmark_llama31.py:123-132 and attention_utils.py:92-119,
is after ``apply_rotary_pos_emb``), so RoPE is applied here, with the
rotate-half convention of the HF Llama/Qwen modules.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_round",
    "bf16_to_f32",
    "f32_to_bf16_bits",
    "rope",
    "attn_layer_inputs",
    "labels_uniform",
    "labels_skewed",
    "classifier_weights",
]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    r = (u + bias) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 (exact)."""
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def rope(x: np.ndarray, positions: np.ndarray, theta: float) -> np.ndarray:
    """Rotate-half RoPE on (..., T, H, D) float32 with per-token positions (T,)."""
    d = x.shape[-1]
    inv_freq = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
    freqs = positions.astype(np.float64)[:, None] * inv_freq[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1)
    cos = np.cos(emb).astype(np.float32)[:, None, :]
    sin = np.sin(emb).astype(np.float32)[:, None, :]
    half = d // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


def attn_layer_inputs(
    seed: int,
    layer: int,
    batch: int,
    n_tokens: int,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int = 128,
    dtype: str = "f32",
    rope_theta: float | None = 500000.0,
    kv_scale: float = 1.0,
    start_pos: int = 0,
):
    """q (B,T,Hq,D), k (B,T,G,D), v (B,T,G,D) float32 for one layer.

    Values are N(0,1) (k and v multiplied by ``kv_scale``), RoPE applied to q and
    k at positions ``start_pos..start_pos+T-1``; rounded to bfloat16 values when
    ``dtype == "bf16"`` (returned as float32 arrays holding bf16 values).
    """
    rng = np.random.Generator(np.random.PCG64([seed, layer, 0xA0E]))
    shp_q = (batch, n_tokens, num_q_heads, head_dim)
    shp_kv = (batch, n_tokens, num_kv_heads, head_dim)
    q = rng.standard_normal(shp_q, dtype=np.float32)
    k = rng.standard_normal(shp_kv, dtype=np.float32) * np.float32(kv_scale)
    v = rng.standard_normal(shp_kv, dtype=np.float32) * np.float32(kv_scale)
    if rope_theta is not None:
        pos = np.arange(start_pos, start_pos + n_tokens)
        q = np.stack([rope(q[b], pos, rope_theta) for b in range(batch)])
        k = np.stack([rope(k[b], pos, rope_theta) for b in range(batch)])
    if dtype == "bf16":
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    elif dtype != "f32":
        raise ValueError(f"dtype must be 'f32' or 'bf16', got {dtype!r}")
    return q, k, v


def labels_uniform(seed: int, num_layers: int, num_kv_heads: int, n_streaming: int) -> np.ndarray:
    """(L, G) float64 labels, 1 = retrieval, 0 = streaming; per layer a uniform
    random choice of ``n_streaming`` streaming KV heads."""
    rng = np.random.Generator(np.random.PCG64([seed, 0x1AB]))
    lab = np.ones((num_layers, num_kv_heads), dtype=np.float64)
    for l in range(num_layers):
        lab[l, rng.permutation(num_kv_heads)[:n_streaming]] = 0.0
    return lab


def labels_skewed(seed: int, num_layers: int, num_kv_heads: int, n_streaming: int,
                  hot_groups: int = 2, weight: float = 4.0) -> np.ndarray:
    """Like :func:`labels_uniform`, but retrieval heads are drawn with KV groups
    ``0..hot_groups-1`` weighted ``weight``x, so they cluster in those groups."""
    rng = np.random.Generator(np.random.PCG64([seed, 0x5CE]))
    n_ret = num_kv_heads - n_streaming
    w = np.ones(num_kv_heads)
    w[:hot_groups] = weight
    lab = np.zeros((num_layers, num_kv_heads), dtype=np.float64)
    for l in range(num_layers):
        ret = rng.choice(num_kv_heads, size=n_ret, replace=False, p=w / w.sum())
        lab[l, ret] = 1.0
    return lab


def classifier_weights(seed: int, layer: int, num_q_heads: int, num_kv_heads: int,
                       head_dim: int, d_model: int, std: float = 0.02):
    """One layer's (q_proj.weight, k_proj.weight) as bfloat16 bit patterns (uint16),
    shapes (Hq*D, d_model) and (G*D, d_model), values N(0, std) rounded to bf16."""
    rng = np.random.Generator(np.random.PCG64([seed, layer, 0xC1A]))
    wq = rng.standard_normal((num_q_heads * head_dim, d_model), dtype=np.float32) * np.float32(std)
    wk = rng.standard_normal((num_kv_heads * head_dim, d_model), dtype=np.float32) * np.float32(std)
    return f32_to_bf16_bits(wq), f32_to_bf16_bits(wk)

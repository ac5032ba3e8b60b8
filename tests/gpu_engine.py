"""Drive the CUDA path with numpy inputs (test helper)."""
import numpy as np
import torch

from aoh_b200 import AoHKVCache, aoh_attention

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16}


def to_dev(x: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to("cuda").to(dtype).contiguous()


def make_cache(spec, labels, batch=1):
    total = sum(spec["chunks"]) + spec["decode"]
    return AoHKVCache(labels, spec["Hq"], batch=batch, sink_size=spec["sink"], recent_size=spec["recent"],
                      max_context=total, dtype=DTYPES[spec["dtype"]])


def step(cache, layer, q, k, v):
    out = aoh_attention(cache, layer, to_dev(q, cache.dtype), to_dev(k, cache.dtype), to_dev(v, cache.dtype))
    return out.float().cpu().numpy()

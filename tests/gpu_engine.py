"""Drive the CUDA path with numpy inputs (test helper)."""
import numpy as np
import torch

from aoh_b200 import AoHKVCache, aoh_attention
from aoh_b200 import synthetic as syn
from oracle import aoh_oracle as orc

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16}


def to_dev(x: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to("cuda").to(dtype).contiguous()


def make_cache(spec, labels, batch=1):
    total = sum(spec["chunks"]) + spec["decode"]
    return AoHKVCache(labels, spec["Hq"], batch=batch, sink_size=spec["sink"], recent_size=spec["recent"],
                      max_context=total, dtype=DTYPES[spec["dtype"]], backend=spec.get("backend", "eager"))


def step(cache, layer, q, k, v):
    out = aoh_attention(cache, layer, to_dev(q, cache.dtype), to_dev(k, cache.dtype), to_dev(v, cache.dtype))
    return out.float().cpu().numpy()


def run_both(dtype, Hq, G, labels, chunks, decode, sink, recent, seed, batch=1, kv_scale=1.0):
    """Run the same seeded sequence through the oracle and the CUDA path; return
    the worst error per step kind."""
    L = labels.shape[0]
    total = sum(chunks) + decode
    inputs = [syn.attn_layer_inputs(seed, l, batch, total, Hq, G, 128, dtype=dtype, kv_scale=kv_scale)
              for l in range(L)]
    oc = orc.OracleKVCache(L, labels, sink, recent, dtype)
    gcache = AoHKVCache(labels, Hq, batch=batch, sink_size=sink, recent_size=recent, max_context=total,
                        dtype=DTYPES[dtype])
    errs = {"prefill": 0.0, "decode": 0.0}
    start = 0
    for c in list(chunks) + [1] * decode:
        for l in range(L):
            q, k, v = (x[:, start:start + c] for x in inputs[l])
            want = orc.layer_attention(oc, l, q, k, v)
            got = step(gcache, l, q, k, v)
            kind = "decode" if c == 1 else "prefill"
            errs[kind] = max(errs[kind], float(np.abs(got - want).max()))
        start += c
    assert gcache.device_status() == 0
    return errs

"""Replay of the golden attention cases through an engine (oracle or CUDA path).

The inputs are regenerated from the seeds recorded in the fixtures (numpy
PCG64, identical on every machine with this numpy); a checksum stored with
each fixture guards against generator drift."""
from __future__ import annotations

import ast
from pathlib import Path

import numpy as np

from aoh_b200 import synthetic as syn

GOLDEN = Path(__file__).resolve().parent / "golden"
ATTN_CASES = ["attn_f32_window", "attn_f32_llama", "attn_bf16_qwen25", "attn_bf16_decode",
              "attn_f32_odd"]
# the decoding-simulation protocol (backend "flash"); made on a CUDA device
FLASH_CASES = ["attn_flash_bf16_small", "attn_flash_bf16_qwen25"]
# bf16 outputs are compared at the bf16 tolerance, f32 outputs at the f32 one
TOL = {"bf16": 2e-2, "f32": 1e-4}


def load_case(name: str):
    z = np.load(GOLDEN / f"{name}.npz")
    spec = ast.literal_eval(str(z["spec"]))
    if "out_bf16" in z:
        ref = syn.bf16_to_f32(z["out_bf16"])
    else:
        ref = z["out_f32"]
    return spec, z["labels"], z["rows"], ref, z["checksum"], [int(s) for s in z["steps"]]


def case_inputs(spec, layers):
    total = sum(spec["chunks"]) + spec["decode"]
    return [syn.attn_layer_inputs(spec["seed"], l, 1, total, spec["Hq"], spec["G"], 128,
                                  dtype=spec["dtype"], rope_theta=500000.0) for l in range(layers)]


def replay(name: str, make_cache, step):
    """Run every chunk and decode step of the case through ``step`` and return
    (spec, got (L, rows, Hq, D), ref (same), input checksum ok)."""
    spec, labels, rows, ref, checksum, steps = load_case(name)
    L = spec["layers"]
    inputs = case_inputs(spec, L)
    ck = np.array([float(np.float64(x).sum()) for l in range(L) for x in inputs[l]])
    cache = make_cache(spec, labels)
    total = sum(steps)
    out = np.zeros((L, total, spec["Hq"], 128), dtype=np.float32)
    start = 0
    for c in steps:
        for l in range(L):
            q, k, v = (x[:, start:start + c] for x in inputs[l])
            out[l, start:start + c] = step(cache, l, q, k, v)[0]
        start += c
    return spec, out[:, rows], ref, bool(np.allclose(ck, checksum, rtol=1e-12, atol=0))

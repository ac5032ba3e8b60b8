"""Generate golden fixtures by running the REFERENCE implementation itself.

Run in a container where the reference project (ernie-research/AoH) is
available; pass its root with ``--ref`` (default: the REF_ROOT environment
variable) -- the project tree, or an installed copy of it.  Writes
``tests/golden/*.npz`` (or ``--out``).  The decoding-simulation ("flash")
cases run the reference's FlashAttention-2 path and need a CUDA device with
flash_attn.  Nothing at test time imports the reference: the fixtures carry
its outputs.

Attention: the reference's patched attention forward
(eval/efficiency/benchmark_llama31.py:187-253, make_aoh_forward) is driven with
a stub attention module whose q/k/v projections return seeded post-RoPE
tensors, already permuted into the reference's retrieval-first head order
(eval/efficiency/reorder_weights.py:40-48), and whose o_proj is the identity;
the cache is the reference's own AoHKVCache (:135-184).  Outputs are mapped
back to the original head order.

Classifier: AoHClassifier.classify (aoh/classifier.py:78-135) on a stub model
exposing ``model.model.layers[i].self_attn.{q_proj,k_proj}.weight`` in bf16 and
a config namespace; ``_model/_config/_info`` are set directly so no checkpoint
is loaded (aoh/weight_extract.py:40-77 reads exactly these attributes).
"""
from __future__ import annotations

import argparse
import os
import sys
import time
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE  # --out: where the fixtures go
sys.path.insert(0, str(HERE.parents[1]))
from aoh_b200 import synthetic as syn  # noqa: E402

# ----------------------------------------------------------------------------
# cases (kept small: fixtures are committed)
# ----------------------------------------------------------------------------

ATTN_CASES = {
    # ring wraps many times, ragged last chunk, both head kinds in each layer
    "attn_f32_window": dict(model="llama", dtype="f32", Hq=4, G=2, layers=2,
                            labels=[[1, 0], [0, 1]], sink=16, recent=32,
                            chunks=[40, 40, 40, 7], decode=6, seed=11, row_stride=1),
    # Llama-3.1-8B head shapes, reference sink/window
    "attn_f32_llama": dict(model="llama", dtype="f32", Hq=32, G=8, layers=1,
                           labels="uniform4", sink=128, recent=256,
                           chunks=[256, 256], decode=3, seed=12, row_stride=16),
    # Qwen2.5-7B group size 7, bf16
    "attn_bf16_qwen25": dict(model="qwen", dtype="bf16", Hq=14, G=2, layers=1,
                             labels=[[0, 1]], sink=128, recent=256,
                             chunks=[256, 192], decode=3, seed=13, row_stride=8),
    # context not a multiple of the page size, decode after a long chunk
    "attn_bf16_decode": dict(model="llama", dtype="bf16", Hq=8, G=2, layers=1,
                             labels=[[1, 0]], sink=128, recent=256,
                             chunks=[500, 500], decode=3, seed=14, row_stride=25),
    # sink/window not multiples of 16, tiny chunks
    "attn_f32_odd": dict(model="llama", dtype="f32", Hq=4, G=2, layers=1,
                         labels=[[0, 1]], sink=5, recent=23, chunks=[9, 30, 1, 17],
                         decode=4, seed=15, row_stride=1),
    # the decoding-simulation protocol (backend "flash": FlashAttention-2 on a
    # CUDA device): the prompt in one call, every head causal over it, the
    # streaming heads trimmed, then decode steps
    "attn_flash_bf16_small": dict(model="llama", dtype="bf16", Hq=8, G=2, layers=2,
                                  labels=[[1, 0], [0, 1]], sink=16, recent=32, chunks=[300],
                                  decode=6, seed=31, row_stride=7, backend="flash"),
    "attn_flash_bf16_qwen25": dict(model="qwen", dtype="bf16", Hq=14, G=2, layers=1,
                                   labels=[[0, 1]], sink=128, recent=256, chunks=[700],
                                   decode=4, seed=32, row_stride=13, backend="flash"),
}

CLS_CASES = {
    "cls_small": dict(L=2, Hq=8, G=2, D=128, dm=512, seed=1),
    "cls_qwen25_7b": dict(L=28, Hq=28, G=4, D=128, dm=3584, seed=0),
    # more seeds of the Qwen2.5-7B-shaped case: how often, and how narrowly,
    # float32 ties in the reference's own ranks decide a label
    **{f"cls_qwen25_7b_s{s}": dict(L=28, Hq=28, G=4, D=128, dm=3584, seed=s) for s in (1, 2, 3, 4)},
}
# Analytical KV storage (the reference's "KV GB" columns): model shape, labels
# per layer as (n_ret, n_str), context, sink, recent.
KV_CASES = {
    "llama31_8b_128k_sp075": dict(L=32, G=8, Hq=32, hidden=4096, head_dim=128, n_ret=2, total=131072),
    "llama31_8b_64k_sp05": dict(L=32, G=8, Hq=32, hidden=4096, head_dim=128, n_ret=4, total=65536),
    "qwen25_7b_64k_sp05": dict(L=28, G=4, Hq=28, hidden=3584, head_dim=None, n_ret=2, total=65536),
    "qwen3_8b_256k_sp075": dict(L=36, G=8, Hq=32, hidden=4096, head_dim=128, n_ret=2, total=262144),
    "short_context_below_window": dict(L=2, G=4, Hq=8, hidden=1024, head_dim=128, n_ret=1, total=200),
}
AGGS = ("mean", "min", "max")
SPARSITIES = (0.25, 0.5, 0.75)


def case_labels(spec, L, G):
    lab = spec["labels"]
    if lab == "uniform4":
        return syn.labels_uniform(spec["seed"], L, G, 4)
    return np.asarray(lab, dtype=np.float64)


def case_inputs(spec, layer):
    total = sum(spec["chunks"]) + spec["decode"]
    return syn.attn_layer_inputs(spec["seed"], layer, 1, total, spec["Hq"], spec["G"], 128,
                                 dtype=spec["dtype"], rope_theta=500000.0)


def run_attention_case(name, spec, ref):
    L, Hq, G, D = spec["layers"], spec["Hq"], spec["G"], 128
    backend = spec.get("backend", "eager")
    dev = "cuda" if backend == "flash" else "cpu"  # flash_attn runs on a CUDA device only
    grp = Hq // G
    tdt = torch.float32 if spec["dtype"] == "f32" else torch.bfloat16
    labels = case_labels(spec, L, G)
    mod = ref["bench_llama"] if spec["model"] == "llama" else ref["bench_qwen"]
    perms, n_ret, n_str = [], [], []
    for l in range(L):
        row = labels[l]
        rk = np.where(row >= 0.5)[0]
        sk = np.where(row < 0.5)[0]
        kv_perm = np.concatenate([rk, sk])
        q_perm = np.concatenate([np.arange(g * grp, (g + 1) * grp) for g in kv_perm])
        perms.append((kv_perm, q_perm))
        n_ret.append(len(rk)); n_str.append(len(sk))
    cache = mod.AoHKVCache(L, n_ret, n_str, spec["sink"], spec["recent"], backend)
    inputs = [case_inputs(spec, l) for l in range(L)]
    steps = list(spec["chunks"]) + [1] * spec["decode"]
    total = sum(steps)
    outs = np.zeros((L, total, Hq, D), dtype=np.float32)
    start = 0
    for c in steps:
        for l in range(L):
            q, k, v = (x[:, start:start + c] for x in inputs[l])
            kv_perm, q_perm = perms[l]
            qt = torch.from_numpy(np.ascontiguousarray(q[:, :, q_perm])).to(dev).to(tdt).reshape(1, c, Hq * D)
            kt = torch.from_numpy(np.ascontiguousarray(k[:, :, kv_perm])).to(dev).to(tdt).reshape(1, c, G * D)
            vt = torch.from_numpy(np.ascontiguousarray(v[:, :, kv_perm])).to(dev).to(tdt).reshape(1, c, G * D)
            stub = types.SimpleNamespace(q_proj=lambda h, t=qt: t, k_proj=lambda h, t=kt: t,
                                         v_proj=lambda h, t=vt: t, o_proj=lambda x: x)
            fwd = mod.make_aoh_forward(l, n_ret[l], n_str[l], Hq, G, D)
            with torch.no_grad():
                o, _ = fwd(stub, torch.zeros(1, c, 1, dtype=tdt, device=dev), position_embeddings=None,
                           past_key_values=cache)
            o = o.float().cpu().numpy().reshape(c, Hq, D)
            outs[l, start:start + c][:, q_perm] = o
        start += c
    # row subset: every row_stride-th prefill row of each chunk + all decode rows
    rows = []
    s = 0
    for c in spec["chunks"]:
        rows.extend(range(s, s + c, spec["row_stride"]))
        rows.append(s + c - 1)
        s += c
    rows.extend(range(s, s + spec["decode"]))
    rows = np.array(sorted(set(rows)), dtype=np.int64)
    sel = outs[:, rows]
    checksum = np.array([float(np.float64(x).sum()) for l in range(L) for x in inputs[l]])
    out = dict(rows=rows, labels=labels, checksum=checksum,
               spec=np.array(repr(spec)), steps=np.array(steps, dtype=np.int64))
    if spec["dtype"] == "bf16":
        out["out_bf16"] = syn.f32_to_bf16_bits(sel)
    else:
        out["out_f32"] = sel
    np.savez_compressed(OUT / f"{name}.npz", **out)
    print(f"[golden] {name}: rows={len(rows)} out={sel.shape}", flush=True)


class _Cfg:
    def __init__(self, L, Hq, G, D, dm):
        self.num_hidden_layers = L
        self.num_attention_heads = Hq
        self.num_key_value_heads = G
        self.hidden_size = dm
        self.head_dim = D


def run_classifier_case(name, spec, ref):
    L, Hq, G, D, dm, seed = (spec[k] for k in ("L", "Hq", "G", "D", "dm", "seed"))
    layers = []
    for l in range(L):
        wq, wk = syn.classifier_weights(seed, l, Hq, G, D, dm)
        q = torch.from_numpy(wq.astype(np.int16)).view(torch.bfloat16)
        k = torch.from_numpy(wk.astype(np.int16)).view(torch.bfloat16)
        attn = types.SimpleNamespace(q_proj=types.SimpleNamespace(weight=q),
                                     k_proj=types.SimpleNamespace(weight=k))
        layers.append(types.SimpleNamespace(self_attn=attn))
    model = types.SimpleNamespace(model=types.SimpleNamespace(layers=layers))
    cfg = _Cfg(L, Hq, G, D, dm)
    out = {}
    for binary in (False, True):
        mode = "binary" if binary else "fp32"
        for agg in AGGS:
            for sp in SPARSITIES:
                clf = ref["AoHClassifier"]("stub", torch_dtype=torch.bfloat16, device="cpu",
                                           binary=binary, agg=agg)
                clf._model, clf._config = model, cfg
                clf._info = ref["get_model_info"](cfg)
                t0 = time.perf_counter()
                labels = clf.classify(sparsity=sp)
                dt = time.perf_counter() - t0
                out[f"{mode}_eff_ranks_q"] = clf.eff_ranks_q
                out[f"{mode}_{agg}_eff_ranks_kv"] = clf.eff_ranks_kv
                out[f"{mode}_{agg}_sp{sp}_labels"] = labels
                out[f"{mode}_classify_seconds"] = np.array(dt)
    np.savez_compressed(OUT / f"{name}.npz", spec=np.array(repr(spec)), **out)
    print(f"[golden] {name} written", flush=True)


def run_kv_storage_cases(ref):
    """kv_storage_gb_full / kv_storage_gb_aoh (eval/efficiency/benchmark_llama31.py:341-351)
    on config namespaces; sink 128, recent 256, bf16."""
    names, full, aoh, spec = [], [], [], []
    for name, c in KV_CASES.items():
        cfg = types.SimpleNamespace(num_hidden_layers=c["L"], num_key_value_heads=c["G"],
                                    num_attention_heads=c["Hq"], hidden_size=c["hidden"])
        if c["head_dim"] is not None:
            cfg.head_dim = c["head_dim"]
        n_ret = [c["n_ret"]] * c["L"]
        n_str = [c["G"] - c["n_ret"]] * c["L"]
        names.append(name)
        full.append(ref["bench_llama"].kv_storage_gb_full(cfg, c["total"]))
        aoh.append(ref["bench_llama"].kv_storage_gb_aoh(cfg, n_ret, n_str, c["total"], 128, 256))
        spec.append(repr(c))
    np.savez_compressed(OUT / "kv_storage.npz", names=np.array(names), specs=np.array(spec),
                        full_gb=np.array(full), aoh_gb=np.array(aoh))
    print(f"[golden] kv_storage: {len(names)} cases", flush=True)


def load_reference(root: Path):
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "eval" / "efficiency"))
    import benchmark_llama31  # noqa: E402
    import benchmark_qwen  # noqa: E402
    from aoh.classifier import AoHClassifier  # noqa: E402
    from aoh.weight_extract import get_model_info  # noqa: E402
    return dict(bench_llama=benchmark_llama31, bench_qwen=benchmark_qwen,
                AoHClassifier=AoHClassifier, get_model_info=get_model_info)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("REF_ROOT", ""))
    ap.add_argument("--only", default="")
    ap.add_argument("--out", default=str(HERE), help="directory for the .npz fixtures")
    args = ap.parse_args()
    global OUT
    OUT = Path(args.out)
    OUT.mkdir(parents=True, exist_ok=True)
    if not args.ref:
        ap.error("pass --ref <reference project root> or set REF_ROOT")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = load_reference(Path(args.ref))
    for name, spec in ATTN_CASES.items():
        if not args.only or args.only in name:
            run_attention_case(name, spec, ref)
    for name, spec in CLS_CASES.items():
        if not args.only or args.only in name:
            run_classifier_case(name, spec, ref)
    if not args.only or args.only in "kv_storage":
        run_kv_storage_cases(ref)


if __name__ == "__main__":
    main()

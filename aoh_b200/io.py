"""Head-map files: the reference's on-disk format (aoh/io.py:9-62).

``eff_rank.npy`` (L, H), ``eff_rank_kv.npy`` (L, G), ``head_classification.npy``
(L, G) float64 labels, and ``results.json`` (run metadata plus per-layer
retrieval/streaming ratios, version "AoH-v1").  Files written here load with
the reference's ``load_results`` and vice versa.
"""
from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path

import numpy as np


def save_results(output_dir: str, eff_ranks_q: np.ndarray, eff_ranks_kv: np.ndarray,
                 head_labels: np.ndarray, metadata: dict) -> None:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    np.save(out / "eff_rank.npy", eff_ranks_q)
    np.save(out / "eff_rank_kv.npy", eff_ranks_kv)
    np.save(out / "head_classification.npy", head_labels)
    per_layer = head_labels.mean(axis=1)
    results = {
        **metadata,
        "version": "AoH-v1",
        "num_layers": int(head_labels.shape[0]),
        "num_kv_heads": int(head_labels.shape[1]),
        "overall_retrieval_ratio": float(head_labels.mean()),
        "overall_streaming_ratio": float(1.0 - head_labels.mean()),
        "retrieval_ratio_per_layer": per_layer.tolist(),
        "streaming_ratio_per_layer": (1.0 - per_layer).tolist(),
    }
    # write-then-rename so a crash never leaves a truncated results.json
    fd, tmp = tempfile.mkstemp(dir=out, prefix=".results.", suffix=".json")
    with os.fdopen(fd, "w", encoding="utf-8") as f:
        json.dump(results, f, indent=2)
    os.replace(tmp, out / "results.json")


# result key -> file name: the reference's names, so head maps move between the two
_FILES = (("eff_ranks_q", "eff_rank.npy"), ("eff_ranks_kv", "eff_rank_kv.npy"),
          ("head_labels", "head_classification.npy"), ("metadata", "results.json"))


def load_results(output_dir: str) -> dict:
    """The four head-map files of ``output_dir`` as a dict (arrays, and the
    run metadata from results.json).  FileNotFoundError, as in the reference,
    when any of them is absent -- naming every absent one."""
    out = Path(output_dir)
    paths = {key: out / name for key, name in _FILES}
    absent = sorted(name for key, name in _FILES if not paths[key].is_file())
    if absent:
        raise FileNotFoundError(f"{out} is not a complete head map: no {', '.join(absent)}")
    loaded = {key: np.load(path) for key, path in paths.items() if key != "metadata"}
    loaded["metadata"] = json.loads(paths["metadata"].read_text(encoding="utf-8"))
    return loaded

"""AoHClassifier: training-free retrieval/streaming head labels from the
effective rank of W_K^T W_Q, with the per-head spectra computed on the GPU.

API and host logic follow the reference (aoh/classifier.py, aoh/effective_rank.py):

* ``AoHClassifier(model_path, torch_dtype="auto", device="cuda", binary=False,
  agg="mean")`` -> ``.classify(sparsity) -> (L, G) float64 in {0, 1}``
  (1 = retrieval), filling ``eff_ranks_q (L, H)``, ``eff_ranks_kv (L, G)`` and
  ``head_labels``; ``.save(dir)`` / ``.from_saved(dir)`` use the reference's
  file format (aoh/io.py:9-62).
* ``compute_all_eff_ranks(model, config, binary, device)`` -> (L, H) float64
  (effective_rank.py:109-142), ``compute_eff_rank(W_Q_h, W_K_g, binary)``
  (:88-106).

The spectra come from libaoh's batched kernels (``aoh_classify_eff_ranks``):
Gram matrices (in ``binary`` mode on the integer tensor cores, exact), Cholesky
whitening and a Householder-tridiagonal + bisection eigen-solve in float64 -- more accurate than the
reference's float32 ``eigvals``.  Aggregation (float64
mean/min/max over each KV group's query heads) and the per-layer choice of the
``round((1 - sparsity) * G)`` lowest-rank KV heads are the reference's own
host arithmetic (classifier.py:102-128).  ``label_margins`` reports, per
layer, the relative gap at the retrieval/streaming boundary, the quantity that
decides whether float32 noise could flip a label.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .io import load_results, save_results


def _device(device) -> torch.device:
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError(f"the classifier kernels run on a CUDA device, got {device!r}")
    return d


def eff_ranks_from_weights(wq: torch.Tensor, wk: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                           head_dim: int = 128, binary: bool = False) -> np.ndarray:
    """(L, H) effective ranks from stacked projection weights on one device.

    wq: (L, H*D, d_model), wk: (L, G*D, d_model), bf16 or float32 (float16 is
    promoted to float32, exactly)."""
    if wq.dim() != 3 or wk.dim() != 3:
        raise ValueError("wq and wk must be (num_layers, heads * head_dim, d_model)")
    if wq.dtype == torch.float16:
        wq = wq.float()
    if wk.dtype == torch.float16:
        wk = wk.float()
    if wq.dtype != wk.dtype or wq.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("weights must both be bfloat16 or float32")
    wq, wk = wq.contiguous(), wk.contiguous()
    L, hd, dm = wq.shape
    if hd != num_q_heads * head_dim or tuple(wk.shape) != (L, num_kv_heads * head_dim, dm):
        raise ValueError("weight shapes do not match the head counts")
    lib = _lib.lib()
    nbytes = lib.aoh_classify_workspace_bytes(L, num_q_heads, num_kv_heads, head_dim)
    ws = torch.empty(max(1, nbytes), dtype=torch.uint8, device=wq.device)
    out = torch.empty((L, num_q_heads), dtype=torch.float64, device=wq.device)
    dt = _lib.BF16 if wq.dtype == torch.bfloat16 else _lib.F32
    with torch.cuda.device(wq.device):
        rc = lib.aoh_classify_eff_ranks(C.c_void_p(wq.data_ptr()), C.c_void_p(wk.data_ptr()), dt, L,
                                        num_q_heads, num_kv_heads, head_dim, dm, int(bool(binary)),
                                        C.c_void_p(out.data_ptr()), C.c_void_p(ws.data_ptr()), ws.numel(),
                                        C.c_void_p(_lib.stream_handle()))
        _lib.check(rc, "aoh_classify_eff_ranks")
        ranks = out.cpu().numpy()
    if not np.all(np.isfinite(ranks)):
        # a bounded device wait gave up: the affected heads' spectra are NaN
        raise RuntimeError("aoh_classify_eff_ranks: a device wait timed out (non-finite effective ranks)")
    return ranks


def get_model_info(config) -> dict:
    """aoh/weight_extract.py:40-63."""
    num_layers = config.num_hidden_layers
    H = config.num_attention_heads
    G = getattr(config, "num_key_value_heads", H)
    d_model = config.hidden_size
    d_head = getattr(config, "head_dim", d_model // H)
    return {"num_layers": num_layers, "H": H, "G": G, "GRP": H // G, "d_head": d_head,
            "d_model": d_model, "is_gqa": G < H}


def _get_layer(model, layer_idx: int):
    """aoh/weight_extract.py:66-77."""
    if hasattr(model, "model") and hasattr(model.model, "layers"):
        return model.model.layers[layer_idx].self_attn
    if hasattr(model, "layers"):
        return model.layers[layer_idx].self_attn
    raise AttributeError(f"Cannot locate layers in model of type {type(model).__name__}. "
                         "Expected model.model.layers or model.layers.")


@torch.no_grad()
def compute_all_eff_ranks(model, config, binary: bool = False, device: str = "cuda") -> np.ndarray:
    """Effective ranks of every query head, (L, H) float64; effective_rank.py:109-142."""
    info = get_model_info(config)
    dev = _device(device)
    L, H, G, D = info["num_layers"], info["H"], info["G"], info["d_head"]
    ws = [_get_layer(model, l).q_proj.weight.data for l in range(L)]
    dt = torch.bfloat16 if all(w.dtype == torch.bfloat16 for w in ws) else torch.float32
    wq = torch.stack([w.to(device=dev, dtype=dt) for w in ws])
    wk = torch.stack([_get_layer(model, l).k_proj.weight.data.to(device=dev, dtype=dt) for l in range(L)])
    return eff_ranks_from_weights(wq, wk, H, G, D, binary)


@torch.no_grad()
def compute_eff_rank(W_Q_h: torch.Tensor, W_K_g: torch.Tensor, binary: bool = False,
                     device: str = "cuda") -> float:
    """Effective rank of one (query head, KV head) pair; effective_rank.py:88-106.

    W_Q_h, W_K_g: (d_head, d_model)."""
    dev = _device(device)
    dt = torch.bfloat16 if W_Q_h.dtype == torch.bfloat16 and W_K_g.dtype == torch.bfloat16 else torch.float32
    d_head, dm = W_Q_h.shape
    wq = W_Q_h.to(device=dev, dtype=dt).reshape(1, d_head, dm)
    wk = W_K_g.to(device=dev, dtype=dt).reshape(1, d_head, dm)
    return float(eff_ranks_from_weights(wq, wk, 1, 1, d_head, binary)[0, 0])


def aggregate_kv(eff_ranks_q: np.ndarray, num_kv_heads: int, agg: str) -> np.ndarray:
    """GQA aggregation in float64, classifier.py:102-116 (MHA: a copy)."""
    L, H = eff_ranks_q.shape
    if num_kv_heads == H:
        return eff_ranks_q.copy()
    grp = H // num_kv_heads
    out = np.zeros((L, num_kv_heads), dtype=np.float64)
    for l in range(L):
        for g in range(num_kv_heads):
            r = eff_ranks_q[l, g * grp:(g + 1) * grp]
            out[l, g] = r.mean() if agg == "mean" else (r.min() if agg == "min" else r.max())
    return out


def labels_from_ranks(eff_ranks_kv: np.ndarray, sparsity: float) -> np.ndarray:
    """Lowest-rank ``round((1 - sparsity) * G)`` KV heads per layer are retrieval
    (1.0); classifier.py:118-128 (Python round: half to even; stable ascending
    argsort order as numpy's default quicksort on these sizes)."""
    L, G = eff_ranks_kv.shape
    k = max(0, min(G, round((1.0 - sparsity) * G)))
    labels = np.zeros((L, G), dtype=np.float64)
    for l in range(L):
        labels[l, np.argsort(eff_ranks_kv[l])[:k]] = 1.0
    return labels


def label_margins(eff_ranks_kv: np.ndarray, sparsity: float) -> np.ndarray:
    """Per layer: relative gap between the highest retrieval and the lowest
    streaming aggregated rank (inf when every head has one label)."""
    L, G = eff_ranks_kv.shape
    k = max(0, min(G, round((1.0 - sparsity) * G)))
    out = np.full(L, np.inf)
    if 0 < k < G:
        for l in range(L):
            s = np.sort(eff_ranks_kv[l])
            out[l] = (s[k] - s[k - 1]) / abs(s[k])
    return out


class AoHClassifier:
    """Training-free attention head classifier (aoh/classifier.py:19-198).

    ``model_path`` is loaded with transformers when ``model`` is not given
    (the reference's ``_ensure_model``, classifier.py:59-76); pass ``model``
    and ``config`` to classify an in-memory model (any object exposing
    ``model.layers[i].self_attn.{q,k}_proj.weight``)."""

    def __init__(self, model_path: str = "", torch_dtype="auto", device: str = "cuda",
                 binary: bool = False, agg: str = "mean", model=None, config=None):
        if agg not in ("mean", "min", "max"):  # classifier.py:41-42
            raise ValueError(f"agg must be 'mean', 'min', or 'max', got {agg!r}")
        self.model_path = model_path
        self.torch_dtype = torch_dtype
        self.device = device
        self.binary = binary
        self.agg = agg
        self._model = model
        self._config = config if config is not None else (getattr(model, "config", None) if model else None)
        if self._config is not None and hasattr(self._config, "text_config"):
            self._config = self._config.text_config
        self._info = get_model_info(self._config) if self._config is not None else None
        self.eff_ranks_q = None
        self.eff_ranks_kv = None
        self.head_labels = None
        self.sparsity = None

    def _ensure_model(self):
        if self._model is None:
            from transformers import AutoModelForCausalLM
            model = AutoModelForCausalLM.from_pretrained(self.model_path, torch_dtype=self.torch_dtype,
                                                         low_cpu_mem_usage=True)
            model.eval()
            cfg = model.config
            if hasattr(cfg, "text_config"):
                cfg = cfg.text_config
            self._model, self._config = model, cfg
            self._info = get_model_info(cfg)

    def classify(self, sparsity: float = 0.5) -> np.ndarray:
        """(num_layers, G) labels: 1.0 = retrieval, 0.0 = streaming."""
        self.sparsity = sparsity
        self._ensure_model()
        info = self._info
        self.eff_ranks_q = compute_all_eff_ranks(self._model, self._config, binary=self.binary,
                                                 device=self.device)
        self.eff_ranks_kv = (aggregate_kv(self.eff_ranks_q, info["G"], self.agg) if info["is_gqa"]
                             else self.eff_ranks_q.copy())
        self.head_labels = labels_from_ranks(self.eff_ranks_kv, sparsity)
        return self.head_labels

    def classify_from_ranks(self, eff_ranks_q: np.ndarray, num_kv_heads: int, sparsity: float) -> np.ndarray:
        """Aggregate and label precomputed per-query-head ranks (e.g. to sweep
        sparsity/agg without recomputing spectra)."""
        self.sparsity = sparsity
        self.eff_ranks_q = eff_ranks_q
        gqa = num_kv_heads < eff_ranks_q.shape[1]
        self.eff_ranks_kv = aggregate_kv(eff_ranks_q, num_kv_heads, self.agg) if gqa else eff_ranks_q.copy()
        self.head_labels = labels_from_ranks(self.eff_ranks_kv, sparsity)
        return self.head_labels

    def save(self, output_dir: str) -> None:
        """classifier.py:137-169 (same files and metadata keys)."""
        if self.head_labels is None:
            raise RuntimeError("Call classify() before save().")
        info = self._info
        metadata = {
            "model": self.model_path,
            "method": "AoH (Autonomy-of-Heads)",
            "mode": "GQA" if info["is_gqa"] else "MHA",
            "agg": self.agg if info["is_gqa"] else "N/A",
            "binary": self.binary,
            "sparsity": self.sparsity,
            "num_layers": info["num_layers"],
            "num_q_heads": info["H"],
            "num_kv_heads": info["G"],
            "group_size": info["GRP"],
            "d_head": info["d_head"],
        }
        save_results(output_dir, eff_ranks_q=self.eff_ranks_q, eff_ranks_kv=self.eff_ranks_kv,
                     head_labels=self.head_labels, metadata=metadata)

    @classmethod
    def from_saved(cls, output_dir: str) -> "AoHClassifier":
        """classifier.py:171-198."""
        data = load_results(output_dir)
        meta = data["metadata"] or {}
        obj = cls.__new__(cls)
        obj.model_path = meta.get("model", "")
        obj.torch_dtype = torch.float32
        obj.device = "cuda"
        obj.binary = meta.get("binary", False)
        obj.agg = meta.get("agg", "mean")
        obj.sparsity = meta.get("sparsity", None)
        obj._model = None
        obj._config = None
        obj._info = {
            "num_layers": meta.get("num_layers", 0),
            "H": meta.get("num_q_heads", 0),
            "G": meta.get("num_kv_heads", 0),
            "GRP": meta.get("group_size", 1),
            "d_head": meta.get("d_head", 0),
            "d_model": 0,
            "is_gqa": meta.get("mode") == "GQA",
        }
        obj.eff_ranks_q = data["eff_ranks_q"]
        obj.eff_ranks_kv = data["eff_ranks_kv"]
        obj.head_labels = data["head_labels"]
        return obj

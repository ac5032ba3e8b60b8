"""aoh_b200: B200-native (sm_100a) head-mixed attention runtime and effective-rank
head classifier, with the API of ernie-research/AoH.

    from aoh_b200 import AoHClassifier, AoHKVCache, aoh_attention
    from aoh_b200 import patch_aoh_model   # HF models (transformers), as the reference's

The CUDA kernels live in libaoh.so (built in-tree by ``python -m aoh_b200.build``)
behind the C ABI of include/aoh.h.
"""
from .attention import aoh_attention, rope_qk
from .cache import AoHKVCache, pages_needed
from .classifier import AoHClassifier, compute_all_eff_ranks, compute_eff_rank, label_margins
from .io import load_results, save_results


def __getattr__(name):
    # HF integration (imports transformers): loaded on first use
    if name in ("patch_aoh_model", "AoHModelCache", "ModelDecodeGraph"):
        from . import hf
        return getattr(hf, name)
    raise AttributeError(f"module 'aoh_b200' has no attribute {name!r}")


__all__ = [
    "AoHClassifier",
    "AoHKVCache",
    "aoh_attention",
    "rope_qk",
    "compute_all_eff_ranks",
    "compute_eff_rank",
    "label_margins",
    "patch_aoh_model",
    "ModelDecodeGraph",
    "load_results",
    "pages_needed",
    "save_results",
]

"""KV memory accounting against the reference's own formulas.

tests/golden/kv_storage.npz holds kv_storage_gb_full / kv_storage_gb_aoh as the
reference computes them (eval/efficiency/benchmark_llama31.py:341-351, the "KV
GB" columns of its efficiency tables), for Llama-3.1-8B, Qwen2.5-7B and
Qwen3-8B shapes and a context below the streaming window; aoh_b200.metrics
and the oracle must reproduce them, and the paged pool's granted pages must
cover exactly what the analytical count says plus the page rounding."""
import ast

import numpy as np
import pytest

from aoh_b200 import metrics
from oracle import aoh_oracle as orc
from tests.golden_cases import GOLDEN


def _cases():
    z = np.load(GOLDEN / "kv_storage.npz")
    return [(str(n), ast.literal_eval(str(s)), float(f), float(a))
            for n, s, f, a in zip(z["names"], z["specs"], z["full_gb"], z["aoh_gb"])]


@pytest.mark.parametrize("name,spec,full_gb,aoh_gb", _cases())
def test_kv_storage_matches_reference(name, spec, full_gb, aoh_gb):
    hd = spec["head_dim"] or spec["hidden"] // spec["Hq"]
    L, G, nr, T = spec["L"], spec["G"], spec["n_ret"], spec["total"]
    n_ret, n_str = [nr] * L, [G - nr] * L
    assert metrics.kv_storage_gb_full(L, G, hd, T) == pytest.approx(full_gb, rel=1e-12)
    assert metrics.kv_storage_gb_aoh(n_ret, n_str, hd, T, 128, 256) == pytest.approx(aoh_gb, rel=1e-12)
    assert orc.kv_storage_gb_aoh(L, hd, n_ret, n_str, T, 128, 256) == pytest.approx(aoh_gb, rel=1e-12)


def test_pool_pages_cover_the_analytical_storage():
    """A cache sized for T tokens holds, per retrieval unit, ceil(T / 16) pages
    and, per streaming unit, ceil(sink / 16) + ceil(recent / 16) pages: the
    reference's analytical bytes rounded up to whole pages (host-side count,
    no device memory)."""
    from aoh_b200.cache import pages_needed
    labels = np.array([[1, 0, 0, 0, 1, 0, 0, 0]] * 4, dtype=np.float64)
    T, sink, recent = 131072, 128, 256
    pages = pages_needed(labels, 1, T, sink, recent)
    page_bytes = 2 * 16 * 128 * 2
    n_ret = [2] * 4
    n_str = [6] * 4
    analytical = metrics.kv_storage_gb_aoh(n_ret, n_str, 128, T, sink, recent) * 1e9
    assert pages * page_bytes == analytical  # 16 | T and 16 | sink + recent: no rounding here
    assert pages_needed(labels, 1, T + 1, sink, recent) * page_bytes > analytical

"""The oracle against outputs of the reference itself (tests/golden/*.npz)."""
import numpy as np
import pytest

from oracle import aoh_oracle as orc
from tests import golden_cases as gc
from aoh_b200 import synthetic as syn


def _oracle_cache(spec, labels):
    return orc.OracleKVCache(spec["layers"], labels, spec["sink"], spec["recent"], spec["dtype"])


def _oracle_step(cache, layer, q, k, v):
    return orc.layer_attention(cache, layer, q, k, v)


@pytest.mark.parametrize("name", gc.ATTN_CASES)
def test_oracle_attention_matches_reference(name):
    spec, got, ref, ck_ok = gc.replay(name, _oracle_cache, _oracle_step)
    assert ck_ok, "seeded input generator drifted from the one the fixture was made with"
    tol = gc.TOL[spec["dtype"]]
    # the oracle restates the reference's arithmetic; it should sit far inside the tolerance
    err = np.abs(got - ref).max()
    assert err <= (tol if spec["dtype"] == "bf16" else 2e-5), err


def test_bf16_round_matches_torch():
    import torch
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 3
    x[:4] = [0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8]  # ties
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(syn.bf16_round(x), want)
    assert np.array_equal(orc.bf16_round(x), want)


def test_streaming_cache_keeps_sink_and_recent():
    k = np.arange(20, dtype=np.float32).reshape(1, 1, 20, 1)
    ks, _ = orc.compress_stream(k, k, 3, 4)
    assert ks.ravel().tolist() == [0, 1, 2, 16, 17, 18, 19]
    assert orc.cached_positions(20, 7, 3).tolist() == [0, 1, 2, 16, 17, 18, 19]


def test_cache_rejects_negative_window():
    with pytest.raises(ValueError):
        orc.OracleKVCache(1, np.ones((1, 2)), -1, 4)

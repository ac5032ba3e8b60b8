"""The oracle against outputs of the reference itself (tests/golden/*.npz)."""
import numpy as np
import pytest

from oracle import aoh_oracle as orc
from tests import golden_cases as gc
from aoh_b200 import synthetic as syn


def _oracle_cache(spec, labels):
    return orc.OracleKVCache(spec["layers"], labels, spec["sink"], spec["recent"], spec["dtype"],
                             backend=spec.get("backend", "eager"))


def _oracle_step(cache, layer, q, k, v):
    return orc.layer_attention(cache, layer, q, k, v)


@pytest.mark.parametrize("name", gc.ATTN_CASES + gc.FLASH_CASES)
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


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_attend_rows_matches_layer_attention(dtype):
    """attend_rows (chosen query rows over a full key history, used for checks
    at full context sizes) agrees with the pinned layer_attention on every row
    of a chunked prefill, for both head kinds and windows the ring wraps past."""
    Hq, G, grp, sink, recent = 8, 2, 4, 16, 40
    labels = np.array([[1, 0]], dtype=np.float64)
    chunks = [100, 37, 64]
    T = sum(chunks)
    q, k, v = syn.attn_layer_inputs(5, 0, 1, T, Hq, G, 128, dtype=dtype)
    cache = orc.OracleKVCache(1, labels, sink, recent, dtype)
    s = 0
    for c in chunks:
        want = orc.layer_attention(cache, 0, q[:, s:s + c], k[:, s:s + c], v[:, s:s + c])
        for g in range(G):
            got = orc.attend_rows(q[0, s:s + c, g * grp:(g + 1) * grp], np.arange(s, s + c), k[0, :s + c, g],
                                  v[0, :s + c, g], labels[0, g] >= 0.5, sink, recent, dtype)
            ref = want[0, :, g * grp:(g + 1) * grp]
            # the same arithmetic over a shorter key range: BLAS may sum in
            # another order, so f32 agrees to rounding and bf16 to one ulp
            tol = 2e-6 + (2.0 ** -7 if dtype == "bf16" else 1e-5) * np.abs(ref)
            assert np.all(np.abs(got - ref) <= tol), (c, g, float(np.abs(got - ref).max()))
        s += c


def test_decode_unit_matches_decode_from_state():
    Hq, G, grp, T, sink, recent = 8, 2, 4, 700, 128, 256
    labels = np.array([1.0, 0.0])
    q, k, v = syn.attn_layer_inputs(6, 0, 1, T + 1, Hq, G, 128, dtype="bf16")
    want = orc.decode_from_state(q[:, T:], k[:, T:], v[:, T:], k[:, :T], v[:, :T], labels, T, sink, recent, "bf16")
    for g in range(G):
        if labels[g] >= 0.5:
            kc, vc = k[0, :T, g], v[0, :T, g]
        else:
            kc = np.concatenate([k[0, :sink, g], k[0, T - recent:T, g]])
            vc = np.concatenate([v[0, :sink, g], v[0, T - recent:T, g]])
        got = orc.decode_unit(q[0, T, g * grp:(g + 1) * grp], k[0, T, g], v[0, T, g], kc, vc, labels[g] >= 0.5, T,
                              sink, recent, "bf16")
        assert np.array_equal(got, want[0, 0, g * grp:(g + 1) * grp]), g

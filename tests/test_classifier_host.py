"""Host logic of the classifier (aggregation, labelling, file format) against
the reference's own outputs: fed the reference's per-head ranks, the labels
must be identical."""
import ast

import numpy as np
import pytest

from aoh_b200 import classifier as clf
from aoh_b200 import io as aio
from oracle import aoh_oracle as orc
from tests.golden_cases import GOLDEN

AGGS = ("mean", "min", "max")
SPS = (0.25, 0.5, 0.75)


@pytest.mark.parametrize("name", ["cls_small", "cls_qwen25_7b"])
@pytest.mark.parametrize("mode", ["fp32", "binary"])
def test_labels_from_reference_ranks_are_identical(name, mode):
    z = np.load(GOLDEN / f"{name}.npz")
    spec = ast.literal_eval(str(z["spec"]))
    ranks = z[f"{mode}_eff_ranks_q"]
    for agg in AGGS:
        kv = clf.aggregate_kv(ranks, spec["G"], agg)
        assert np.array_equal(kv, z[f"{mode}_{agg}_eff_ranks_kv"])
        for sp in SPS:
            assert np.array_equal(clf.labels_from_ranks(kv, sp), z[f"{mode}_{agg}_sp{sp}_labels"])
            c = clf.AoHClassifier(agg=agg)
            assert np.array_equal(c.classify_from_ranks(ranks, spec["G"], sp), z[f"{mode}_{agg}_sp{sp}_labels"])


def test_round_half_even_and_agg_validation():
    r = np.array([[3.0, 1.0, 2.0, 4.0]])
    # round(0.5 * 1)... G=4, sparsity 0.375 -> round(2.5) = 2 (banker's rounding)
    assert clf.labels_from_ranks(r, 0.375).tolist() == [[0, 1, 1, 0]]
    assert clf.labels_from_ranks(r, 1.0).sum() == 0
    assert clf.labels_from_ranks(r, 0.0).sum() == 4
    with pytest.raises(ValueError):
        clf.AoHClassifier(agg="median")
    with pytest.raises(RuntimeError):
        clf.AoHClassifier().save("/tmp/never")


def test_save_load_roundtrip_reference_format(tmp_path):
    z = np.load(GOLDEN / "cls_small.npz")
    c = clf.AoHClassifier(agg="min")
    c._info = {"num_layers": 2, "H": 8, "G": 2, "GRP": 4, "d_head": 128, "d_model": 512, "is_gqa": True}
    c.classify_from_ranks(z["fp32_eff_ranks_q"], 2, 0.5)
    c.save(str(tmp_path))
    assert sorted(p.name for p in tmp_path.iterdir()) == [
        "eff_rank.npy", "eff_rank_kv.npy", "head_classification.npy", "results.json"]
    back = clf.AoHClassifier.from_saved(str(tmp_path))
    assert np.array_equal(back.head_labels, c.head_labels)
    assert back.agg == "min" and back._info["is_gqa"] and back.sparsity == 0.5
    with pytest.raises(FileNotFoundError):
        aio.load_results(str(tmp_path / "missing"))


def test_label_margins():
    kv = np.array([[1.0, 2.0, 2.0, 5.0]])
    assert clf.label_margins(kv, 0.5)[0] == 0.0
    assert np.isinf(clf.label_margins(kv, 1.0)[0])

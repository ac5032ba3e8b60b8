"""GPU effective ranks and labels against the reference's outputs.

Effective ranks: within 1e-4 relative (observed ~1e-6: the reference's own
float32 eigvals noise).  Labels: every layer decision matches the reference's
bit for bit, except where the reference's own float32 ranks tie at the
retrieval/streaming boundary (gap within a few float32 ulps): there its label
is decided by its LAPACK build's rounding, which no other arithmetic
reproduces.  For the seed-0 Qwen2.5-7B-shaped case those decisions are pinned
exactly; for four more seeds each differing decision's gap is bounded and
printed."""
import ast

import numpy as np
import pytest
import torch

from aoh_b200 import classifier as clf
from aoh_b200 import synthetic as syn
from tests.golden_cases import GOLDEN

pytestmark = pytest.mark.gpu


def _weights(spec):
    L, Hq, G, D, dm, seed = (spec[k] for k in ("L", "Hq", "G", "D", "dm", "seed"))
    wq, wk = [], []
    for l in range(L):
        a, b = syn.classifier_weights(seed, l, Hq, G, D, dm)
        wq.append(torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16))
        wk.append(torch.from_numpy(b.astype(np.int16)).view(torch.bfloat16))
    return torch.stack(wq).cuda(), torch.stack(wk).cuda()


# The decisions of the seed-0 Qwen2.5-7B-shaped case that differ from the
# reference's: --binary mode, max aggregation, where the reference's own
# aggregated ranks tie in float32 at the retrieval/streaming boundary.
KNOWN_FLIPS = {"cls_qwen25_7b": {("binary", "max", 0.5, 12), ("binary", "max", 0.75, 9), ("binary", "max", 0.75, 12)}}
# The reference's float32 ranks deviate from exact ones by up to 1.3e-6 relative
# (measured against a float64 solve), so two of them closer than about twice
# that -- 22 float32 ulps -- can be ordered either way by its own rounding.
MAX_TIE_ULPS = 24


def boundary_ulps(kv_ranks: np.ndarray, sparsity: float) -> np.ndarray:
    """Per layer, the gap between the highest-ranked retrieval KV head and the
    lowest-ranked streaming one (the decision the label rests on) in float32
    ulps of the ranks; inf when every head has the same label."""
    L, G = kv_ranks.shape
    k = max(0, min(G, round((1.0 - sparsity) * G)))
    out = np.full(L, np.inf)
    if 0 < k < G:
        r = np.sort(kv_ranks, axis=1)
        out = (r[:, k] - r[:, k - 1]) / np.spacing(np.abs(r[:, k - 1]).astype(np.float32)).astype(np.float64)
    return out


@pytest.mark.parametrize("name", ["cls_small", "cls_qwen25_7b"] + [f"cls_qwen25_7b_s{s}" for s in (1, 2, 3, 4)])
@pytest.mark.parametrize("mode", ["fp32", "binary"])
def test_eff_ranks_and_labels(cuda_device, name, mode):
    """Ranks within 1e-4 relative of the reference's; every layer decision equal
    to the reference's except where the reference's own float32 ranks tie at
    the boundary (within MAX_TIE_ULPS) -- and, for the seed-0 case, exactly the
    known three."""
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"{name} fixture not generated")
    z = np.load(path)
    spec = ast.literal_eval(str(z["spec"]))
    wq, wk = _weights(spec)
    ranks = clf.eff_ranks_from_weights(wq, wk, spec["Hq"], spec["G"], spec["D"], binary=(mode == "binary"))
    ref = z[f"{mode}_eff_ranks_q"]
    assert np.all(np.abs(ranks - ref) <= 1e-4 * np.abs(ref))
    assert np.array_equal(ranks, ranks.astype(np.float32).astype(np.float64))  # float(fp32) values
    flips = {}
    for agg in ("mean", "min", "max"):
        kv = clf.aggregate_kv(ranks, spec["G"], agg)
        for sp in (0.25, 0.5, 0.75):
            lab = clf.labels_from_ranks(kv, sp)
            want = z[f"{mode}_{agg}_sp{sp}_labels"]
            ulps = boundary_ulps(z[f"{mode}_{agg}_eff_ranks_kv"], sp)
            for l in np.where((lab != want).any(axis=1))[0]:
                flips[(mode, agg, sp, int(l))] = float(ulps[l])
    print(f"{name} {mode}: differing decisions (reference boundary gap in float32 ulps): {flips}")
    for key, gap in flips.items():
        assert gap <= MAX_TIE_ULPS, (key, gap)
    if name in KNOWN_FLIPS:
        assert set(flips) == {f for f in KNOWN_FLIPS[name] if f[0] == mode}, flips


def test_classifier_api_on_stub_model(cuda_device):
    import types
    z = np.load(GOLDEN / "cls_small.npz")
    spec = ast.literal_eval(str(z["spec"]))
    wq, wk = _weights(spec)
    layers = [types.SimpleNamespace(self_attn=types.SimpleNamespace(
        q_proj=types.SimpleNamespace(weight=wq[l]), k_proj=types.SimpleNamespace(weight=wk[l])))
        for l in range(spec["L"])]
    cfg = types.SimpleNamespace(num_hidden_layers=spec["L"], num_attention_heads=spec["Hq"],
                                num_key_value_heads=spec["G"], hidden_size=spec["dm"], head_dim=spec["D"])
    model = types.SimpleNamespace(model=types.SimpleNamespace(layers=layers), config=cfg)
    c = clf.AoHClassifier(model=model, config=cfg, agg="mean")
    labels = c.classify(0.5)
    assert np.array_equal(labels, z["fp32_mean_sp0.5_labels"])
    r = clf.compute_eff_rank(wq[0, :128], wk[0, :128])
    assert abs(r - z["fp32_eff_ranks_q"][0, 0]) <= 1e-4 * r


@pytest.mark.parametrize("dm", [512, 320])
def test_binary_ranks_exact(cuda_device, dm):
    """Binary mode: the Gram matrices are sums of -1/0/+1 products, exact in
    integers -- on the integer tensor cores when d_model is a multiple of 128
    (512), in the SIMT kernel otherwise (320) -- so the effective ranks equal the
    oracle's float64 restatement (exact Grams, symmetric eigen-solve) to within
    one float32 ulp of the stored value.  Weights include exact zeros."""
    from oracle import aoh_oracle as orc

    L, Hq, G, D = 2, 8, 2, 128
    rng = np.random.default_rng(dm)
    w = rng.standard_normal((2, L, Hq * D, dm)).astype(np.float32)
    w[:, :, :, ::7] = 0.0  # sign(0) = 0 must contribute nothing
    wq = torch.from_numpy(w[0]).to(torch.bfloat16)
    wk = torch.from_numpy(w[1, :, :G * D]).to(torch.bfloat16)
    ranks = clf.eff_ranks_from_weights(wq.cuda(), wk.cuda(), Hq, G, D, binary=True)
    want = orc.compute_all_eff_ranks([x.float().numpy() for x in wq], [x.float().numpy() for x in wk], Hq, G, D,
                                     binary=True, exact=True)
    ulp = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(ranks - want) <= ulp), np.max(np.abs(ranks - want) / ulp)

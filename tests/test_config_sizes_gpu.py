"""CUDA path vs the oracle at the benchmark configurations' own sizes, through
the C ABI (aoh_attn_prefill / aoh_attn_decode / aoh_kv_append).

* Config 1 in full: Llama-3.1-8B heads (32 / 8), fp32, 4 of 8 KV heads
  streaming, RoPE theta 5e5, sixteen 256-token prefill chunks then 64 decode
  steps -- every output row against the oracle at the fp32 tolerance.
* Config 3 at 64K: Qwen2.5-7B heads (28 / 4, group 7), bf16, 2 of 4 KV heads
  streaming: the last 4096-token chunk over 61,440 cached tokens (the call the
  benchmark's prefill sample times) and the last 256-token chunk over 65,280
  cached tokens, on a sample of query rows (every 64th / 8th row and the first
  and last row of every 128-row block) against the oracle over the full key
  history.
* Config 4 at 256K: Qwen3-8B heads (32 / 8), bf16, batch 8, 262,144 cached
  tokens, retrieval heads skewed into KV groups 0-1: one decode layer, every
  (sequence, KV head) unit against the oracle.

Tolerances: 2e-2 absolute for bf16 outputs, 1e-4 for fp32."""
import numpy as np
import pytest
import torch

from aoh_b200 import AoHKVCache, aoh_attention
from aoh_b200 import synthetic as syn
from oracle import aoh_oracle as orc
from tests import gpu_engine as ge

pytestmark = pytest.mark.gpu

F = lambda t: t.float().cpu().numpy()  # noqa: E731


def test_config1_full_fp32(cuda_device):
    labels = syn.labels_uniform(1, 1, 8, 4)
    errs = ge.run_both("f32", 32, 8, labels, [256] * 16, 64, 128, 256, seed=1)
    assert errs["prefill"] <= 1e-4 and errs["decode"] <= 1e-4, errs


def _fill(cache, layer, k, v, upto, chunk=8192):
    """Append history rows [0, upto) straight into the pages."""
    for s in range(0, upto, chunk):
        e = min(upto, s + chunk)
        cache.kv_seq_len = s
        cache.append_layer(layer, k[:, s:e].contiguous(), v[:, s:e].contiguous())
    cache.kv_seq_len = upto


def _sample_rows(c, stride):
    rows = set(range(0, c, stride))
    for b0 in range(0, c, 128):
        rows.add(b0)
        rows.add(min(c, b0 + 128) - 1)
    return np.array(sorted(rows))


@pytest.mark.parametrize("past,chunk,stride", [(61440, 4096, 64), (65280, 256, 8)])
def test_config3_prefill_rows_at_64k(cuda_device, past, chunk, stride):
    Hq, G, D, sink, recent = 28, 4, 128, 128, 256
    grp = Hq // G
    labels = np.array([[1, 0, 1, 0]], dtype=np.float64)
    T = past + chunk
    gen = torch.Generator(device="cuda").manual_seed(2024 + chunk)
    k = torch.randn((1, T, G, D), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, T, G, D), generator=gen, device="cuda").to(torch.bfloat16)
    q = torch.randn((1, chunk, Hq, D), generator=gen, device="cuda").to(torch.bfloat16)
    cache = AoHKVCache(labels, Hq, sink_size=sink, recent_size=recent, max_context=T, dtype=torch.bfloat16)
    _fill(cache, 0, k, v, past)
    out = aoh_attention(cache, 0, q, k[:, past:].contiguous(), v[:, past:].contiguous())
    assert cache.device_status() == 0
    rows = _sample_rows(chunk, stride)
    got, qn, kn, vn = F(out[0, rows]), F(q[0, rows]), F(k[0]), F(v[0])
    worst = 0.0
    for g in range(G):
        heads = slice(g * grp, (g + 1) * grp)
        want = orc.attend_rows(qn[:, heads], past + rows, kn[:, g], vn[:, g], labels[0, g] >= 0.5, sink, recent,
                               "bf16")
        worst = max(worst, float(np.abs(got[:, heads] - want).max()))
    assert worst <= 2e-2, worst


def test_config4_batch8_256k_skewed_decode(cuda_device):
    Hq, G, B, D, T, sink, recent = 32, 8, 8, 128, 262144, 128, 256
    grp = Hq // G
    labels = syn.labels_skewed(0, 36, G, 6)[:1]  # layer 0 of the benchmark's skewed labels
    ret = [g for g in range(G) if labels[0, g] >= 0.5]
    cache = AoHKVCache(labels, Hq, batch=B, sink_size=sink, recent_size=recent, max_context=T + 1,
                       dtype=torch.bfloat16, reserve_all=True)
    gen = torch.Generator(device="cuda").manual_seed(4)
    # the oracle's state per unit: retrieval rows all kept (bf16 bits on the
    # host), streaming units only the sink and the last `recent` rows
    hist = {(kv, g): np.empty((B, T, D), dtype=np.int16) for kv in range(2) for g in ret}
    keep = {}
    chunk = 8192
    for s in range(0, T, chunk):
        kc = (torch.randn((B, chunk, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
        vc = (torch.randn((B, chunk, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
        cache.kv_seq_len = s
        cache.append_layer(0, kc, vc)
        for kv, t in ((0, kc), (1, vc)):
            for g in ret:
                hist[(kv, g)][:, s:s + chunk] = t[:, :, g].view(torch.int16).cpu().numpy()
            if s == 0:
                keep[(kv, "sink")] = F(t[:, :sink])
            if s + chunk == T:
                keep[(kv, "recent")] = F(t[:, chunk - recent:])
    cache.kv_seq_len = T
    q = torch.randn((B, 1, Hq, D), generator=gen, device="cuda").to(torch.bfloat16)
    kn = (torch.randn((B, 1, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    vn = (torch.randn((B, 1, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    got = F(aoh_attention(cache, 0, q, kn, vn))
    assert cache.device_status() == 0
    qn, knn, vnn = F(q), F(kn), F(vn)
    worst = 0.0
    for b in range(B):
        for g in range(G):
            if g in ret:
                kc = syn.bf16_to_f32(hist[(0, g)][b].view(np.uint16))
                vc = syn.bf16_to_f32(hist[(1, g)][b].view(np.uint16))
            else:
                kc = np.concatenate([keep[(0, "sink")][b, :, g], keep[(0, "recent")][b, :, g]])
                vc = np.concatenate([keep[(1, "sink")][b, :, g], keep[(1, "recent")][b, :, g]])
            want = orc.decode_unit(qn[b, 0, g * grp:(g + 1) * grp], knn[b, 0, g], vnn[b, 0, g], kc, vc, g in ret, T,
                                   sink, recent, "bf16")
            worst = max(worst, float(np.abs(got[b, 0, g * grp:(g + 1) * grp] - want).max()))
    assert worst <= 2e-2, worst
    assert cache.kv_seq_len == T + 1


def test_decode_group7_batch8_clusters_of_4(cuda_device):
    """Qwen2.5-7B heads (28 / 4, group 7), batch 8, every KV head retrieval,
    16,384 cached tokens: 32 split units, which the plan runs in clusters of 4
    (clusters of 8 would leave fewer than 2 streaming CTAs per SM).  A
    cluster CTA's output slice (7 x 128 / 4 = 224 outputs) is longer than the
    CTA, so its threads combine two outputs each.  Every unit against the oracle."""
    Hq, G, B, D, T, sink, recent = 28, 4, 8, 128, 16384, 128, 256
    grp = Hq // G
    labels = np.ones((1, G), dtype=np.float64)
    cache = AoHKVCache(labels, Hq, batch=B, sink_size=sink, recent_size=recent, max_context=T + 1,
                       dtype=torch.bfloat16, reserve_all=True)
    gen = torch.Generator(device="cuda").manual_seed(11)
    k = (torch.randn((B, T, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, T, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    _fill(cache, 0, k, v, T)
    q = torch.randn((B, 1, Hq, D), generator=gen, device="cuda").to(torch.bfloat16)
    kn = (torch.randn((B, 1, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    vn = (torch.randn((B, 1, G, D), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    got = F(aoh_attention(cache, 0, q, kn, vn))
    assert cache.device_status() == 0
    qn, knn, vnn, kc, vc = F(q), F(kn), F(vn), F(k), F(v)
    worst = 0.0
    for b in range(B):
        for g in range(G):
            want = orc.decode_unit(qn[b, 0, g * grp:(g + 1) * grp], knn[b, 0, g], vnn[b, 0, g], kc[b, :, g],
                                   vc[b, :, g], True, T, sink, recent, "bf16")
            worst = max(worst, float(np.abs(got[b, 0, g * grp:(g + 1) * grp] - want).max()))
    assert worst <= 2e-2, worst

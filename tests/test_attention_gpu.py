"""CUDA attention path vs the reference's outputs (golden fixtures) and vs the
oracle on seeded inputs, through the C ABI (aoh_attn_prefill / aoh_attn_decode).

Tolerances: 2e-2 absolute for bf16, 1e-4 for float32."""
import numpy as np
import pytest
import torch

from aoh_b200 import AoHKVCache, aoh_attention
from aoh_b200 import synthetic as syn
from oracle import aoh_oracle as orc
from tests import golden_cases as gc
from tests import gpu_engine as ge

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", gc.ATTN_CASES)
def test_golden_cases(cuda_device, name):
    spec, got, ref, ck_ok = gc.replay(name, ge.make_cache, ge.step)
    assert ck_ok
    tol = gc.TOL[spec["dtype"]]
    err = np.abs(got - ref).max()
    assert err <= tol, f"{name}: max abs err {err} > {tol}"


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_llama_shapes_against_oracle(cuda_device, dtype):
    labels = syn.labels_uniform(3, 2, 8, 6)
    errs = ge.run_both(dtype, 32, 8, labels, [256, 256, 300], 5, 128, 256, seed=21)
    tol = gc.TOL[dtype]
    assert errs["prefill"] <= tol and errs["decode"] <= tol, errs


def test_qwen25_group7_batch2(cuda_device):
    labels = np.array([[1, 0, 0, 1], [0, 0, 0, 1]], dtype=np.float64)
    errs = ge.run_both("bf16", 28, 4, labels, [200, 77], 4, 128, 256, seed=22, batch=2)
    assert max(errs.values()) <= 2e-2, errs


@pytest.mark.parametrize("Hq,labels_row", [(8, [1, 0]), (14, [0, 1])])
def test_split_kv_prefill_against_oracle(cuda_device, Hq, labels_row):
    """Chunks whose retrieval CTAs are cut into key ranges (split-KV + combine):
    a long first chunk (row blocks with fewer key tiles than splits, so some
    ranges are empty), then short chunks over a long cache; group sizes 4 (head
    pairs) and 7 (pairs plus a single-head CTA)."""
    labels = np.array([labels_row], dtype=np.float64)
    errs = ge.run_both("bf16", Hq, 2, labels, [3000, 2500, 256, 200, 129], 2, 128, 256, seed=24)
    assert max(errs.values()) <= 2e-2, errs


@pytest.mark.parametrize("sink,recent", [(0, 0), (0, 40), (7, 0), (16, 16), (130, 250)])
def test_window_edge_cases(cuda_device, sink, recent):
    labels = np.array([[0, 1]], dtype=np.float64)
    for dtype in ("f32", "bf16"):
        errs = ge.run_both(dtype, 8, 2, labels, [37, 64, 5], 6, sink, recent, seed=23)
        assert max(errs.values()) <= gc.TOL[dtype], (dtype, errs)


def test_decode_from_empty_cache(cuda_device):
    # past_len = 0: every head attends to the new key only
    labels = np.array([[1, 0]], dtype=np.float64)
    errs = ge.run_both("bf16", 8, 2, labels, [], 3, 128, 256, seed=24)
    assert errs["decode"] <= 2e-2


@pytest.mark.parametrize("name", gc.FLASH_CASES)
def test_flash_protocol_golden_cases(cuda_device, name):
    """The decoding-simulation protocol (the prompt in one call, every head
    causal over it, then decode steps) against the reference's FlashAttention-2
    path on the same inputs."""
    spec, got, ref, ck_ok = gc.replay(name, ge.make_cache, ge.step)
    assert ck_ok
    err = np.abs(got - ref).max()
    assert err <= gc.TOL[spec["dtype"]], f"{name}: max abs err {err}"


def test_flash_protocol_rejects_a_second_prompt_call(cuda_device):
    labels = np.array([[1, 0]], dtype=np.float64)
    cache = AoHKVCache(labels, 8, max_context=64, dtype=torch.bfloat16, backend="flash")
    q = torch.zeros((1, 8, 8, 128), dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros((1, 8, 2, 128), dtype=torch.bfloat16, device="cuda")
    aoh_attention(cache, 0, q, kv, kv)
    with pytest.raises(NotImplementedError):
        aoh_attention(cache, 0, q, kv, kv)  # a multi-token call over a non-empty cache
    aoh_attention(cache, 0, q[:, :1], kv[:, :1], kv[:, :1])  # decode steps follow the prompt
    assert cache.kv_seq_len == 9 and cache.device_status() == 0


def _fill_cache_bf16(cache, layer, k_ctx, v_ctx, chunk=8192):
    """Write a context straight into the pages (AoHKVCache.append_layer)."""
    T = k_ctx.shape[1]
    for s in range(0, T, chunk):
        e = min(T, s + chunk)
        cache.kv_seq_len = s
        cache.append_layer(layer, k_ctx[:, s:e].contiguous(), v_ctx[:, s:e].contiguous())
    cache.kv_seq_len = T


@pytest.mark.parametrize("T", [4096 + 7, 131072])
def test_long_context_decode_against_oracle(cuda_device, T):
    """One decode step of a Llama-3.1-8B-shaped layer over a T-token paged
    context (75% streaming heads), against the oracle on the same data."""
    Hq, G, B = 32, 8, 1
    labels = syn.labels_uniform(5, 1, G, 6)
    gen = torch.Generator(device="cuda").manual_seed(1234)
    k_ctx = (torch.randn((B, T, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    v_ctx = (torch.randn((B, T, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    q = torch.randn((B, 1, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
    kn = (torch.randn((B, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    vn = (torch.randn((B, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    cache = AoHKVCache(labels, Hq, batch=B, max_context=T + 2, dtype=torch.bfloat16)
    _fill_cache_bf16(cache, 0, k_ctx, v_ctx)
    out = aoh_attention(cache, 0, q, kn, vn)
    got = out.float().cpu().numpy()
    f = lambda t: t.float().cpu().numpy()
    want = orc.decode_from_state(f(q), f(kn), f(vn), f(k_ctx), f(v_ctx), labels[0], T, 128, 256, "bf16")
    err = np.abs(got - want).max()
    assert err <= 2e-2, err
    assert cache.kv_seq_len == T + 1
    assert cache.device_status() == 0
    # the new token was appended at position T: a second step sees it
    q2 = torch.randn((B, 1, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
    cache2_k = torch.cat([k_ctx, kn], 1)
    cache2_v = torch.cat([v_ctx, vn], 1)
    kn2 = (torch.randn((B, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    vn2 = (torch.randn((B, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    got2 = aoh_attention(cache, 0, q2, kn2, vn2).float().cpu().numpy()
    want2 = orc.decode_from_state(f(q2), f(kn2), f(vn2), f(cache2_k), f(cache2_v), labels[0], T + 1, 128, 256,
                                  "bf16")
    assert np.abs(got2 - want2).max() <= 2e-2


def test_streaming_heads_touch_only_their_pages(cuda_device):
    """A streaming unit owns sink + ring pages only; poisoning every other page
    of the pool must not change its output."""
    Hq, G, T = 8, 2, 3000
    labels = np.array([[0, 0]], dtype=np.float64)
    gen = torch.Generator(device="cuda").manual_seed(7)
    k_ctx = (torch.randn((1, T, G, 128), generator=gen, device="cuda")).to(torch.bfloat16)
    v_ctx = (torch.randn((1, T, G, 128), generator=gen, device="cuda")).to(torch.bfloat16)
    cache = AoHKVCache(labels, Hq, batch=1, max_context=T + 1, dtype=torch.bfloat16)
    assert cache.num_pages == 2 * (8 + 16)
    _fill_cache_bf16(cache, 0, k_ctx, v_ctx, chunk=1000)
    q = torch.randn((1, 1, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
    kn = torch.randn((1, 1, G, 128), generator=gen, device="cuda").to(torch.bfloat16)
    out = aoh_attention(cache, 0, q, kn, kn, advance=False).float().cpu().numpy()
    f = lambda t: t.float().cpu().numpy()
    want = orc.decode_from_state(f(q), f(kn), f(kn), f(k_ctx), f(v_ctx), labels[0], T, 128, 256, "bf16")
    assert np.abs(out - want).max() <= 2e-2


def test_bad_arguments_raise(cuda_device):
    labels = np.array([[1, 0]], dtype=np.float64)
    cache = AoHKVCache(labels, 8, max_context=64, dtype=torch.bfloat16)
    q = torch.zeros((1, 1, 8, 128), dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros((1, 1, 2, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        aoh_attention(cache, 1, q, kv, kv)
    with pytest.raises(ValueError):
        aoh_attention(cache, 0, q.float(), kv, kv)
    cache.kv_seq_len = 64
    with pytest.raises(torch.OutOfMemoryError):
        aoh_attention(cache, 0, q, kv, kv)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_append_layout_roundtrip(cuda_device, dtype):
    """aoh_kv_append writes rows where aoh_kv_locate says they are, in the
    documented page layout (pre-swizzled for bf16), for both head kinds."""
    labels = np.array([[1, 0]], dtype=np.float64)
    sink, recent, T = 20, 40, 137
    cache = AoHKVCache(labels, 4, batch=2, sink_size=sink, recent_size=recent, max_context=T, dtype=dtype)
    gen = torch.Generator(device="cuda").manual_seed(5)
    k = torch.randn((2, T, 2, 128), generator=gen, device="cuda").to(dtype)
    v = torch.randn((2, T, 2, 128), generator=gen, device="cuda").to(dtype)
    for s in range(0, T, 50):
        e = min(T, s + 50)
        cache.kv_seq_len = s
        cache.append_layer(0, k[:, s:e].contiguous(), v[:, s:e].contiguous())
    cache.kv_seq_len = T
    for seq in range(2):
        ret_pos = list(range(T))
        kk, vv = cache.read_rows(0, seq, 0, ret_pos)
        assert torch.equal(kk, k[seq, :, 0]) and torch.equal(vv, v[seq, :, 0])
        ring = (recent + 15) // 16 * 16
        str_pos = list(range(sink)) + list(range(T - ring, T))
        kk, vv = cache.read_rows(0, seq, 1, str_pos)
        assert torch.equal(kk, k[seq, str_pos, 1]) and torch.equal(vv, v[seq, str_pos, 1])
        assert cache.locate(0, seq, 1, sink + 1) == (-1, -1)  # evicted
    assert cache.device_status() == 0


@pytest.mark.parametrize("Hq,labels_row", [(4, [1, 0]), (14, [0, 1]), (2, [1, 0])])
def test_prefill_append_layout(cuda_device, Hq, labels_row):
    """The bf16 prefill kernel appends its chunk's rows itself (retrieval rows
    from the two-head CTAs' spare warp, or the one-head CTAs' when the group has
    one head; streaming sink and ring rows from the unit's last CTA).  After
    every chunk -- starts off the page grid, across the sink boundary, past ring
    wraps, a split-KV chunk over a long cache -- every held row equals its
    input bit for bit, for group sizes 2, 7 and 1."""
    labels = np.array([labels_row], dtype=np.float64)
    sink, recent = 20, 40
    chunks = [100, 37, 200, 300, 1500, 256, 129]
    T = sum(chunks)
    cache = AoHKVCache(labels, Hq, batch=2, sink_size=sink, recent_size=recent, max_context=T, dtype=torch.bfloat16)
    gen = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn((2, T, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn((2, T, 2, 128), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((2, T, 2, 128), generator=gen, device="cuda").to(torch.bfloat16)
    ring = (recent + 15) // 16 * 16
    s = 0
    for c in chunks:
        aoh_attention(cache, 0, q[:, s:s + c].contiguous(), k[:, s:s + c].contiguous(), v[:, s:s + c].contiguous())
        s += c
        for seq in range(2):
            for g in range(2):
                if labels_row[g]:
                    pos = list(range(s))
                else:
                    pos = list(range(min(sink, s))) + list(range(max(sink, s - ring), s))
                kk, vv = cache.read_rows(0, seq, g, pos)
                assert torch.equal(kk, k[seq, pos, g]) and torch.equal(vv, v[seq, pos, g]), (c, seq, g)
    assert cache.device_status() == 0


def test_graph_decode_matches_eager_and_oracle(cuda_device):
    """Decode steps replayed from a CUDA graph (device-resident length,
    programmatic dependent launch between layers) equal the eager path and the
    oracle, and the cache advances exactly as the reference's does."""
    from aoh_b200.graph import DecodeStepGraph
    Hq, G, L, T, steps = 32, 8, 3, 3000, 4
    labels = syn.labels_uniform(9, L, G, 6)
    gen = torch.Generator(device="cuda").manual_seed(11)
    k_ctx = [(torch.randn((1, T, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16) for _ in range(L)]
    v_ctx = [(torch.randn((1, T, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16) for _ in range(L)]
    caches = []
    for _ in range(2):
        c = AoHKVCache(labels, Hq, max_context=T + steps + 8, dtype=torch.bfloat16)
        for l in range(L):
            _fill_cache_bf16(c, l, k_ctx[l], v_ctx[l], chunk=1024)
        caches.append(c)
    eager, graphed = caches
    qs = [torch.randn((L, 1, 1, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16) for _ in range(steps)]
    ks = [(torch.randn((L, 1, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16) for _ in range(steps)]
    vs = [(torch.randn((L, 1, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16) for _ in range(steps)]
    qb, kb, vb = qs[0].clone(), ks[0].clone(), vs[0].clone()
    ob = torch.empty_like(qb)
    g = DecodeStepGraph(graphed, qb, kb, vb, ob, max_steps=steps)
    # the graph's uncaptured first launch is a dry run: it appended nothing, so
    # each streaming unit's oldest window row (the ring slot an append at T
    # would take) still equals the eager cache's
    for l in range(L):
        for kv in range(G):
            if labels[l, kv] < 0.5:
                a = graphed.read_rows(l, 0, kv, [T - 256, T - 1])
                b = eager.read_rows(l, 0, kv, [T - 256, T - 1])
                assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), (l, kv)
    f = lambda t: t.float().cpu().numpy()
    for s in range(steps):
        want = torch.stack([aoh_attention(eager, l, qs[s][l], ks[s][l], vs[s][l]) for l in range(L)])
        qb.copy_(qs[s]); kb.copy_(ks[s]); vb.copy_(vs[s])
        g.replay()
        got = ob.clone()
        assert torch.allclose(got.float(), want.float(), atol=2e-2, rtol=0)
        # oracle for layer 0 at this step
        kk = torch.cat([k_ctx[0]] + [ks[j][0] for j in range(s)], 1)
        vv = torch.cat([v_ctx[0]] + [vs[j][0] for j in range(s)], 1)
        ref = orc.decode_from_state(f(qs[s][0]), f(ks[s][0]), f(vs[s][0]), f(kk), f(vv), labels[0], T + s,
                                    128, 256, "bf16")
        assert np.abs(f(got[0]) - ref).max() <= 2e-2
    assert graphed.kv_seq_len == eager.kv_seq_len == T + steps
    assert graphed.device_status() == 0 and eager.device_status() == 0


def test_prefill_partitioned_cache(cuda_device):
    """A cache holding only some units (as one rank's share of the multi-GPU
    partition): the prefill appends exactly the owned units' rows, touches no
    other unit (such a write would trip the device check word), and the owned
    heads' outputs match a cache that holds every unit."""
    labels = np.array([[1, 0]], dtype=np.float64)
    Hq, grp, sink, recent = 14, 7, 20, 40
    owned = np.array([[[1, 0], [0, 1]]], dtype=np.uint8)  # seq 0: retrieval group, seq 1: streaming group
    chunks = [100, 37, 200, 1500, 256]
    T = sum(chunks)
    kw = dict(batch=2, sink_size=sink, recent_size=recent, max_context=T, dtype=torch.bfloat16)
    part = AoHKVCache(labels, Hq, owned=owned, **kw)
    full = AoHKVCache(labels, Hq, **kw)
    gen = torch.Generator(device="cuda").manual_seed(10)
    q = torch.randn((2, T, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn((2, T, 2, 128), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((2, T, 2, 128), generator=gen, device="cuda").to(torch.bfloat16)
    ring = (recent + 15) // 16 * 16
    s = 0
    for c in chunks:
        args = [x[:, s:s + c].contiguous() for x in (q, k, v)]
        got = aoh_attention(part, 0, *args)
        want = aoh_attention(full, 0, *args)
        s += c
        for seq, g in ((0, 0), (1, 1)):
            heads = slice(g * grp, (g + 1) * grp)
            err = (got[seq, :, heads].float() - want[seq, :, heads].float()).abs().max().item()
            assert err <= 2e-2, (c, seq, g, err)
            pos = list(range(s)) if labels[0, g] else list(range(min(sink, s))) + list(range(max(sink, s - ring), s))
            kk, vv = part.read_rows(0, seq, g, pos)
            assert torch.equal(kk, k[seq, pos, g]) and torch.equal(vv, v[seq, pos, g]), (c, seq, g)
    assert part.device_status() == 0 and full.device_status() == 0


def test_softmax_exp2_polynomial(cuda_device):
    """The prefill softmax computes 3 of every 8 exponentials with a cubic on
    the FMA pipe instead of the MUFU.  Against an exact float64 2^x: over
    [-125, 8] its relative error stays below 7.6e-5 -- under half a bf16 ulp
    of P, which is rounded to bf16 next -- and the bf16 rounding of its result
    is within one bf16 ulp of the rounded exact value; below -125, where the
    result sits at the bottom of the normal range (x is clamped to -126), the
    absolute error stays under 2^-138, nothing next to a row sum of at least 1."""
    import ctypes as C

    from aoh_b200 import _lib
    xs = np.concatenate([np.linspace(-126.0, 8.0, 2_000_001), np.arange(-126, 9, dtype=np.float64),
                         np.arange(-126, 8, dtype=np.float64) + 0.5]).astype(np.float32)
    x = torch.from_numpy(xs).cuda()
    out = torch.empty_like(x)
    _lib.check(_lib.lib().aoh_diag_exp2_poly(C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), x.numel(),
                                             C.c_void_p(_lib.stream_handle())), "aoh_diag_exp2_poly")
    got = out.cpu().numpy().astype(np.float64)
    want = np.exp2(xs.astype(np.float64))
    m = xs >= -125
    rel = np.abs(got[m] - want[m]) / want[m]
    assert rel.max() < 7.6e-5, (float(rel.max()), float(xs[m][np.argmax(rel)]))
    assert np.abs(got[~m] - want[~m]).max() < 2.0 ** -138
    gb = syn.bf16_round(got[m].astype(np.float32)).astype(np.float64)
    wb = syn.bf16_round(want[m].astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(gb - wb) <= np.spacing(wb.astype(np.float32)).astype(np.float64) * 65536)

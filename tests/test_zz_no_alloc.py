"""aoh_attn_decode_noalloc: the decode entry point for callers that cannot
allocate device memory -- plugin hosts that give an op only its input and
output buffers, and runtimes that may not allocate after start-up.  Its
split-KV scratch is a static device array inside libaoh.so instead of a
caller-owned workspace.

Checked through the C ABI against aoh_attn_decode (same cache contents, same
inputs) on two consecutive decode steps, at the bf16 tolerance of the other
attention tests.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

from aoh_b200 import AoHKVCache, _lib
from aoh_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_decode_matches_workspace_decode(cuda_device):
    Hq, G, T = 32, 8, 20000
    labels = syn.labels_uniform(21, 1, G, 6)
    gen = torch.Generator(device="cuda").manual_seed(42)
    ref = AoHKVCache(labels, Hq, max_context=T + 4, dtype=torch.bfloat16, reserve_all=True)
    tst = AoHKVCache(labels, Hq, max_context=T + 4, dtype=torch.bfloat16, reserve_all=True)
    pv = ref.pool_view()
    pv.copy_((torch.randn(pv.shape, generator=gen, device="cuda") * 0.5).to(torch.bfloat16))
    tst.pool.copy_(ref.pool)
    assert ref.unit_pages(0, 0, 0) == tst.unit_pages(0, 0, 0)  # same page ids: same layout
    ref.kv_seq_len = tst.kv_seq_len = T
    lib = _lib.lib()
    ws = ref.decode_workspace()
    st = C.c_void_p(_lib.stream_handle())
    for _ in range(2):
        q = torch.randn((1, 1, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
        k = (torch.randn((1, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
        v = (torch.randn((1, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
        want = torch.full_like(q, float("nan"))
        got = torch.full_like(q, float("nan"))
        _lib.check(lib.aoh_attn_decode(ref._h, 0, ref.kv_seq_len, _p(q), _p(k), _p(v), _p(want), _p(ws),
                                       ws.numel(), st), "aoh_attn_decode")
        _lib.check(lib.aoh_attn_decode_noalloc(tst._h, 0, tst.kv_seq_len, _p(q), _p(k), _p(v), _p(got), st),
                   "aoh_attn_decode_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert torch.allclose(got.float(), want.float(), atol=2e-2, rtol=0)
        ref.kv_seq_len += 1
        tst.kv_seq_len += 1
    assert ref.device_status() == 0 and tst.device_status() == 0
    assert torch.equal(ref.pool, tst.pool)  # both appended the same two tokens in the same slots


def test_noalloc_rejects_layers_beyond_its_scratch(cuda_device):
    # 33 sequences x 8 KV heads = 264 units > the 256 tickets of the static scratch
    labels = np.zeros((1, 8))
    cache = AoHKVCache(labels, 8, batch=33, sink_size=16, recent_size=16, max_context=64, dtype=torch.bfloat16)
    q = torch.zeros((33, 1, 8, 128), dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros((33, 1, 8, 128), dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib().aoh_attn_decode_noalloc(cache._h, 0, 0, _p(q), _p(kv), _p(kv), _p(q),
                                           C.c_void_p(_lib.stream_handle()))
    assert rc == _lib.UNSUPPORTED
    assert b"static scratch" in _lib.lib().aoh_last_error()


def test_noalloc_partitioned_cache_and_device_length(cuda_device):
    """A cache holding only some units (one rank's share of the multi-GPU
    partition, no peers attached), decoded with the length read from the
    device (AOH_PAST_LEN_DEVICE, the mode a replayed decode step uses): the
    owned heads match aoh_attn_decode on the same cache contents, on two
    consecutive steps."""
    Hq, G, B, T = 28, 4, 2, 9000
    grp = Hq // G
    labels = np.array([[1, 0, 1, 0]], dtype=np.float64)
    owned = np.zeros((1, B, G), dtype=np.uint8)
    owned[0, 0, [0, 1]] = 1  # sequence 0: a retrieval and a streaming group
    owned[0, 1, [2]] = 1     # sequence 1: a retrieval group
    gen = torch.Generator(device="cuda").manual_seed(43)
    kw = dict(batch=B, max_context=T + 4, dtype=torch.bfloat16, owned=owned, reserve_all=True)
    ref = AoHKVCache(labels, Hq, **kw)
    tst = AoHKVCache(labels, Hq, **kw)
    pv = ref.pool_view()
    pv.copy_((torch.randn(pv.shape, generator=gen, device="cuda") * 0.5).to(torch.bfloat16))
    tst.pool.copy_(ref.pool)
    lib = _lib.lib()
    st = C.c_void_p(_lib.stream_handle())
    _lib.check(lib.aoh_kv_set_length(tst._h, T, st), "aoh_kv_set_length")
    ws = ref.decode_workspace()
    for step in range(2):
        q = torch.randn((B, 1, Hq, 128), generator=gen, device="cuda").to(torch.bfloat16)
        k = (torch.randn((B, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
        v = (torch.randn((B, 1, G, 128), generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
        want = torch.full_like(q, float("nan"))
        got = torch.full_like(q, float("nan"))
        _lib.check(lib.aoh_attn_decode(ref._h, 0, T + step, _p(q), _p(k), _p(v), _p(want), _p(ws), ws.numel(), st),
                   "aoh_attn_decode")
        _lib.check(lib.aoh_attn_decode_noalloc(tst._h, 0, _lib.PAST_LEN_DEVICE, _p(q), _p(k), _p(v), _p(got), st),
                   "aoh_attn_decode_noalloc")
        _lib.check(lib.aoh_kv_advance(tst._h, 1, st), "aoh_kv_advance")
        torch.cuda.synchronize()
        for b in range(B):
            for g in range(G):
                heads = slice(g * grp, (g + 1) * grp)
                if owned[0, b, g]:
                    assert torch.isfinite(got[b, :, heads].float()).all()
                    assert torch.allclose(got[b, :, heads].float(), want[b, :, heads].float(), atol=2e-2, rtol=0)
                else:  # units stored elsewhere are not computed here
                    assert torch.isnan(got[b, :, heads].float()).all()
    assert ref.device_status() == 0 and tst.device_status() == 0
    assert torch.equal(ref.pool, tst.pool)

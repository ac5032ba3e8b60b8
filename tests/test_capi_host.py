"""C ABI checks that need no GPU: every symbol of include/aoh.h is exported,
and the host-side cache bookkeeping / partition behave as specified."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from aoh_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    txt = (ROOT / "include" / "aoh.h").read_text()
    return sorted(set(re.findall(r"AOH_API [^;(]*?\b(aoh_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _declared_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(L, name), name
    assert sorted(_lib.exported_symbols()) == declared
    assert L.aoh_abi_version() == _lib.ABI_VERSION


def _cfg(labels, batch=1, hq=8, sink=128, recent=256, max_ctx=1024, pages=None, owned=None, dtype=_lib.BF16):
    labels = np.ascontiguousarray(labels, dtype=np.uint8)
    L, G = labels.shape
    if pages is None:
        n_ret = int(labels.sum()) * batch
        n_str = (labels.size - int(labels.sum())) * batch
        pages = n_ret * (-(-max_ctx // 16)) + n_str * (-(-sink // 16) - (-recent // 16))
    own_p = None
    if owned is not None:
        owned = np.ascontiguousarray(owned, dtype=np.uint8)
        own_p = owned.ctypes.data_as(C.POINTER(C.c_uint8))
    cfg = _lib.KVConfig(L, batch, hq, G, 128, 16, dtype, sink, recent, max_ctx, pages,
                        labels.ctypes.data_as(C.POINTER(C.c_uint8)), own_p)
    return cfg, (labels, owned)


def _create(cfg):
    h = C.c_void_p()
    rc = _lib.lib().aoh_kv_create(C.byref(cfg), C.byref(h))
    return rc, h


def test_create_validates_arguments():
    L = _lib.lib()
    cfg, keep = _cfg([[1, 0]], sink=-1)
    rc, _ = _create(cfg)
    assert rc == _lib.INVALID and b"non-negative" in L.aoh_last_error()
    cfg, keep = _cfg([[1, 0]])
    cfg.head_dim = 64
    assert _create(cfg)[0] == _lib.UNSUPPORTED
    cfg, keep = _cfg([[1, 0]], hq=7)
    assert _create(cfg)[0] == _lib.INVALID
    cfg, keep = _cfg([[2, 0]])
    assert _create(cfg)[0] == _lib.INVALID
    cfg, keep = _cfg([[1, 0]], pages=3)  # streaming needs 8 + 16 pages
    assert _create(cfg)[0] == _lib.OUT_OF_PAGES


def test_paging_reserve_release_and_row_offsets():
    L = _lib.lib()
    labels = np.array([[1, 0, 1, 0], [0, 0, 1, 1]])
    cfg, keep = _cfg(labels, batch=2, max_ctx=100, sink=20, recent=40)
    rc, h = _create(cfg)
    assert rc == 0
    total = cfg.num_pages
    str_pages = 2 + 3  # ceil(20/16) + ceil(40/16)
    n_str_units = 4 * 2
    assert L.aoh_kv_free_pages(h) == total - n_str_units * str_pages
    # reserve 33 tokens -> 3 pages per retrieval unit (4 retrieval units x 2 seqs)
    assert L.aoh_kv_reserve(h, -1, 33) == 0
    assert L.aoh_kv_free_pages(h) == total - n_str_units * str_pages - 8 * 3
    n = C.c_int32()
    buf = (C.c_int32 * 16)()
    assert L.aoh_kv_unit_pages(h, 0, 1, 0, buf, 16, C.byref(n)) == 0 and n.value == 3
    pages = list(buf[:3])
    assert len(set(pages)) == 3
    def locate(layer, seq, g, pos, past):
        pg, sl = C.c_int32(), C.c_int32()
        assert L.aoh_kv_locate(h, layer, seq, g, pos, past, C.byref(pg), C.byref(sl)) == 0
        return pg.value, sl.value
    # retrieval: position 17 -> page 1, slot 1
    assert locate(0, 1, 0, 17, 33) == (pages[1], 1)
    assert locate(0, 1, 0, 40, 33) == (-1, -1)  # not yet cached
    # streaming ring: sink 20 -> positions < 20 in sink pages; position 95 of a 96-token context
    assert L.aoh_kv_unit_pages(h, 0, 0, 1, buf, 16, C.byref(n)) == 0 and n.value == str_pages
    sp = list(buf[:str_pages])
    r = (95 - 20) % 48
    assert locate(0, 0, 1, 95, 96) == (sp[2 + r // 16], r % 16)
    assert locate(0, 0, 1, 19, 96) == (sp[1], 3)
    assert locate(0, 0, 1, 30, 96) == (-1, -1)  # evicted (older than the ring)
    # exceeding max_context and exhausting the pool
    assert L.aoh_kv_reserve(h, -1, 101) == _lib.OUT_OF_PAGES
    assert L.aoh_kv_release(h, 1) == 0
    assert L.aoh_kv_free_pages(h) == total - n_str_units * str_pages - 4 * 3
    # tables are host-only until bound
    assert L.aoh_kv_sync(h, None) == _lib.STATE
    L.aoh_kv_destroy(h)


def test_pool_exhaustion_is_reported_and_consistent():
    L = _lib.lib()
    cfg, keep = _cfg([[1, 1]], max_ctx=1024, pages=10, sink=0, recent=0)
    rc, h = _create(cfg)
    assert rc == 0
    assert L.aoh_kv_reserve(h, -1, 16 * 5) == 0
    assert L.aoh_kv_reserve(h, -1, 16 * 6) == _lib.OUT_OF_PAGES
    assert b"exhausted" in L.aoh_last_error()
    assert L.aoh_kv_free_pages(h) == 0
    L.aoh_kv_destroy(h)


def test_owned_mask_limits_pages():
    L = _lib.lib()
    labels = np.array([[1, 0]])
    owned = np.array([[[1, 0]]])
    cfg, keep = _cfg(labels, owned=owned, max_ctx=64, pages=4)
    rc, h = _create(cfg)
    assert rc == 0
    assert L.aoh_kv_reserve(h, -1, 64) == 0
    n = C.c_int32()
    assert L.aoh_kv_unit_pages(h, 0, 0, 1, None, 0, C.byref(n)) == 0 and n.value == 0
    L.aoh_kv_destroy(h)


def test_partition_balances_touched_tokens():
    L = _lib.lib()
    labels = np.ascontiguousarray([[1, 1, 0, 0, 0, 0, 0, 0]], dtype=np.uint8)
    B, G, ctx = 8, 8, 262144
    for ranks in (1, 2, 4, 8):
        out = np.zeros((1, B, G), dtype=np.int32)
        rc = L.aoh_partition(labels.ctypes.data_as(C.POINTER(C.c_uint8)), 1, B, G, ctx, 128, 256, ranks,
                             out.ctypes.data_as(C.POINTER(C.c_int32)))
        assert rc == 0
        heavy = np.bincount(out[0][:, :2].ravel(), minlength=ranks)
        assert heavy.max() - heavy.min() <= 1  # 16 retrieval units spread evenly
        assert set(np.unique(out)) == set(range(ranks))
    bad = np.ascontiguousarray([[3]], dtype=np.uint8)
    out = np.zeros(1, dtype=np.int32)
    assert L.aoh_partition(bad.ctypes.data_as(C.POINTER(C.c_uint8)), 1, 1, 1, 10, 1, 1, 2,
                           out.ctypes.data_as(C.POINTER(C.c_int32))) == _lib.INVALID


def test_gather_entry_points_validate_arguments():
    """Output-gather entry points: argument errors are reported before any CUDA call."""
    L = _lib.lib()
    cfg, keep = _cfg([[1, 0]])
    rc, h = _create(cfg)
    assert rc == 0
    # waiting needs peers
    assert L.aoh_gather_wait(h, 0, 5, None) == _lib.INVALID and b"no peers" in L.aoh_last_error()
    regions = (C.c_void_p * 2)(C.c_void_p(4096), C.c_void_p(8192))
    flags = (C.c_void_p * 2)(C.c_void_p(4096), C.c_void_p(8192))
    assert L.aoh_kv_set_peers(h, 9, 0, regions, 1024, flags) == _lib.INVALID       # more than 8 ranks
    assert L.aoh_kv_set_peers(h, 2, 2, regions, 1024, flags) == _lib.INVALID       # rank outside [0, n)
    assert L.aoh_kv_set_peers(h, 2, 0, None, 1024, flags) == _lib.INVALID         # no region table
    assert L.aoh_kv_set_peers(h, 2, 0, regions, 0, flags) == _lib.INVALID          # zero-sized regions
    bad = (C.c_void_p * 2)(C.c_void_p(4096), None)
    assert L.aoh_kv_set_peers(h, 2, 0, regions, 1024, bad) == _lib.INVALID         # a null flag array
    odd = (C.c_void_p * 2)(C.c_void_p(4096), C.c_void_p(8194))
    assert L.aoh_kv_set_peers(h, 2, 0, regions, 1024, odd) == _lib.INVALID         # misaligned flags
    assert L.aoh_kv_set_peers(h, 0, 0, None, 0, None) == _lib.OK                   # detach is always fine
    L.aoh_kv_destroy(h)
    # f32 caches have no gather
    cfg, keep = _cfg([[1, 0]], dtype=_lib.F32)
    rc, h = _create(cfg)
    assert L.aoh_kv_set_peers(h, 2, 0, regions, 1024, flags) == _lib.UNSUPPORTED
    L.aoh_kv_destroy(h)
    ptr = C.c_void_p()
    handle = (C.c_uint8 * _lib.IPC_HANDLE_BYTES)()
    assert L.aoh_shared_alloc(0, C.byref(ptr), handle) == _lib.INVALID
    assert L.aoh_shared_alloc(64, None, handle) == _lib.INVALID
    assert L.aoh_shared_open(None, C.byref(ptr)) == _lib.INVALID
    assert L.aoh_shared_free(None) == _lib.OK and L.aoh_shared_close(None) == _lib.OK


def test_attention_entry_points_need_a_bound_cache():
    """The attention entry points report a null cache, or one never bound to
    device memory, before any CUDA call; the allocation-free decode takes bf16
    caches only."""
    L = _lib.lib()
    buf = C.c_void_p(4096)
    assert L.aoh_attn_prefill(None, 0, 0, 4, buf, buf, buf, buf, None) == _lib.INVALID
    assert b"null cache" in L.aoh_last_error()
    cfg, keep = _cfg([[1, 0]])
    rc, h = _create(cfg)
    assert rc == 0
    assert L.aoh_attn_prefill(h, 0, 0, 4, buf, buf, buf, buf, None) == _lib.STATE
    assert b"not bound" in L.aoh_last_error()
    assert L.aoh_attn_decode(h, 0, 0, buf, buf, buf, buf, None, 0, None) == _lib.STATE
    assert L.aoh_attn_decode_noalloc(h, 0, 0, buf, buf, buf, buf, None) == _lib.STATE
    assert L.aoh_kv_append(h, 0, 0, 4, buf, buf, None) == _lib.STATE
    L.aoh_kv_destroy(h)
    cfg, keep = _cfg([[1, 0]], dtype=_lib.F32)
    rc, h = _create(cfg)
    assert L.aoh_attn_decode_noalloc(h, 0, 0, buf, buf, buf, buf, None) == _lib.UNSUPPORTED
    L.aoh_kv_destroy(h)


def test_decode_dry_run_switch():
    """aoh_kv_set_decode_append: a null cache is an argument error; on a cache
    it toggles (host state only, no CUDA call), any non-zero value enabling."""
    L = _lib.lib()
    assert L.aoh_kv_set_decode_append(None, 0) == _lib.INVALID
    assert b"null cache" in L.aoh_last_error()
    cfg, keep = _cfg([[1, 0]])
    rc, h = _create(cfg)
    assert rc == 0
    for v in (0, 1, 0, 7):
        assert L.aoh_kv_set_decode_append(h, v) == 0
    L.aoh_kv_destroy(h)

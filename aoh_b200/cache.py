"""Paged head-mixed KV cache (device memory owned by torch, bookkeeping in libaoh).

Counterpart of the reference's ``AoHKVCache`` (eval/efficiency/
benchmark_llama31.py:135-184): retrieval KV heads keep every token, streaming
KV heads keep ``sink_size`` + ``recent_size`` tokens.  Instead of per-layer
tensors grown by ``torch.cat`` and trimmed by ``compress_stream``
(attention_utils.py:23-42) -- an O(T) copy per layer per step -- every
(layer, sequence, KV head) unit owns 16-token pages in one pool:
retrieval units grow by pages, streaming units own a fixed set of sink pages
plus a ring of window pages, and appending a token writes one row.

``kv_seq_len`` has the reference's meaning: tokens already cached, advanced
after the last layer of a forward (benchmark_llama31.py:249-250).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib

PAGE_SIZE = 16
HEAD_DIM = 128


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _lib.BF16
    if dtype == torch.float32:
        return _lib.F32
    raise ValueError(f"dtype must be torch.bfloat16 or torch.float32, got {dtype}")


def pages_needed(labels: np.ndarray, batch: int, max_context: int, sink_size: int, recent_size: int,
                 owned: np.ndarray | None = None) -> int:
    """Pool pages for ``max_context`` tokens per sequence."""
    labels = np.asarray(labels)
    L, G = labels.shape
    ret = (labels >= 0.5)[:, None, :].repeat(batch, axis=1)
    own = np.ones((L, batch, G), bool) if owned is None else np.asarray(owned, bool).reshape(L, batch, G)
    n_ret = int((ret & own).sum())
    n_str = int((~ret & own).sum())
    ret_pages = -(-max_context // PAGE_SIZE)
    str_pages = -(-sink_size // PAGE_SIZE) + -(-recent_size // PAGE_SIZE)
    return n_ret * ret_pages + n_str * str_pages


class AoHKVCache:
    """Paged KV cache for one model (all layers).

    Args:
        labels: (num_layers, num_kv_heads) array, >= 0.5 = retrieval (the
            reference's ``head_classification.npy`` / ``classify()`` output).
        num_q_heads: query heads per layer.
        batch: sequences; all share ``kv_seq_len`` as in the reference.
        sink_size, recent_size: streaming window (reference defaults 128/256).
        max_context: tokens a sequence may reach.
        dtype: torch.bfloat16 or torch.float32 (the q/k/v dtype).
        num_pages: pool size; default = exactly what ``max_context`` needs.
        owned: optional (num_layers, batch, num_kv_heads) mask of units stored
            on this device (multi-GPU partition); others get no pages.
        reserve_all: grant every retrieval page up front (no growth later).
        backend: "eager" (the reference's eager protocol: streaming heads see
            sink + window in every call) or "flash" (its decoding-simulation
            protocol, eval/efficiency/attention_utils.py:45-89: the prompt is
            prefilled in one call in which every head attends causally to the
            whole prompt, then decode steps as in the eager protocol).
    """

    def __init__(self, labels, num_q_heads: int, *, batch: int = 1, sink_size: int = 128,
                 recent_size: int = 256, max_context: int, dtype: torch.dtype = torch.bfloat16,
                 device=None, num_pages: int | None = None, owned=None, reserve_all: bool = False,
                 head_dim: int = HEAD_DIM, backend: str = "eager"):
        if sink_size < 0 or recent_size < 0:  # benchmark_llama31.py:257-258
            raise ValueError("sink_size and recent_size must be non-negative")
        if backend not in ("eager", "flash"):
            raise ValueError(f"backend must be 'eager' or 'flash', got {backend!r}")
        self.backend = backend
        labels = np.asarray(labels, dtype=np.float64)
        if labels.ndim != 2:
            raise ValueError(f"labels must be (num_layers, num_kv_heads), got shape {labels.shape}")
        self.labels = labels
        self.num_layers, self.num_kv_heads = labels.shape
        self.num_q_heads = int(num_q_heads)
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        self.grp = self.num_q_heads // self.num_kv_heads
        self.batch = int(batch)
        self.head_dim = int(head_dim)
        self.sink_size, self.recent_size = int(sink_size), int(recent_size)
        self.max_context = int(max_context)
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.n_ret = [int((labels[i] >= 0.5).sum()) for i in range(self.num_layers)]
        self.n_str = [self.num_kv_heads - n for n in self.n_ret]
        self.kv_seq_len = 0
        # While True, decode calls read the device-resident length (set with
        # aoh_kv_set_length, advanced by aoh_kv_advance) instead of kv_seq_len and
        # leave kv_seq_len alone: how a captured decode step is recorded.
        self.device_length = False
        self.owned = None if owned is None else np.ascontiguousarray(owned, dtype=np.uint8).reshape(
            self.num_layers, self.batch, self.num_kv_heads)
        if num_pages is None:
            num_pages = pages_needed(labels, self.batch, self.max_context, self.sink_size,
                                     self.recent_size, self.owned)
        self.num_pages = int(num_pages)

        self._labels_u8 = np.ascontiguousarray(labels >= 0.5, dtype=np.uint8)
        cfg = _lib.KVConfig(self.num_layers, self.batch, self.num_q_heads, self.num_kv_heads,
                            self.head_dim, PAGE_SIZE, _dtype_code(dtype), self.sink_size,
                            self.recent_size, self.max_context, self.num_pages,
                            self._labels_u8.ctypes.data_as(C.POINTER(C.c_uint8)),
                            None if self.owned is None else
                            self.owned.ctypes.data_as(C.POINTER(C.c_uint8)))
        h = C.c_void_p()
        self._L = _lib.lib()
        _lib.check(self._L.aoh_kv_create(C.byref(cfg), C.byref(h)), "AoHKVCache")
        self._h = h
        pool_b, tab_b = C.c_int64(), C.c_int64()
        _lib.check(self._L.aoh_kv_buffer_sizes(h, C.byref(pool_b), C.byref(tab_b)))
        # pool aligned to 1024 B (TMA swizzle atoms); torch's allocator gives >= 512 B, so over-allocate
        # zero-filled: slots not yet written never hold NaN/Inf bit patterns
        self._pool_raw = torch.zeros(pool_b.value + 1024, dtype=torch.uint8, device=self.device)
        off = (-self._pool_raw.data_ptr()) % 1024
        self.pool = self._pool_raw[off:off + pool_b.value]
        self.tables = torch.zeros(tab_b.value, dtype=torch.uint8, device=self.device)
        _lib.check(self._L.aoh_kv_bind(h, C.c_void_p(self.pool.data_ptr()),
                                       C.c_void_p(self.tables.data_ptr()),
                                       C.c_void_p(_lib.stream_handle())), "AoHKVCache.bind")
        self._reserved = 0
        self._ws = None
        if reserve_all:
            self.reserve(self.max_context)

    # -- reference Cache hooks (benchmark_llama31.py:155-166) -------------------
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.kv_seq_len

    def get_max_cache_shape(self):
        return None

    # -- paging ----------------------------------------------------------------
    def reserve(self, n_tokens: int) -> None:
        """Grant retrieval pages so positions < n_tokens are stored (grows in
        1024-token steps, capped at max_context)."""
        if n_tokens <= self._reserved:
            return
        # whole 128-token runs keep 8 consecutive page ids per key tile (the
        # prefill kernel then fetches a tile with 4 TMA loads instead of 32 copies)
        target = min(self.max_context, -(-max(n_tokens, self._reserved + 1024) // 128) * 128)
        _lib.check(self._L.aoh_kv_reserve(self._h, -1, target), "AoHKVCache.reserve")
        _lib.check(self._L.aoh_kv_sync(self._h, C.c_void_p(_lib.stream_handle())))
        self._reserved = target

    def free_pages(self) -> int:
        return int(self._L.aoh_kv_free_pages(self._h))

    def unit_pages(self, layer: int, seq: int, kv_head: int) -> list[int]:
        n = C.c_int32()
        _lib.check(self._L.aoh_kv_unit_pages(self._h, layer, seq, kv_head, None, 0, C.byref(n)))
        buf = (C.c_int32 * max(1, n.value))()
        _lib.check(self._L.aoh_kv_unit_pages(self._h, layer, seq, kv_head, buf, n.value, C.byref(n)))
        return list(buf[: n.value])

    def locate(self, layer: int, seq: int, kv_head: int, position: int) -> tuple[int, int]:
        """(page, slot) holding ``position`` of a unit, (-1, -1) if not held."""
        pg, sl = C.c_int32(), C.c_int32()
        _lib.check(self._L.aoh_kv_locate(self._h, layer, seq, kv_head, position, self.kv_seq_len,
                                         C.byref(pg), C.byref(sl)))
        return int(pg.value), int(sl.value)

    def read_rows(self, layer: int, seq: int, kv_head: int, positions) -> tuple[torch.Tensor, torch.Tensor]:
        """K and V rows (len(positions), head_dim) as stored in the pool
        (inspection/tests; decodes the bf16 page swizzle)."""
        pv = self.pool_view()
        ks, vs = [], []
        d = torch.arange(self.head_dim, device=self.device)
        for p in positions:
            pg, sl = self.locate(layer, seq, kv_head, int(p))
            if pg < 0:
                raise KeyError(f"position {p} of unit ({layer}, {seq}, {kv_head}) is not stored")
            flat = pv[pg].reshape(-1)
            for kv, acc in ((0, ks), (1, vs)):
                if self.dtype == torch.bfloat16:
                    idx = ((d >> 6) * 2048 + kv * 1024 + sl * 64 + (((d >> 3) & 7) ^ (sl & 7)) * 8 + (d & 7))
                else:
                    idx = (kv * PAGE_SIZE + sl) * self.head_dim + d
                acc.append(flat[idx])
        return torch.stack(ks), torch.stack(vs)

    def pool_view(self) -> torch.Tensor:
        """The pool as (num_pages, 2, 16, head_dim) of the cache dtype."""
        return self.pool.view(self.dtype).view(self.num_pages, 2, PAGE_SIZE, self.head_dim)

    def device_status(self) -> int:
        """Read and clear the device check word (0: no bounds check or bounded
        wait tripped).  After a timed-out wait the library re-zeroes the ticket
        counters it owns; the decode workspace is this object's, so it is
        re-zeroed here."""
        f = C.c_int32()
        _lib.check(self._L.aoh_kv_device_status(self._h, C.byref(f), C.c_void_p(_lib.stream_handle())))
        if f.value & 2 and self._ws is not None:
            self._ws.zero_()
        return int(f.value)

    def decode_workspace(self) -> torch.Tensor:
        if self._ws is None:
            n = int(self._L.aoh_decode_workspace_bytes(self._h))
            self._ws = torch.zeros(n, dtype=torch.uint8, device=self.device)
        return self._ws

    # -- AoHKVCache.append_layer (benchmark_llama31.py:171-184) -----------------
    def append_layer(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append k/v (B, C, G, D) at positions kv_seq_len.. of ``layer_idx``."""
        _check_kv(self, k, v)
        C_ = k.shape[1]
        self.reserve(self.kv_seq_len + C_)
        _lib.check(self._L.aoh_kv_append(self._h, layer_idx, self.kv_seq_len, C_,
                                         C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                                         C.c_void_p(_lib.stream_handle())), "append_layer")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.aoh_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check_kv(cache: AoHKVCache, k: torch.Tensor, v: torch.Tensor) -> None:
    want = (cache.batch, k.shape[1], cache.num_kv_heads, cache.head_dim)
    for name, t in (("k", k), ("v", v)):
        if tuple(t.shape) != want:
            raise ValueError(f"{name} must have shape (batch, q_len, num_kv_heads, head_dim) = {want}, "
                             f"got {tuple(t.shape)}")
        if t.dtype != cache.dtype:
            raise ValueError(f"{name} dtype {t.dtype} != cache dtype {cache.dtype}")
        if t.device != cache.device:
            raise ValueError(f"{name} is on {t.device}, cache on {cache.device}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")

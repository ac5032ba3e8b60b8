"""Output gather across the GPUs of one node for multi-GPU decode.

The (sequence, KV head) units of each layer are partitioned over the ranks
(``aoh_partition``, one process per GPU).  Every rank must see every unit's
output before the next layer.  Instead of a collective after the attention
kernel, the decode kernel stores each finished unit's rows straight into the
output region of every rank over NVLink (peer pointers opened with CUDA IPC)
and release-stores a per-(layer, unit) flag there; ``wait(layer)`` is the
layer boundary, a stream-ordered kernel that returns once all units of the
layer have arrived.  The reference has no multi-GPU attention (its drivers
place whole layers on devices, eval/efficiency/benchmark_llama31.py:354-374).

    g = PeerGather(cache, out_shape=(L, B, 1, Hq, D))   # collective: every rank
    out = g.out                                          # bf16 tensor in the shared region
    aoh_attention(cache, l, q, k, v, out=out[l]); g.wait(l)
    g.close()                                            # collective as well

torch.distributed must be initialised (any backend: only the 64-byte IPC
handles are exchanged through it).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .cache import AoHKVCache


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                         "strides": None, "version": 3}


class PeerGather:
    """Attach an NVLink output gather to ``cache`` (collective over ``group``).

    out_shape: shape of the bf16 output tensor every rank decodes into (the
    same on all ranks); ``out`` is that tensor, living in this rank's shared
    region.  ``flags`` (int32, layers x batch x KV heads) holds the arrival
    flags written by the owners of the units.
    """

    def __init__(self, cache: AoHKVCache, out_shape, group=None):
        import torch.distributed as dist

        if cache.dtype != torch.bfloat16:
            raise ValueError("PeerGather needs a bfloat16 cache")
        self.cache = cache
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= 8:
            raise ValueError("PeerGather spans 1 to 8 ranks of one node")
        L = self._L = _lib.lib()
        out_numel = 1
        for d in out_shape:
            out_numel *= int(d)
        self.out_bytes = out_numel * 2
        n_flags = cache.num_layers * cache.batch * cache.num_kv_heads
        self._flag_off = (self.out_bytes + 255) // 256 * 256
        total = self._flag_off + n_flags * 4
        ptr = C.c_void_p()
        handle = (C.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        _lib.check(L.aoh_shared_alloc(total, C.byref(ptr), handle), "aoh_shared_alloc")
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self._own)
                continue
            hb = (C.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h)
            p = C.c_void_p()
            _lib.check(L.aoh_shared_open(hb, C.byref(p)), f"aoh_shared_open(rank {r})")
            self._opened.append(p.value)
            bases.append(p.value)
        outs = (C.c_void_p * self.world)(*bases)
        flags = (C.c_void_p * self.world)(*[b + self._flag_off for b in bases])
        _lib.check(L.aoh_kv_set_peers(cache._h, self.world, self.rank, outs, self.out_bytes, flags),
                   "aoh_kv_set_peers")
        dev = cache.device
        self.out = torch.as_tensor(_DeviceArray(self._own, out_numel, "<i2"), device=dev).view(
            torch.bfloat16).view(tuple(int(d) for d in out_shape))
        self.flags = torch.as_tensor(_DeviceArray(self._own + self._flag_off, n_flags, "<i4"), device=dev)
        dist.barrier(group=group)  # every rank is attached before anyone decodes

    def wait(self, layer: int, past_len: int = _lib.PAST_LEN_DEVICE, stream=None) -> None:
        """Stream-ordered: the layer's outputs of all ranks are here after this."""
        _lib.check(self._L.aoh_gather_wait(self.cache._h, layer, past_len, C.c_void_p(_lib.stream_handle(stream))),
                   "aoh_gather_wait")

    def detach(self) -> None:
        _lib.check(self._L.aoh_kv_set_peers(self.cache._h, 0, 0, None, 0, None), "aoh_kv_set_peers")

    def attach(self) -> None:
        """Re-attach after ``detach`` (same regions)."""
        bases = [None] * self.world
        it = iter(self._opened)
        for r in range(self.world):
            bases[r] = self._own if r == self.rank else next(it)
        outs = (C.c_void_p * self.world)(*bases)
        flags = (C.c_void_p * self.world)(*[b + self._flag_off for b in bases])
        _lib.check(self._L.aoh_kv_set_peers(self.cache._h, self.world, self.rank, outs, self.out_bytes, flags),
                   "aoh_kv_set_peers")

    def close(self) -> None:
        """Detach and release the regions (collective: no rank may still store here)."""
        import torch.distributed as dist

        if self._own is None:
            return
        self.detach()
        torch.cuda.synchronize(self.cache.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.check(self._L.aoh_shared_close(C.c_void_p(p)), "aoh_shared_close")
        self._opened = []
        self.out = None
        self.flags = None
        _lib.check(self._L.aoh_shared_free(C.c_void_p(self._own)), "aoh_shared_free")
        self._own = None

"""One rank of the two-GPU output-gather test (launched by test_gather_gpu.py).

Each rank owns the (sequence, KV head) units aoh_partition gives it and
decodes them with the output gather attached; afterwards every rank must hold
every unit's output, matching a cache on the same GPU that owns all units.
Checked for eager calls (host past_len) and for the CUDA-graph step, with the
layer boundary kept (a wait after each layer) and with the waits overlapping
the next layers' decode kernels.
Rendezvous and the IPC handle exchange use gloo; the data path is the decode
kernel's own stores over NVLink.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from aoh_b200 import AoHKVCache, _lib, aoh_attention  # noqa: E402
from aoh_b200.gather import PeerGather  # noqa: E402
from aoh_b200.graph import DecodeStepGraph  # noqa: E402

L, B, HQ, G, D = 2, 3, 8, 2, 128
SINK, RECENT = 16, 48
CHUNKS = [256, 300]  # prefill, then decode steps
STEPS = 4
T_EXTRA = 2 * STEPS + 2 * (STEPS + 2) + 8  # positions the eager steps and both graphs use


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    labels = np.array([[1, 0], [0, 1]], dtype=np.float64)
    owner = np.zeros((L, B, G), dtype=np.int32)
    lab_u8 = np.ascontiguousarray(labels >= 0.5, dtype=np.uint8)
    T_total = sum(CHUNKS) + T_EXTRA
    _lib.check(_lib.lib().aoh_partition(lab_u8.ctypes.data_as(C.POINTER(C.c_uint8)), L, B, G, sum(CHUNKS), SINK,
                                        RECENT, world, owner.ctypes.data_as(C.POINTER(C.c_int32))), "partition")
    assert set(np.unique(owner)) <= set(range(world))
    mine = AoHKVCache(labels, HQ, batch=B, sink_size=SINK, recent_size=RECENT, max_context=T_total,
                      dtype=torch.bfloat16, device=dev, owned=(owner == rank).astype(np.uint8))
    full = AoHKVCache(labels, HQ, batch=B, sink_size=SINK, recent_size=RECENT, max_context=T_total,
                      dtype=torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(1234)  # same inputs on every rank

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)

    for c in CHUNKS:  # prefill both caches with the same chunks
        for l in range(L):
            q, k, v = rnd(B, c, HQ, D), rnd(B, c, G, D), rnd(B, c, G, D)
            aoh_attention(mine, l, q, k, v)
            aoh_attention(full, l, q, k, v)
    peer = PeerGather(mine, out_shape=(L, B, 1, HQ, D))
    bad = 0
    # eager decode steps: explicit past_len, a gather wait per layer
    for _ in range(STEPS):
        past = mine.kv_seq_len
        for l in range(L):
            q, k, v = rnd(B, 1, HQ, D), rnd(B, 1, G, D), rnd(B, 1, G, D)
            aoh_attention(mine, l, q, k, v, out=peer.out[l])
            peer.wait(l, past_len=past)
            ref = aoh_attention(full, l, q, k, v)
            err = (peer.out[l].float() - ref.float()).abs().max().item()
            if not err <= 2e-2:
                print(f"rank {rank} eager layer {l}: max abs err {err}", flush=True)
                bad += 1
    torch.cuda.synchronize()
    # CUDA-graph steps: the same inputs replayed on both caches, with the layer
    # boundary kept, then with the waits overlapping the next layers' decode
    for overlap in (False, True):
        q, k, v = rnd(L, B, 1, HQ, D), rnd(L, B, 1, G, D), rnd(L, B, 1, G, D)
        ref_out = torch.zeros((L, B, 1, HQ, D), dtype=torch.bfloat16, device=dev)
        g_mine = DecodeStepGraph(mine, q, k, v, peer.out, max_steps=STEPS + 2, gather=peer, overlap_gather=overlap)
        g_full = DecodeStepGraph(full, q, k, v, ref_out, max_steps=STEPS + 2)
        dist.barrier()
        for _ in range(STEPS):
            peer.out.zero_()
            torch.cuda.synchronize()
            dist.barrier()  # no rank stores into a region another rank is still clearing
            g_mine.replay()
            g_full.replay()
            torch.cuda.synchronize()
            err = (peer.out.float() - ref_out.float()).abs().max().item()
            if not err <= 2e-2:
                print(f"rank {rank} graph step (overlap={overlap}): max abs err {err}", flush=True)
                bad += 1
            dist.barrier()
        del g_mine, g_full
    status = mine.device_status()
    if status != 0:
        print(f"rank {rank}: device check word {status}", flush=True)
        bad += 1
    peer.close()
    dist.destroy_process_group()
    print(f"rank {rank}: {'FAIL' if bad else 'ok'}", flush=True)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())

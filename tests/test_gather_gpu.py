"""Output gather over NVLink between two GPUs (one process per GPU), and the
gather wait's time bound on one GPU.

The two-GPU test is skipped with fewer than two GPUs; its ranks rendezvous
over gloo on 127.0.0.1 (gather_worker.py says what each rank checks).
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_gather_two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "tests" / "gather_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(": ok") == 2, r.stdout[-3000:]


def test_gather_wait_gives_up_on_a_rank_that_never_publishes(cuda_device):
    """One GPU, two ranks' worth of regions: rank 1's output region and flag
    array are a second local buffer that no decode kernel ever publishes to.
    aoh_gather_wait must give up in bounded time (its peer limit is 1 s),
    record a wait timeout in the check word instead of hanging the stream, and
    the cache must work normally after the status has been read."""
    import ctypes as C
    import time

    import numpy as np
    import torch

    from aoh_b200 import AoHKVCache, _lib, aoh_attention

    L, B, Hq, G, D, T = 1, 2, 8, 2, 128, 300
    labels = np.array([[1, 0]], dtype=np.float64)
    owned = np.zeros((L, B, G), dtype=np.uint8)
    owned[:, 0, :] = 1  # this rank owns sequence 0; sequence 1 belongs to the silent rank
    cache = AoHKVCache(labels, Hq, batch=B, sink_size=16, recent_size=32, max_context=T + 4,
                       dtype=torch.bfloat16, owned=owned, reserve_all=True)
    gen = torch.Generator(device="cuda").manual_seed(3)
    pv = cache.pool_view()
    pv.copy_((torch.randn(pv.shape, generator=gen, device="cuda") * 0.5).to(torch.bfloat16))
    cache.kv_seq_len = T
    regions = [torch.zeros((L, B, 1, Hq, D), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    flags = [torch.zeros(L * B * G, dtype=torch.int32, device="cuda") for _ in range(2)]
    lib = _lib.lib()
    outs = (C.c_void_p * 2)(*[r.data_ptr() for r in regions])
    fl = (C.c_void_p * 2)(*[f.data_ptr() for f in flags])
    _lib.check(lib.aoh_kv_set_peers(cache._h, 2, 0, outs, regions[0].numel() * 2, fl), "aoh_kv_set_peers")
    q = torch.randn((B, 1, Hq, D), generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, 1, G, D), generator=gen, device="cuda").to(torch.bfloat16)
    aoh_attention(cache, 0, q, k, k, out=regions[0][0], advance=False)
    torch.cuda.synchronize()
    st = C.c_void_p(_lib.stream_handle())
    t0 = time.perf_counter()
    _lib.check(lib.aoh_gather_wait(cache._h, 0, T, st), "aoh_gather_wait")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    status = cache.device_status()
    assert status & 2, f"check word {status}: the wait should have recorded a timeout"
    assert waited < 2.0, f"the bounded wait took {waited:.2f} s"
    # this rank's units were published to both ranks, the silent rank's never
    want = np.zeros((L, B, G), dtype=np.int32)
    want[:, 0, :] = T + 1
    for f in flags:
        assert np.array_equal(f.cpu().numpy().reshape(L, B, G), want)
    assert torch.equal(regions[0][:, 0], regions[1][:, 0]) and regions[0][:, 0].abs().sum() > 0
    # the status read cleared the word: a wait whose units all arrived passes at once
    _lib.check(lib.aoh_kv_set_peers(cache._h, 0, 0, None, 0, None), "aoh_kv_set_peers")
    owned_all = AoHKVCache(labels, Hq, batch=B, sink_size=16, recent_size=32, max_context=T + 4,
                           dtype=torch.bfloat16, reserve_all=True)
    owned_all.kv_seq_len = T
    region = torch.zeros((L, B, 1, Hq, D), dtype=torch.bfloat16, device="cuda")
    flag = torch.zeros(L * B * G, dtype=torch.int32, device="cuda")
    _lib.check(lib.aoh_kv_set_peers(owned_all._h, 1, 0, (C.c_void_p * 1)(region.data_ptr()), region.numel() * 2,
                                    (C.c_void_p * 1)(flag.data_ptr())), "aoh_kv_set_peers")
    aoh_attention(owned_all, 0, q, k, k, out=region[0], advance=False)
    t0 = time.perf_counter()
    _lib.check(lib.aoh_gather_wait(owned_all._h, 0, T, st), "aoh_gather_wait")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    assert owned_all.device_status() == 0
    assert cache.device_status() == 0

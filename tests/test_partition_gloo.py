"""Multi-GPU host logic on CPU ranks (gloo, world size 2, 127.0.0.1).

Each rank computes the partition of the (sequence, KV head) units (every rank
must get the same table), decodes only the units it owns with the oracle and
places them in a zero-filled output of the whole layer; the exchange step
(all-reduce of disjoint units) must reproduce the single-process decode of
every unit bit for bit.  In the second case one rank leaves before the
exchange: the other rank's collective must fail within the process group's
timeout instead of hanging.
"""
import ctypes as C
import json
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

L_, B_, HQ_, G_, D_, T_ = 2, 3, 8, 4, 32, 700
SINK_, RECENT_ = 16, 48


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(layer: int):
    rng = np.random.default_rng(100 + layer)
    q = rng.standard_normal((B_, 1, HQ_, D_), dtype=np.float32)
    kn = rng.standard_normal((B_, 1, G_, D_), dtype=np.float32)
    vn = rng.standard_normal((B_, 1, G_, D_), dtype=np.float32)
    kc = rng.standard_normal((B_, T_, G_, D_), dtype=np.float32)
    vc = rng.standard_normal((B_, T_, G_, D_), dtype=np.float32)
    return q, kn, vn, kc, vc


def _labels():
    # retrieval heads clustered in KV groups 0-1 (the skew the partition must absorb)
    return np.array([[1, 1, 0, 0], [1, 0, 0, 0]], dtype=np.float64)


def _rank_main(rank: int, world: int, port: int, mode: str, out_dir: str) -> None:
    import torch
    import torch.distributed as dist

    from aoh_b200 import _lib
    from oracle import aoh_oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    result = {"rank": rank}
    labels = _labels()
    lab_u8 = np.ascontiguousarray(labels >= 0.5, dtype=np.uint8)
    owner = np.zeros((L_, B_, G_), dtype=np.int32)
    _lib.check(_lib.lib().aoh_partition(lab_u8.ctypes.data_as(C.POINTER(C.c_uint8)), L_, B_, G_, T_, SINK_, RECENT_,
                                        world, owner.ctypes.data_as(C.POINTER(C.c_int32))), "aoh_partition")
    tables = [torch.zeros(owner.size, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(tables, torch.from_numpy(owner.ravel().copy()))
    result["same_table"] = all(bool((t.numpy() == owner.ravel()).all()) for t in tables)
    grp = HQ_ // G_
    mine = np.zeros((L_, B_, 1, HQ_, D_), dtype=np.float32)
    full = np.zeros_like(mine)
    for l in range(L_):
        q, kn, vn, kc, vc = _inputs(l)
        full[l] = orc.decode_from_state(q, kn, vn, kc, vc, labels[l], T_, SINK_, RECENT_, "f32")
        for b in range(B_):
            for g in range(G_):
                if owner[l, b, g] != rank:
                    continue
                hs = slice(g * grp, (g + 1) * grp)
                mine[l, b:b + 1, :, hs] = orc.decode_from_state(
                    q[b:b + 1, :, hs], kn[b:b + 1, :, g:g + 1], vn[b:b + 1, :, g:g + 1], kc[b:b + 1, :, g:g + 1],
                    vc[b:b + 1, :, g:g + 1], labels[l, g:g + 1], T_, SINK_, RECENT_, "f32")
    if mode == "leave" and rank == 1:
        result["left"] = True  # this rank goes away before the exchange
    else:
        t = torch.from_numpy(mine)
        try:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            result["exact"] = bool(np.array_equal(t.numpy(), full))
            result["raised"] = False
        except Exception as e:  # noqa: BLE001 - the failure is the point of the second case
            result["raised"] = True
            result["error"] = type(e).__name__
    (Path(out_dir) / f"rank{rank}.json").write_text(json.dumps(result))
    if not result.get("raised") and not result.get("left"):
        dist.destroy_process_group()


def _run(mode: str, tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.spawn(_rank_main, args=(2, _free_port(), mode, str(tmp_path)), nprocs=2, join=False)
    ok = ctx.join(timeout=120)
    while not ok:
        ok = ctx.join(timeout=120)
    return [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(2)]


def test_partitioned_decode_matches_single_process(tmp_path):
    res = _run("gather", tmp_path)
    for r in res:
        assert r["same_table"]
        assert r["raised"] is False
        assert r["exact"], r


def test_rank_leaving_before_exchange_fails_fast(tmp_path):
    import time

    t0 = time.time()
    res = _run("leave", tmp_path)
    assert res[1]["left"]
    assert res[0]["raised"], res[0]
    assert time.time() - t0 < 100

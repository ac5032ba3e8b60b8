#!/usr/bin/env python3
"""Benchmark: head-mixed decode attention, microseconds per layer at 128K context.

Workload (one step = one decode token through every layer's attention):
  Llama-3.1-8B attention shapes (32 query heads, 8 KV heads, head_dim 128),
  32 layers, bf16, batch 1 per GPU, 131072-token paged context (16-token
  pages), 6 of 8 KV heads streaming per layer (labels seeded uniform), sink 128,
  window 256, KV ~ 0.5*N(0,1), q ~ N(0,1).  Synthetic data (no checkpoint or
  dataset is needed or available); the cache is filled on the device.

  --gpus N > 1 (one process per GPU, torchrun): N sequences of 128K, the
  (sequence, KV head) units of every layer partitioned across ranks by the
  longest-processing-time rule on touched KV tokens; each rank attends its
  units and its decode kernel stores every finished unit's output into all
  ranks' output buffers over NVLink (CUDA IPC peer pointers) with a flag per
  unit; a wait kernel per layer is the layer boundary, and the whole step is
  one CUDA graph (weak scaling: per-GPU work is fixed).  ``--gather nccl``
  instead all-gathers the outputs with NCCL after each layer, eagerly (the
  library-collective baseline).  ``value`` is microseconds per (layer,
  sequence) for the whole job.

Also reported on the same line: the decode kernel's HBM roofline fraction,
an end-to-end number through the public API with host buffers, the CPU
reference (the oracle's restatement of the reference's eager path) on a
bounded sample, bf16 prefill TFLOP/s on a bounded sample of the 64K chunked
prefill, and the classifier's label agreement with the reference.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl aoh|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L_LAYERS, HQ, G, D, T_CTX = 32, 32, 8, 128, 131072
N_STREAM, SINK, RECENT, KV_SCALE, SEED = 6, 128, 256, 0.5, 0
METRIC = "decode attn us/layer @128K"
WORKLOAD = "llama31_8b_decode_128k"
BATCH_FIXED = 0      # > 0: strong scaling with this many sequences (else one per GPU)
SKEWED_LABELS = False


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def decode_layer_bytes(T: int, n_ret_units: int, n_str_units: int, B: int) -> int:
    """Algorithmic HBM bytes of one decode launch (one layer): K+V rows read
    (retrieval: T cached keys; streaming: min(T, sink+recent)), the new K/V row
    read once and written once per unit, q read, output written, page ids read."""
    row = 2 * D * 2  # K + V, bf16
    kv = n_ret_units * T * row + n_str_units * min(T, SINK + RECENT) * row
    new = (n_ret_units + n_str_units) * row * 2
    qo = 2 * B * HQ * D * 2
    tables = n_ret_units * (-(-T // 16)) * 4 + n_str_units * ((SINK + RECENT) // 16) * 4
    return kv + new + qo + tables


# ----------------------------------------------------------------------------
# CPU reference (oracle restatement of the reference's eager decode)
# ----------------------------------------------------------------------------

def cpu_reference_layer_us(n_calls: int, budget_s: float = 60.0):
    """Time the eager decode of one layer at 128K on the host cores: the
    reference's AoHKVCache state (full retrieval KV, compressed streaming KV)
    and its per-layer forward (torch.cat + repeat_kv + fp32 scores + softmax +
    P.V + append), restated in numpy, with every host core for its BLAS
    (torchrun sets OMP_NUM_THREADS=1 otherwise).  Stops after n_calls or once
    budget_s has passed (at least 2 calls).  Returns (us per layer call,
    threads, calls timed)."""
    from threadpoolctl import threadpool_limits

    from oracle import aoh_oracle as orc
    threads = os.cpu_count() or 1
    limiter = threadpool_limits(limits=threads)
    rng = np.random.Generator(np.random.PCG64(SEED))
    labels = np.ones((1, G))
    labels[0, :N_STREAM] = 0.0
    cache = orc.OracleKVCache(1, labels, SINK, RECENT, "bf16")
    nr, ns = cache.n_ret[0], cache.n_str[0]
    bf = orc.bf16_round
    cache.full_k[0] = bf(rng.standard_normal((1, nr, T_CTX, D), dtype=np.float32) * 0.5)
    cache.full_v[0] = bf(rng.standard_normal((1, nr, T_CTX, D), dtype=np.float32) * 0.5)
    cache.stream_k[0] = bf(rng.standard_normal((1, ns, SINK + RECENT, D), dtype=np.float32) * 0.5)
    cache.stream_v[0] = bf(rng.standard_normal((1, ns, SINK + RECENT, D), dtype=np.float32) * 0.5)
    cache.kv_seq_len = T_CTX
    q = bf(rng.standard_normal((1, 1, HQ, D), dtype=np.float32))
    k = bf(rng.standard_normal((1, 1, G, D), dtype=np.float32) * 0.5)
    v = bf(rng.standard_normal((1, 1, G, D), dtype=np.float32) * 0.5)
    orc.layer_attention(cache, 0, q, k, v)  # warm-up
    t0 = time.perf_counter()
    done = 0
    while done < max(1, n_calls):
        orc.layer_attention(cache, 0, q, k, v)
        done += 1
        if done >= 2 and time.perf_counter() - t0 > budget_s:
            break
    dt = (time.perf_counter() - t0) / done
    limiter.restore_original_limits()
    return dt * 1e6, threads, done


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    us, cores, n = cpu_reference_layer_us(max(1, args.steps), budget_s=90.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/layer",
        "n_gpus": args.gpus, "steps": n, "warmup": 1, "ms_per_step": round(us * L_LAYERS / 1000, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "layers": L_LAYERS, "batch": 1, "context": T_CTX,
                   "streaming_kv_heads": f"{N_STREAM}/{G}", "sink": SINK, "window": RECENT},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/layer", "cores": cores, "kind": "port",
                         "sample": f"{n} decode calls of one layer at 128K (numpy restatement of the reference's "
                                   f"eager AoHKVCache forward, {cores} BLAS threads; at most 90 s of calls); "
                                   "a step is one layer"},
        "e2e": {"value": round(us, 1), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

def run_aoh(args):
    import torch
    import torch.distributed as dist

    import aoh_b200
    from aoh_b200 import AoHKVCache, aoh_attention, synthetic as syn
    from aoh_b200 import _lib
    import ctypes as C

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    B = BATCH_FIXED or world  # default: one sequence per GPU (weak scaling)
    labels = (syn.labels_skewed if SKEWED_LABELS else syn.labels_uniform)(SEED, L_LAYERS, G, N_STREAM)
    n_ret_layer = int((labels[0] >= 0.5).sum())
    # partition (sequence, KV head) units over ranks
    owner = np.zeros((L_LAYERS, B, G), dtype=np.int32)
    if world > 1:
        lab_u8 = np.ascontiguousarray(labels >= 0.5, dtype=np.uint8)
        _lib.check(_lib.lib().aoh_partition(lab_u8.ctypes.data_as(C.POINTER(C.c_uint8)), L_LAYERS, B, G,
                                            T_CTX, SINK, RECENT, world,
                                            owner.ctypes.data_as(C.POINTER(C.c_int32))), "aoh_partition")
    owned = (owner == rank).astype(np.uint8)
    max_ctx = T_CTX + args.warmup + args.steps + 2 * (args.e2e_steps + 2) + 4096 + 5 * 400
    cache = AoHKVCache(labels, HQ, batch=B, sink_size=SINK, recent_size=RECENT, max_context=max_ctx,
                       dtype=torch.bfloat16, device=dev, owned=owned, reserve_all=True)
    gen = torch.Generator(device=dev).manual_seed(SEED + 17 * rank)
    pv = cache.pool_view()
    for i in range(0, pv.shape[0], 65536):  # fill the pool in slabs (no large fp32 temporaries)
        sl = pv[i:i + 65536]
        sl.copy_((torch.randn(sl.shape, generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16))
    cache.kv_seq_len = T_CTX
    q = torch.randn((L_LAYERS, B, 1, HQ, D), generator=gen, device=dev).to(torch.bfloat16)
    kn = (torch.randn((L_LAYERS, B, 1, G, D), generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16)
    vn = (torch.randn((L_LAYERS, B, 1, G, D), generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16)
    peer = None
    if world > 1 and args.gather == "peer":
        from aoh_b200.gather import PeerGather
        peer = PeerGather(cache, out_shape=(L_LAYERS, B, 1, HQ, D))
        out = peer.out  # decoded straight into the shared output region
        out.zero_()
    else:
        out = torch.zeros((L_LAYERS, B, 1, HQ, D), dtype=torch.bfloat16, device=dev)

    # NCCL gather plumbing (--gather nccl): pack owned (b, g) head groups, all-gather, unpack
    if world > 1 and peer is None:
        grp = HQ // G
        packs, unpack = [], []
        max_units = max(int((owner[l] == r).sum()) for l in range(L_LAYERS) for r in range(world))
        for l in range(L_LAYERS):
            mine = np.flatnonzero(owner[l].ravel() == rank)
            idx = np.full(max_units, mine[0] if len(mine) else 0, dtype=np.int64)
            idx[:len(mine)] = mine
            packs.append(torch.from_numpy(idx).to(dev))
            allidx, src = [], []
            for r in range(world):
                units = np.flatnonzero(owner[l].ravel() == r)
                allidx.extend(units.tolist())
                src.extend((r * max_units + np.arange(len(units))).tolist())
            unpack.append((torch.tensor(src, device=dev), torch.tensor(allidx, device=dev)))
        gathered = torch.empty((world * max_units, grp * D), dtype=torch.bfloat16, device=dev)

    def layer(l, q_l, k_l, v_l, o_l):
        aoh_attention(cache, l, q_l, k_l, v_l, out=o_l)
        if world > 1:
            flat = o_l.view(B * G, -1)
            mine = flat.index_select(0, packs[l])
            dist.all_gather_into_tensor(gathered, mine)
            src, dst = unpack[l]
            flat.index_copy_(0, dst, gathered.index_select(0, src))

    graph = None
    if world == 1 or peer is not None:
        from aoh_b200.graph import DecodeStepGraph
        graph = DecodeStepGraph(cache, q, kn, vn, out,
                                max_steps=args.warmup + args.steps + args.e2e_steps + 8 + 5 * 400,
                                gather=peer)
    used_graph = graph is not None

    def step():
        if graph is not None:
            graph.replay()
            return
        for l in range(L_LAYERS):
            layer(l, q[l], kn[l], vn[l], out[l])

    def barrier():
        if world > 1:
            dist.barrier()

    # ---------------- device-timed region ----------------
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "") or "")
    clocks = ClockSampler(("GPU-" + uuid) if uuid and not uuid.startswith("GPU-") else (uuid or local))
    clocks.start()  # sampling runs through warm-up and the timed steps (the same steady load)
    for _ in range(args.warmup):
        step()
    # more warm-up until nvidia-smi reports under load (2 s at most); ranks are
    # coupled step by step, so all of them decide together and run the same steps
    t_w = time.perf_counter()
    for _ in range(400):  # pages are reserved for 5 * 400 extra steps
        torch.cuda.synchronize()
        flags = torch.tensor([0 if clocks.lines else 1, 1 if time.perf_counter() - t_w >= 2.0 else 0],
                             device=dev, dtype=torch.int32)
        if world > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MAX)
        if flags[0].item() == 0 or flags[1].item() == 1:
            break
        for _ in range(5):
            step()
    barrier()
    torch.cuda.synchronize()
    T0 = cache.kv_seq_len
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_us = (time.perf_counter() - h0) * 1e6 / (args.steps * L_LAYERS)
    ev1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert cache.device_status() == 0, "device-side check tripped"
    us_layer_seq = ms * 1000.0 / (L_LAYERS * B)

    # roofline of the decode kernel (the only kernel in the N=1 step)
    hbm, bf16_peak, peak_src = measured_peaks()
    T_mid = T0 + args.steps // 2
    n_ret_units = int(((labels >= 0.5)[:, None, :].repeat(B, 1) & (owned > 0)).sum()) // L_LAYERS
    n_str_units = int(owned.sum()) // L_LAYERS - n_ret_units
    bytes_launch = decode_layer_bytes(T_mid, n_ret_units, n_str_units, B)
    launch_us = ms * 1000.0 / L_LAYERS
    achieved = bytes_launch / (launch_us * 1e-6) / 1e9
    # DRAM bytes per launch from the committed ncu summary (64K capture scaled to 128K)
    traffic = None
    tp = ROOT / "profiles" / "decode_bf16_64k_ncu_full.md"
    if tp.exists() and T_CTX == 131072:
        import re
        m = re.search(r"dram_bytes_per_launch_128k = (\d+)", tp.read_text())
        traffic = int(m.group(1)) if m else None

    # ---------------- end to end through the public API, host buffers ----------------
    e2e = None
    if args.e2e_steps > 0:
        qh = q.cpu().pin_memory()
        kh = kn.cpu().pin_memory()
        vh = vn.cpu().pin_memory()
        oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        if graph is not None:
            qd, kd, vd = q, kn, vn  # the graph's input buffers
        else:
            qd, kd, vd = torch.empty_like(q), torch.empty_like(kn), torch.empty_like(vn)

        def e2e_step():
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
            if graph is not None:
                graph.replay()
            else:
                for l in range(L_LAYERS):
                    layer(l, qd[l], kd[l], vd[l], out[l])
            oh.copy_(out, non_blocking=True)

        e2e_step()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": round(ems * 1000.0 / (L_LAYERS * B), 2), "unit": "us/layer",
               "h2d_bytes_per_step": int(q.numel() + kn.numel() + vn.numel()) * 2,
               "d2h_bytes_per_step": int(out.numel()) * 2}

    extras = {}
    if rank == 0 and world == 1:
        if not args.no_prefill:
            extras["prefill"] = {
                "workload": "qwen25_7b_chunked_prefill_64k (28 layers, 28/4 heads, 2/4 streaming, bf16)",
                "chunk_4096": prefill_full(torch, dev, bf16_peak, 4096),
                "chunk_256": prefill_full(torch, dev, bf16_peak, 256),
                "kernel_sample": prefill_sample(torch, dev, bf16_peak),
            }
        if not args.no_classifier:
            extras["labels_exact"] = classifier_check(torch, dev)
    cpu = None
    if rank == 0 and world == 1 and args.cpu_calls > 0:
        us_cpu, cores, n_cpu = cpu_reference_layer_us(args.cpu_calls, budget_s=30.0)
        cpu = {"value": round(us_cpu, 1), "unit": "us/layer", "cores": cores, "kind": "port",
               "sample": f"{n_cpu} decode calls of one layer at 128K context (numpy restatement of the "
                         "reference's eager AoHKVCache forward: cat + repeat_kv + fp32 scores + softmax + P.V + "
                         "append)"}

    if world > 1:
        graph = None
        if peer is not None:
            torch.cuda.synchronize()
            peer.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(us_layer_seq, 3), "unit": "us/layer", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False,
        "scaling": "strong" if BATCH_FIXED else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "layers": L_LAYERS, "sequences": B, "context": T_CTX,
                   "q_heads": HQ, "kv_heads": G, "head_dim": D, "page": 16,
                   "streaming_kv_heads": f"{N_STREAM}/{G}", "sink": SINK, "window": RECENT,
                   "parallelism": f"units{world}" if world > 1 else "single",
                   "l2": f"no flush: {bytes_launch * L_LAYERS / 1e9:.2f} GB of KV per step >> 126 MB L2"},
        "tokens_per_s": round(B / (ms / 1000.0), 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": peak_src,
                     "kernel": "decode_bf16_kernel", "bytes_per_launch": bytes_launch,
                     "avg_launch_us": round(launch_us, 3)},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "gpu_launches": (L_LAYERS * (2 if peer is not None else 1) + (1 if used_graph else 0)) * args.steps,
        "launch_mode": "cuda_graph+pdl" if used_graph else "eager+pdl",
        "gather": None if world == 1 else ("nvlink_peer_stores" if peer is not None else "nccl_all_gather"),
        "host_enqueue_us_per_layer": round(host_us, 2),
        "clocks": clk,
        **extras,
    }
    print(json.dumps(line), flush=True)
    return 0


def prefill_sample(torch, dev, bf16_peak):
    """bf16 prefill TFLOP/s on a bounded sample of the 64K chunked prefill
    (Qwen2.5-7B shapes, one layer, 2 of 4 KV heads streaming): the last 4096-token
    chunk at 61440 cached tokens."""
    from aoh_b200 import AoHKVCache, aoh_attention
    from aoh_b200.metrics import attention_flops
    Hq, Gq, past, C = 28, 4, 61440, 4096
    labels = np.array([[1, 0, 1, 0]], dtype=np.float64)
    cache = AoHKVCache(labels, Hq, batch=1, max_context=past + C, dtype=torch.bfloat16, device=dev,
                       reserve_all=True)
    gen = torch.Generator(device=dev).manual_seed(3)
    pv = cache.pool_view()
    pv.copy_(torch.randn(pv.shape, generator=gen, device=dev).to(torch.bfloat16))
    cache.kv_seq_len = past
    q = torch.randn((1, C, Hq, D), generator=gen, device=dev).to(torch.bfloat16)
    k = torch.randn((1, C, Gq, D), generator=gen, device=dev).to(torch.bfloat16)
    v = torch.randn((1, C, Gq, D), generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    for _ in range(2):
        aoh_attention(cache, 0, q, k, v, out=out, advance=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        aoh_attention(cache, 0, q, k, v, out=out, advance=False)
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1000.0 / reps
    grp = Hq // Gq
    flops = 2 * grp * (attention_flops(C, past, True, 128, 256) + attention_flops(C, past, False, 128, 256))
    tf = flops / sec / 1e12
    return {"tflops": round(tf, 2), "frac_of_bf16_peak": round(tf / bf16_peak, 4), "ms": round(sec * 1e3, 3),
            "sample": "1 layer, last 4096-token chunk at 61440 cached tokens, Qwen2.5-7B heads, 2/4 streaming",
            "flops": flops}


def prefill_full(torch, dev, bf16_peak, chunk: int, context: int = 65536, layers: int = 28):
    """Chunked prefill to ``context`` tokens through every layer: Qwen2.5-7B
    shapes (28 query / 4 KV heads, head_dim 128), bf16, 2 of 4 KV heads streaming
    per layer (seeded), sink 128, window 256, q/k/v ~ N(0,1) generated once per
    layer and reused for every chunk (values do not change the work).  The whole
    prefill runs twice: the first pass warms up (kernel attributes, split-KV
    scratch sized for every chunk), the second is timed with CUDA events.  Flops
    count only masked-in (query, key) pairs."""
    from aoh_b200 import AoHKVCache, aoh_attention
    from aoh_b200 import synthetic as syn
    from aoh_b200.metrics import attention_flops
    Hq, Gq, sink, recent = 28, 4, 128, 256
    grp = Hq // Gq
    labels = syn.labels_uniform(31, layers, Gq, 2)
    cache = AoHKVCache(labels, Hq, batch=1, sink_size=sink, recent_size=recent, max_context=context,
                       dtype=torch.bfloat16, device=dev, reserve_all=True)
    gen = torch.Generator(device=dev).manual_seed(5)
    qs = [torch.randn((1, chunk, Hq, D), generator=gen, device=dev).to(torch.bfloat16) for _ in range(layers)]
    ks = [torch.randn((1, chunk, Gq, D), generator=gen, device=dev).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn((1, chunk, Gq, D), generator=gen, device=dev).to(torch.bfloat16) for _ in range(layers)]
    out = torch.empty_like(qs[0])

    def run():
        cache.kv_seq_len = 0
        for _ in range(0, context, chunk):
            for l in range(layers):
                aoh_attention(cache, l, qs[l], ks[l], vs[l], out=out)

    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    assert cache.device_status() == 0, "device-side check tripped"
    sec = e0.elapsed_time(e1) / 1000.0
    flops = 0
    for start in range(0, context, chunk):
        f_ret = attention_flops(chunk, start, True, sink, recent)
        f_str = attention_flops(chunk, start, False, sink, recent)
        for l in range(layers):
            n_ret = int((labels[l] >= 0.5).sum())
            flops += grp * (n_ret * f_ret + (Gq - n_ret) * f_str)
    tf = flops / sec / 1e12
    cache.close()
    return {"chunk": chunk, "tflops": round(tf, 2), "frac_of_bf16_peak": round(tf / bf16_peak, 4),
            "seconds": round(sec, 4), "flops": flops, "calls": layers * (context // chunk)}


def whole_model(torch, dev, context: int = 131072, decode_steps: int = 20, full_baseline: bool = True):
    """Whole-model decode ms/token, the reference's Table 11 decode column
    (eval/efficiency/benchmark_llama31.py: decode steps after a long context,
    sink 128 / window 256): Llama-3.1-8B architecture with random-init bf16
    weights (no checkpoint is available), 6 of 8 KV heads streaming per layer
    (sparsity 0.75, labels seeded uniform), patched with patch_aoh_model; and,
    on the same GPU, the unpatched model with transformers' own attention over
    a full KV cache (the "full attention" column).  Both caches are filled with
    synthetic K/V (0.5 * N(0,1)) of `context` tokens instead of running the
    prefill (decode time depends on the cache's size, not its values; prefill
    is measured on its own).  Each decode step (one token, its logits) is timed
    with CUDA events; the median is reported."""
    from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM

    from aoh_b200 import synthetic as syn
    from aoh_b200.hf import patch_aoh_model
    L, KVH = 32, 8
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=14336, num_hidden_layers=L, num_attention_heads=32,
                      num_key_value_heads=KVH, head_dim=128, vocab_size=128256, rope_theta=500000.0,
                      max_position_embeddings=context + decode_steps + 64)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    gen = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (1, decode_steps + 2), generator=gen, device=dev)

    def decode(cache):
        times = []
        with torch.no_grad():
            model(input_ids=ids[:, :1], past_key_values=cache, use_cache=True)  # warm-up step
            for t in range(decode_steps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                model(input_ids=ids[:, 1 + t:2 + t], past_key_values=cache, use_cache=True)
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
        return float(np.median(times))

    res = {"model": "llama31_8b_random_init_bf16", "context": context, "decode_steps": decode_steps,
           "cache": "synthetic K/V of the context length (no prefill)"}
    if full_baseline:
        full = DynamicCache()
        for l in range(L):
            k = (torch.randn((1, KVH, context, D), generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16)
            v = (torch.randn((1, KVH, context, D), generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16)
            full.update(k, v, l)
            del k, v
        ms = decode(full)
        res["full_attention"] = {"decode_ms_per_token": round(ms, 3),
                                 "attention": str(model.config._attn_implementation)}
        del full
        torch.cuda.empty_cache()
    labels = syn.labels_uniform(SEED, L, KVH, 6)
    make_cache, n_ret, n_str = patch_aoh_model(model, labels, SINK, RECENT)
    cache = make_cache(max_context=context + decode_steps + 8)
    cache.paged.reserve(context + decode_steps + 8)
    pv = cache.paged.pool_view()
    for i in range(0, pv.shape[0], 65536):
        sl = pv[i:i + 65536]
        sl.copy_((torch.randn(sl.shape, generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16))
    cache.kv_seq_len = context
    ms = decode(cache)
    res["aoh_sp0.75"] = {"decode_ms_per_token": round(ms, 3), "kv_pool_gb": round(cache.paged.pool.numel() / 1e9, 3)}
    assert cache.paged.device_status() == 0, "device-side check tripped"
    if full_baseline:
        res["decode_speedup_vs_full"] = round(res["full_attention"]["decode_ms_per_token"] / ms, 2)
    return res


def classifier_check(torch, dev):
    """AoH classifier on seeded Qwen2.5-7B-shaped projections (28 layers, 28/4
    heads, hidden 3584, bf16): GPU effective ranks -> labels vs the reference's
    labels stored in tests/golden/cls_qwen25_7b.npz, both modes, 3 aggregations
    x 3 sparsities."""
    from aoh_b200 import classifier as clf
    from aoh_b200 import synthetic as syn
    z = np.load(ROOT / "tests" / "golden" / "cls_qwen25_7b.npz")
    L, H, Gk, Dh, dm = 28, 28, 4, 128, 3584
    wq = torch.empty((L, H * Dh, dm), dtype=torch.bfloat16, device=dev)
    wk = torch.empty((L, Gk * Dh, dm), dtype=torch.bfloat16, device=dev)
    for l in range(L):
        a, b = syn.classifier_weights(0, l, H, Gk, Dh, dm)
        wq[l].copy_(torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16))
        wk[l].copy_(torch.from_numpy(b.astype(np.int16)).view(torch.bfloat16))
    res = {}
    for mode in ("fp32", "binary"):
        clf.eff_ranks_from_weights(wq, wk, H, Gk, Dh, binary=mode == "binary")  # warm-up
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ranks = clf.eff_ranks_from_weights(wq, wk, H, Gk, Dh, binary=mode == "binary")
        sec = time.perf_counter() - t0
        match = total = sub_noise = 0
        for agg in ("mean", "min", "max"):
            kv = clf.aggregate_kv(ranks, Gk, agg)
            for sp in (0.25, 0.5, 0.75):
                lab = clf.labels_from_ranks(kv, sp)
                want = z[f"{mode}_{agg}_sp{sp}_labels"]
                margins = clf.label_margins(kv, sp)
                for l in range(L):
                    total += 1
                    if np.array_equal(lab[l], want[l]):
                        match += 1
                    elif margins[l] < 2e-6:
                        sub_noise += 1
        rel = float(np.max(np.abs(ranks - z[f"{mode}_eff_ranks_q"]) / z[f"{mode}_eff_ranks_q"]))
        res[mode] = {"layer_decisions_equal": f"{match}/{total}", "differ_below_ref_fp32_noise": sub_noise,
                     "max_rel_rank_err": rel, "gpu_seconds": round(sec, 4),
                     "ref_cpu_seconds": round(float(z[f"{mode}_classify_seconds"]), 3)}
    return res


def _set_workload(context: int, layers: int, name: str = "llama31_8b_decode_128k") -> None:
    global T_CTX, L_LAYERS, WORKLOAD, BATCH_FIXED, SKEWED_LABELS, METRIC
    if name == "qwen3_8b_decode_256k_b8":
        # batched long decode across GPUs: Qwen3-8B attention shapes (32 query /
        # 8 KV heads), 36 layers, 8 sequences of 262144 tokens, 6/8 streaming,
        # retrieval heads clustered in KV groups 0-1; strong scaling
        T_CTX, L_LAYERS, BATCH_FIXED, SKEWED_LABELS = 262144, 36, 8, True
        WORKLOAD, METRIC = name, "decode attn us/(layer*sequence) @256K batch 8"
        return
    if context != T_CTX or layers != L_LAYERS:
        T_CTX, L_LAYERS = context, layers
        WORKLOAD = f"llama31_8b_decode_{T_CTX}_ctx_{L_LAYERS}_layers"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["aoh", "reference"], default="aoh")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-calls", type=int, default=10)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-classifier", action="store_true")
    ap.add_argument("--prefill-only", action="store_true", help="only the prefill sample (profiling)")
    ap.add_argument("--whole-model", action="store_true",
                    help="only the whole-model decode ms/token (random-init Llama-3.1-8B, --context tokens)")
    ap.add_argument("--prefill-full", type=int, default=0, metavar="CHUNK",
                    help="only the full 64K chunked prefill at this chunk size")
    ap.add_argument("--context", type=int, default=131072, help="cached tokens (profiling cases)")
    ap.add_argument("--layers", type=int, default=32, help="layers (profiling cases)")
    ap.add_argument("--workload", choices=["llama31_8b_decode_128k", "qwen3_8b_decode_256k_b8"],
                    default="llama31_8b_decode_128k",
                    help="decode workload; the second is the 8-sequence 256K strong-scaling case")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="N > 1: output gather by peer stores from the decode kernel, or NCCL all-gather")
    args = ap.parse_args()
    _set_workload(args.context, args.layers, args.workload)
    if args.warmup < 3 and args.impl == "aoh":
        print("note: --warmup raised to 3", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.prefill_only:
        import torch
        torch.cuda.set_device(0)
        _, bf16_peak, _ = measured_peaks()
        print(json.dumps({"prefill": prefill_sample(torch, torch.device("cuda", 0), bf16_peak)}), flush=True)
        return 0
    if args.whole_model:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps({"whole_model": whole_model(torch, torch.device("cuda", 0), context=args.context)}),
              flush=True)
        return 0
    if args.prefill_full:
        import torch
        torch.cuda.set_device(0)
        _, bf16_peak, _ = measured_peaks()
        print(json.dumps({"prefill": prefill_full(torch, torch.device("cuda", 0), bf16_peak, args.prefill_full)}),
              flush=True)
        return 0
    return run_aoh(args)


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python3
"""Benchmark: head-mixed decode attention, microseconds per (layer, sequence).

Headline workload (one step = one decode token through every layer's attention):
  Llama-3.1-8B attention shapes (32 query heads, 8 KV heads, head_dim 128),
  32 layers, bf16, one sequence per GPU, 131072-token paged context (16-token
  pages), 6 of 8 KV heads streaming per layer (labels seeded uniform), sink 128,
  window 256, KV ~ 0.5*N(0,1), q ~ N(0,1).  Synthetic data (no checkpoint or
  dataset is needed or available); every (layer, sequence, KV head) unit's
  pages are filled on the device from a generator seeded by the unit, so any
  cache holding that unit -- on any rank -- holds the same values.

  --gpus N > 1 (one process per GPU, torchrun): N sequences (weak scaling),
  the (sequence, KV head) units of every layer partitioned across ranks by the
  longest-processing-time rule on touched KV tokens; each rank attends its
  units and its decode kernel stores every finished unit's output into all
  ranks' output buffers over NVLink (CUDA IPC peer pointers) with a flag per
  unit; a wait kernel per layer is the layer boundary, and the whole step is
  one CUDA graph.  ``--gather nccl`` instead all-gathers the outputs with NCCL
  after each layer, eagerly (the library-collective baseline).

Also on the same line, at every N:
  * ``parity``: one layer decoded eagerly through the partitioned caches and
    the gather, against a cache on the same GPU that owns every unit of that
    layer (same per-unit data, same inputs), max over ranks;
  * ``batched_256k``: the strong-scaling workload -- Qwen3-8B attention shapes,
    36 layers, 8 sequences of 262144 tokens, 6 of 8 KV heads streaming with
    retrieval heads skewed into KV groups 0-1 -- with its own timing, roofline
    and parity;
and at N = 1 only: the decode kernel's HBM roofline, an end-to-end number
through the public API with host buffers, the reference's own eager decode
timed on the host cores (``cpu_baseline``), bf16 prefill TFLOP/s of the 64K
chunked prefill with the reference's prefill timed on a window of its last
chunks, the classifier's labels against the reference's with the reference's
classify timed in the same run, KV memory accounting, and whole-model decode
ms/token.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl aoh|reference]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D, SINK, RECENT, KV_SCALE, SEED = 128, 128, 256, 0.5, 0
WORKLOADS = {
    # headline: one 128K sequence per GPU (weak scaling)
    "llama31_8b_decode_128k": dict(layers=32, hq=32, g=8, context=131072, n_stream=6, skewed=False, batch=0,
                                   metric="decode attn us/layer @128K"),
    # batched long decode across GPUs: 8 sequences in total (strong scaling)
    "qwen3_8b_decode_256k_b8": dict(layers=36, hq=32, g=8, context=262144, n_stream=6, skewed=True, batch=8,
                                    metric="decode attn us/(layer*sequence) @256K batch 8"),
}
MAIN = "llama31_8b_decode_128k"
BATCHED = "qwen3_8b_decode_256k_b8"
# profiled DRAM bytes per decode launch at 128K, valid while the decode sources are unchanged
TRAFFIC_PROFILE = ROOT / "profiles" / "decode_bf16_128k_dram.md"
DECODE_SOURCES = ["aoh_b200/csrc/decode_sm100.cu", "aoh_b200/csrc/common.cuh", "aoh_b200/csrc/page_layout.cuh"]


# ----------------------------------------------------------------------------
# workload description (shared by both arms, so their config keys are equal)
# ----------------------------------------------------------------------------

def workload(name: str, context: int | None = None, layers: int | None = None) -> dict:
    w = dict(WORKLOADS[name], name=name)
    if context and context != w["context"] or layers and layers != w["layers"]:
        w["context"] = context or w["context"]
        w["layers"] = layers or w["layers"]
        w["name"] = f"{name}_ctx{w['context']}_layers{w['layers']}"
    return w


def n_sequences(w: dict, world: int) -> int:
    return w["batch"] or world


def labels_of(w: dict) -> np.ndarray:
    from aoh_b200 import synthetic as syn
    f = syn.labels_skewed if w["skewed"] else syn.labels_uniform
    return f(SEED, w["layers"], w["g"], w["n_stream"])


def decode_layer_bytes(T: int, n_ret_units: int, n_str_units: int, B: int, hq: int) -> int:
    """Algorithmic HBM bytes of one decode launch (one layer): K+V rows read
    (retrieval: T cached keys; streaming: min(T, sink+recent)), the new K/V row
    read once and written once per unit, q read, output written, page ids read."""
    row = 2 * D * 2  # K + V, bf16
    kv = n_ret_units * T * row + n_str_units * min(T, SINK + RECENT) * row
    new = (n_ret_units + n_str_units) * row * 2
    qo = 2 * B * hq * D * 2
    tables = n_ret_units * (-(-T // 16)) * 4 + n_str_units * ((SINK + RECENT) // 16) * 4
    return kv + new + qo + tables


def line_config(w: dict, world: int) -> dict:
    B = n_sequences(w, world)
    n_ret = w["g"] - w["n_stream"]
    step_gb = w["layers"] * decode_layer_bytes(w["context"], n_ret * B, w["n_stream"] * B, B, w["hq"]) / 1e9
    return {"workload": w["name"], "layers": w["layers"], "sequences": B, "context": w["context"],
            "q_heads": w["hq"], "kv_heads": w["g"], "head_dim": D, "page": 16,
            "streaming_kv_heads": f"{w['n_stream']}/{w['g']}" + (" (skewed to groups 0-1)" if w["skewed"] else ""),
            "sink": SINK, "window": RECENT, "parallelism": f"units{world}" if world > 1 else "single",
            "l2": f"no flush: {step_gb:.2f} GB of KV per step (all ranks) >> 126 MB L2"}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def decode_sources_sha16() -> str:
    h = hashlib.sha256()
    for f in DECODE_SOURCES:
        h.update((ROOT / f).read_bytes())
    return h.hexdigest()[:16]


def profiled_traffic(context: int):
    """(bytes per launch, note) from the committed ncu capture of the decode
    kernel at 128K, only while the decode sources still hash to the profiled ones."""
    if context != 131072 or not TRAFFIC_PROFILE.exists():
        return None, "no capture for this context"
    txt = TRAFFIC_PROFILE.read_text()
    m = re.search(r"dram_bytes_per_launch = (\d+)", txt)
    s = re.search(r"decode_sources_sha16 = ([0-9a-f]{16})", txt)
    if not m or not s:
        return None, "capture summary incomplete"
    if s.group(1) != decode_sources_sha16():
        return None, f"capture predates the current decode sources ({s.group(1)})"
    return int(m.group(1)), f"ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch at 128K ({TRAFFIC_PROFILE.name})"


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
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


def clock_sampler(torch, dev):
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "") or "")
    return ClockSampler(("GPU-" + uuid) if uuid and not uuid.startswith("GPU-") else (uuid or dev.index))


# ----------------------------------------------------------------------------
# CPU baselines: the reference's own eager code (baseline/_ref), else the port
# ----------------------------------------------------------------------------

def _reference_or_none():
    try:
        from oracle import ref_driver
        return ref_driver, ref_driver.load(), None
    except Exception as e:  # not installed / does not import: the numpy port stands in
        return None, None, f"{type(e).__name__}: {e}"


def cpu_decode_layer(w: dict, warmup: int, steps: int, budget_s: float):
    """One layer's decode step at the workload's context on the host cores:
    the reference's patched forward over its AoHKVCache (kind "reference"),
    or the numpy restatement of it (kind "port") when the reference is not
    installed.  Warm-up calls, then up to ``steps`` timed calls within
    ``budget_s`` (at least one).  Returns a dict."""
    rd, ref, why = _reference_or_none()
    if ref is not None:
        cores = rd.use_all_cores()
        call = rd.decode_layer_call(ref, num_q=w["hq"], num_kv=w["g"], n_stream=w["n_stream"],
                                    context=w["context"], sink=SINK, recent=RECENT, kv_scale=KV_SCALE, seed=SEED)
        kind, what = "reference", ("the reference's own make_aoh_forward + AoHKVCache (eval/efficiency/"
                                   "benchmark_llama31.py), eager torch on the CPU")
    else:
        from threadpoolctl import threadpool_limits
        from oracle import aoh_oracle as orc
        cores = os.cpu_count() or 1
        threadpool_limits(limits=cores)
        rng = np.random.Generator(np.random.PCG64(SEED))
        labels = np.ones((1, w["g"]))
        labels[0, :w["n_stream"]] = 0.0
        cache = orc.OracleKVCache(1, labels, SINK, RECENT, "bf16")
        nr, ns, T, bf = cache.n_ret[0], cache.n_str[0], w["context"], orc.bf16_round
        cache.full_k[0] = bf(rng.standard_normal((1, nr, T, D), dtype=np.float32) * KV_SCALE)
        cache.full_v[0] = bf(rng.standard_normal((1, nr, T, D), dtype=np.float32) * KV_SCALE)
        keep = min(T, SINK + RECENT)
        cache.stream_k[0] = bf(rng.standard_normal((1, ns, keep, D), dtype=np.float32) * KV_SCALE)
        cache.stream_v[0] = bf(rng.standard_normal((1, ns, keep, D), dtype=np.float32) * KV_SCALE)
        cache.kv_seq_len = T
        q = bf(rng.standard_normal((1, 1, w["hq"], D), dtype=np.float32))
        kk = bf(rng.standard_normal((1, 1, w["g"], D), dtype=np.float32) * KV_SCALE)
        vv = bf(rng.standard_normal((1, 1, w["g"], D), dtype=np.float32) * KV_SCALE)
        call = lambda: orc.layer_attention(cache, 0, q, kk, vv)  # noqa: E731
        kind, what = "port", f"numpy restatement of the reference's eager AoHKVCache forward (reference unavailable: {why})"
    t_start = time.perf_counter()
    for _ in range(max(1, warmup)):
        call()
        if time.perf_counter() - t_start > budget_s / 2:
            break
    times = []
    t0 = time.perf_counter()
    while len(times) < max(1, steps):
        s = time.perf_counter()
        call()
        times.append(time.perf_counter() - s)
        if time.perf_counter() - t0 > budget_s:
            break
    us = float(np.median(times)) * 1e6
    return {"us": us, "cores": cores, "kind": kind, "calls": len(times), "what": what,
            "total_s": float(sum(times))}


def cpu_prefill_window(chunk: int = 256, n_chunks: int = 3, context: int = 65536, budget_s: float = 60.0):
    """The reference's own prefill (Qwen2 patched forward, one layer, 2 of 4 KV
    heads streaming) over the last ``n_chunks`` chunks of a ``context``-token
    chunked prefill; the first chunk warms up (its large temporaries fault in)
    and the rest are timed.  Returns (seconds, masked-in flops, chunks timed,
    cores, kind) or None when the reference is not installed (the port has no
    prefill path of comparable cost)."""
    from aoh_b200.metrics import attention_flops
    rd, ref, why = _reference_or_none()
    if ref is None:
        return None, why
    cores = rd.use_all_cores()
    past0 = context - n_chunks * chunk
    calls = rd.prefill_chunk_calls(ref, past=past0, chunk=chunk, n_chunks=n_chunks, sink=SINK, recent=RECENT,
                                   seed=SEED)
    calls[0]()
    secs, flops, done = 0.0, 0, 0
    t_all = time.perf_counter()
    for i, call in enumerate(calls[1:], start=1):
        s = time.perf_counter()
        call()
        secs += time.perf_counter() - s
        past = past0 + i * chunk
        flops += 7 * 2 * (attention_flops(chunk, past, True, SINK, RECENT) + attention_flops(chunk, past, False, SINK, RECENT))
        done += 1
        if time.perf_counter() - t_all > budget_s:
            break
    return (secs, flops, done, cores, "reference"), None


# ----------------------------------------------------------------------------
# reference arm
# ----------------------------------------------------------------------------

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    w = workload(args.workload, args.context, args.layers)
    r = cpu_decode_layer(w, warmup=args.warmup, steps=args.steps, budget_s=150.0)
    us = r["us"]
    sample = (f"{r['calls']} timed decode steps of one layer of one sequence at {w['context']} tokens ({r['what']}, "
              f"{r['cores']} threads; median); a step is one layer of one sequence, whose cost does not depend on "
              f"how many sequences the job holds")
    line = {
        "impl": "reference", "metric": w["metric"], "value": round(us, 1), "unit": "us/layer",
        "n_gpus": args.gpus, "steps": r["calls"], "warmup": args.warmup, "ms_per_step": round(us / 1000, 3),
        "higher_is_better": False, "scaling": "strong" if w["batch"] else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "config": line_config(w, world),
        "cpu_baseline": {"value": round(us, 1), "unit": "us/layer", "cores": r["cores"], "kind": r["kind"],
                         "sample": sample},
        "e2e": {"value": round(us, 1), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# GPU arm: one decode workload (fill, parity, graph, timing, e2e)
# ----------------------------------------------------------------------------

def unit_seed(l: int, b: int, g: int) -> int:
    return (SEED * 1_000_003 + (l * 4096 + b) * 64 + g) & 0x7FFFFFFFFFFF


def fill_units(torch, cache, layer_offset: int = 0) -> None:
    """Fill every page each stored unit owns, in the unit's own page order, from
    a generator seeded by (layer + layer_offset, sequence, KV head): two caches
    holding the same unit with the same page count hold the same values."""
    pv = cache.pool_view()
    gen = torch.Generator(device=cache.device)
    for l in range(cache.num_layers):
        for b in range(cache.batch):
            for g in range(cache.num_kv_heads):
                if cache.owned is not None and not cache.owned[l, b, g]:
                    continue
                pages = cache.unit_pages(l, b, g)
                if not pages:
                    continue
                gen.manual_seed(unit_seed(l + layer_offset, b, g))
                vals = torch.randn((len(pages), 2, 16, D), generator=gen, device=cache.device)
                pv.index_copy_(0, torch.tensor(pages, dtype=torch.long, device=cache.device),
                               vals.mul_(KV_SCALE).to(torch.bfloat16))


def run_decode(torch, dist, w: dict, args, world: int, rank: int, dev, peaks: dict, e2e_steps: int,
               gather: str = "peer") -> dict:
    import ctypes as C

    from aoh_b200 import AoHKVCache, _lib, aoh_attention

    L, HQ, G, T = w["layers"], w["hq"], w["g"], w["context"]
    B = n_sequences(w, world)
    labels = labels_of(w)
    owner = np.zeros((L, B, G), dtype=np.int32)
    if world > 1:
        lab_u8 = np.ascontiguousarray(labels >= 0.5, dtype=np.uint8)
        _lib.check(_lib.lib().aoh_partition(lab_u8.ctypes.data_as(C.POINTER(C.c_uint8)), L, B, G, T, SINK, RECENT,
                                            world, owner.ctypes.data_as(C.POINTER(C.c_int32))), "aoh_partition")
    owned = (owner == rank).astype(np.uint8)
    clock_steps = 5 * 400  # pages reserved for the clock warm-up below
    strict_steps = min(args.steps, 100) if world > 1 and gather == "peer" else 0
    max_ctx = T + args.warmup + args.steps + 2 * (e2e_steps + 2) + 8 + clock_steps + 16 + 2 * (strict_steps + 4)
    cache = AoHKVCache(labels, HQ, batch=B, sink_size=SINK, recent_size=RECENT, max_context=max_ctx,
                       dtype=torch.bfloat16, device=dev, owned=owned, reserve_all=True)
    fill_units(torch, cache)
    cache.kv_seq_len = T
    gen = torch.Generator(device=dev).manual_seed(SEED + 1)  # the same inputs on every rank
    q = torch.randn((L, B, 1, HQ, D), generator=gen, device=dev).to(torch.bfloat16)
    kn = (torch.randn((L, B, 1, G, D), generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16)
    vn = (torch.randn((L, B, 1, G, D), generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16)
    peer = None
    if world > 1 and gather == "peer":
        from aoh_b200.gather import PeerGather
        peer = PeerGather(cache, out_shape=(L, B, 1, HQ, D))
        out = peer.out  # decoded straight into the shared output region
        out.zero_()
    else:
        out = torch.zeros((L, B, 1, HQ, D), dtype=torch.bfloat16, device=dev)

    # NCCL gather plumbing (--gather nccl): pack owned (b, g) head groups, all-gather, unpack
    if world > 1 and peer is None:
        grp = HQ // G
        packs, unpack = [], []
        max_units = max(int((owner[l] == r).sum()) for l in range(L) for r in range(world))
        for l in range(L):
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

    def layer(l, q_l, k_l, v_l, o_l, advance=True):
        aoh_attention(cache, l, q_l, k_l, v_l, out=o_l, advance=advance)
        if world > 1 and peer is None:
            flat = o_l.view(B * G, -1)
            mine = flat.index_select(0, packs[l])
            dist.all_gather_into_tensor(gathered, mine)
            src, dst = unpack[l]
            flat.index_copy_(0, dst, gathered.index_select(0, src))
        elif peer is not None:
            peer.wait(l, past_len=cache.kv_seq_len)

    # ---- parity: one layer decoded eagerly through this rank's cache and the
    # gather, against a cache on this GPU that owns every unit of the layer ----
    lp = L // 2
    layer(lp, q[lp], kn[lp], vn[lp], out[lp], advance=False)
    ref = AoHKVCache(labels[lp:lp + 1], HQ, batch=B, sink_size=SINK, recent_size=RECENT, max_context=max_ctx,
                     dtype=torch.bfloat16, device=dev, reserve_all=True)
    fill_units(torch, ref, layer_offset=lp)
    ref.kv_seq_len = T
    want = aoh_attention(ref, 0, q[lp], kn[lp], vn[lp], advance=False)
    torch.cuda.synchronize()
    perr = torch.tensor([(out[lp].float() - want.float()).abs().max().item(),
                         float(ref.device_status() | cache.device_status())], device=dev)
    del ref, want
    torch.cuda.empty_cache()
    if world > 1:
        dist.all_reduce(perr, op=dist.ReduceOp.MAX)
    parity = {"layer": lp, "max_abs_err": float(perr[0]), "tol": 2e-2,
              "ok": bool(perr[0] <= 2e-2 and perr[1] == 0),
              "against": "a cache on each rank's GPU owning every unit of the layer (same per-unit data and "
                         "inputs), after the eager decode through this rank's partition and the output gather; "
                         "max over ranks"}

    graph = None
    if world == 1 or peer is not None:
        from aoh_b200.graph import DecodeStepGraph
        # the step's layers are independent (every layer's q, k, v given up front),
        # so each layer's gather wait overlaps the next layers' decode kernels
        graph = DecodeStepGraph(cache, q, kn, vn, out,
                                max_steps=args.warmup + args.steps + e2e_steps + 8 + clock_steps, gather=peer,
                                overlap_gather=peer is not None)

    def step():
        if graph is not None:
            graph.replay()
            return
        for l in range(L):
            layer(l, q[l], kn[l], vn[l], out[l])

    def barrier():
        if world > 1:
            dist.barrier()

    # ---------------- device-timed region ----------------
    clocks = clock_sampler(torch, dev)
    clocks.start()  # sampling runs through warm-up and the timed steps (the same steady load)
    for _ in range(args.warmup):
        step()
    # more warm-up until nvidia-smi reports under load (2 s at most); ranks are
    # coupled step by step, so all of them decide together and run the same steps
    t_w = time.perf_counter()
    for _ in range(clock_steps // 5):
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
    host_us = (time.perf_counter() - h0) * 1e6 / (args.steps * L)
    ev1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    status = cache.device_status()
    assert status == 0, f"device-side check tripped ({status})"

    # the same step with the layer boundary kept: every layer's wait before the
    # next layer's decode (what a model whose next layer reads this output needs)
    boundary = None
    if strict_steps:
        sg = DecodeStepGraph(cache, q, kn, vn, out, max_steps=strict_steps + 4, gather=peer)
        for _ in range(3):
            sg.replay()
        barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(strict_steps):
            sg.replay()
        s1.record()
        torch.cuda.synchronize()
        sms = s0.elapsed_time(s1) / strict_steps
        t = torch.tensor([sms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sms = float(t.item())
        boundary = {"strict_us_layer_seq": round(sms * 1000.0 / (L * B), 3),
                    "overlapped_us_layer_seq": round(ms * 1000.0 / (L * B), 3), "strict_steps": strict_steps,
                    "note": "value overlaps each layer's gather wait with the next layers' decode (the step's "
                            "layers are independent); strict waits for every rank's units after each layer"}
        sg = None
        assert cache.device_status() == 0

    # roofline of this rank's decode kernel (the only kernel in the N=1 step)
    T_mid = T0 + args.steps // 2
    n_ret_units = int(((labels >= 0.5)[:, None, :].repeat(B, 1) & (owned > 0)).sum()) // L
    n_str_units = int(owned.sum()) // L - n_ret_units
    bytes_launch = decode_layer_bytes(T_mid, n_ret_units, n_str_units, B, HQ)
    launch_us = ms * 1000.0 / L
    achieved = bytes_launch / (launch_us * 1e-6) / 1e9

    # ---------------- end to end through the public API, host buffers ----------------
    e2e = None
    if e2e_steps > 0:
        qh = q.cpu().pin_memory()
        kh = kn.cpu().pin_memory()
        vh = vn.cpu().pin_memory()
        oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        qd, kd, vd = q, kn, vn  # the graph's (or the eager loop's) input buffers

        def e2e_step():
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
            step()
            oh.copy_(out, non_blocking=True)

        e2e_step()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1) / e2e_steps
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": round(ems * 1000.0 / (L * B), 2), "unit": "us/layer",
               "h2d_bytes_per_step": int(q.numel() + kn.numel() + vn.numel()) * 2,
               "d2h_bytes_per_step": int(out.numel()) * 2}

    from aoh_b200 import metrics
    kv_mem = {"pool_gb_granted_this_rank": round(metrics.kv_pool_gb(cache), 3),
              "analytical_gb_aoh": round(metrics.kv_storage_gb_aoh(
                  [int((labels[l] >= 0.5).sum()) * B for l in range(L)],
                  [int((labels[l] < 0.5).sum()) * B for l in range(L)], D, T, SINK, RECENT), 3),
              "analytical_gb_full": round(metrics.kv_storage_gb_full(L, G * B, D, T), 3),
              "note": "analytical: the reference's kv_storage_gb_aoh / _full formulas (all sequences, all ranks) "
                      "at the context length; granted: pages this rank's pool holds (reserved for the whole run)"}

    graphed = graph is not None
    # kernels of this library per timed step: a decode kernel per layer (plus a
    # gather wait per layer when peers are attached) and the length advance
    per_step = L * (2 if peer is not None else 1) + (1 if graphed else 0)
    graph = None
    if peer is not None:
        torch.cuda.synchronize()
        peer.close()
    cache.close()
    del cache, q, kn, vn, out
    torch.cuda.empty_cache()
    return {"ms": ms, "us_layer_seq": ms * 1000.0 / (L * B), "B": B, "launch_us": launch_us,
            "bytes_launch": bytes_launch, "achieved": achieved, "e2e": e2e, "parity": parity, "clocks": clk,
            "host_us": host_us, "gpu_launches": per_step * args.steps, "kv_memory": kv_mem,
            "launch_mode": "cuda_graph+pdl" if graphed else "eager+pdl",
            "gather": None if world == 1 else ("nvlink_peer_stores" if peer is not None else "nccl_all_gather"),
            "layer_boundary": boundary}


# ----------------------------------------------------------------------------
# N = 1 extras: prefill, classifier, whole model
# ----------------------------------------------------------------------------

def prefill_sample(torch, dev, peaks, C: int = 4096):
    """bf16 prefill TFLOP/s on a bounded sample of the 64K chunked prefill
    (Qwen2.5-7B shapes, one layer, 2 of 4 KV heads streaming): the last chunk of
    C tokens (4096: at 61440 cached tokens, three launches of about 2 ms, so the
    burst peak; 256: at 65280, the call the 256-token prefill repeats)."""
    from aoh_b200 import AoHKVCache, aoh_attention
    from aoh_b200.metrics import attention_flops
    Hq, Gq, past = 28, 4, 65536 - C
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
    cache.close()
    return {"tflops": round(tf, 2), "frac": round(tf / peaks["bf16"], 4), "peak": "bf16 burst (3 launches)",
            "ms": round(sec * 1e3, 3), "flops": flops,
            "sample": f"1 layer, last {C}-token chunk at {past} cached tokens, Qwen2.5-7B heads, 2/4 streaming"}


def prefill_full(torch, dev, peaks, chunk: int, context: int = 65536, layers: int = 28):
    """Chunked prefill to ``context`` tokens through every layer: Qwen2.5-7B
    shapes (28 query / 4 KV heads, head_dim 128), bf16, 2 of 4 KV heads streaming
    per layer (seeded), sink 128, window 256, q/k/v ~ N(0,1) generated once per
    layer and reused for every chunk (values do not change the work).  The whole
    prefill runs twice: the first pass warms up (kernel attributes, split-KV
    scratch sized for every chunk), the second is timed with CUDA events.  Flops
    count only masked-in (query, key) pairs; the timed region lasts about half a
    second, so the fraction is of the sustained bf16 peak."""
    from aoh_b200 import AoHKVCache, aoh_attention
    from aoh_b200 import synthetic as syn
    from aoh_b200.metrics import attention_flops
    Hq, Gq = 28, 4
    grp = Hq // Gq
    labels = syn.labels_uniform(31, layers, Gq, 2)
    cache = AoHKVCache(labels, Hq, batch=1, sink_size=SINK, recent_size=RECENT, max_context=context,
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
        f_ret = attention_flops(chunk, start, True, SINK, RECENT)
        f_str = attention_flops(chunk, start, False, SINK, RECENT)
        for l in range(layers):
            n_ret = int((labels[l] >= 0.5).sum())
            flops += grp * (n_ret * f_ret + (Gq - n_ret) * f_str)
    tf = flops / sec / 1e12
    cache.close()
    return {"chunk": chunk, "tflops": round(tf, 2), "frac": round(tf / peaks["bf16_sustained"], 4),
            "peak": "bf16 sustained", "seconds": round(sec, 4), "flops": flops, "calls": layers * (context // chunk)}


def prefill_block(torch, dev, peaks):
    from aoh_b200.metrics import attention_flops
    res = {"workload": "qwen25_7b_chunked_prefill_64k (28 layers, 28/4 heads, 2/4 streaming, bf16)",
           "chunk_4096": prefill_full(torch, dev, peaks, 4096),
           "chunk_256": prefill_full(torch, dev, peaks, 256),
           "kernel_sample": prefill_sample(torch, dev, peaks)}
    win, why = cpu_prefill_window()
    if win is None:
        res["cpu_baseline"] = {"value": None, "unavailable": why}
        return res
    secs, wflops, done, cores, kind = win
    total = res["chunk_256"]["flops"]
    extrap = secs * total / wflops
    res["cpu_baseline"] = {
        "value": round(extrap, 1), "unit": "s (full 64K prefill at chunk 256, extrapolated)", "cores": cores,
        "kind": kind, "tflops": round(wflops / secs / 1e12, 4),
        "sample": (f"{done} 256-token chunks of one layer ending at 65536 tokens (after one untimed chunk), the "
                   f"reference's own Qwen2 patched forward on the CPU ({cores} threads): {secs:.2f} s for "
                   f"{wflops:.3e} masked-in flops, scaled to the full prefill's {total:.3e} flops (28 layers, "
                   f"every chunk) -- the shorter early chunks run at a lower CPU rate, so this favours the CPU"),
        "vs_gpu_chunk_256": round(extrap / res["chunk_256"]["seconds"], 1)}
    return res


def classifier_block(torch, dev):
    """AoH classifier on seeded Qwen2.5-7B-shaped projections (28 layers, 28/4
    heads, hidden 3584, bf16): GPU effective ranks -> labels vs the reference's
    labels stored in tests/golden/cls_qwen25_7b.npz, both modes, 3 aggregations
    x 3 sparsities; and the reference's own AoHClassifier.classify on the same
    weights, timed on the host cores in this run (its labels checked too)."""
    from aoh_b200 import classifier as clf
    from aoh_b200 import synthetic as syn
    z = np.load(ROOT / "tests" / "golden" / "cls_qwen25_7b.npz")
    L, H, Gk, Dh, dm = 28, 28, 4, 128, 3584
    bits = [syn.classifier_weights(0, l, H, Gk, Dh, dm) for l in range(L)]
    wq = torch.empty((L, H * Dh, dm), dtype=torch.bfloat16, device=dev)
    wk = torch.empty((L, Gk * Dh, dm), dtype=torch.bfloat16, device=dev)
    for l in range(L):
        wq[l].copy_(torch.from_numpy(bits[l][0].astype(np.int16)).view(torch.bfloat16))
        wk[l].copy_(torch.from_numpy(bits[l][1].astype(np.int16)).view(torch.bfloat16))
    rd, ref, why = _reference_or_none()
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
        r = {"layer_decisions_equal": f"{match}/{total}", "differ_below_ref_fp32_noise": sub_noise,
             "max_rel_rank_err": rel, "gpu_seconds": round(sec, 4)}
        if ref is not None:
            cores = rd.use_all_cores()
            secs, labels = rd.classify_seconds(ref, [b[0] for b in bits], [b[1] for b in bits], H, Gk, dm,
                                               binary=mode == "binary", agg="mean", sparsity=0.5)
            r["cpu_baseline"] = {"value": round(secs, 3), "unit": "s per classify (28 x 28 heads)", "cores": cores,
                                 "kind": "reference",
                                 "sample": "the reference's own AoHClassifier.classify (agg mean, sparsity 0.5) "
                                           "on the same bf16 weights, on the host cores in this run",
                                 "labels_equal_stored": bool(np.array_equal(labels, z[f"{mode}_mean_sp0.5_labels"]))}
            r["vs_cpu"] = round(secs / sec, 1)
        else:
            r["cpu_baseline"] = {"value": None, "unavailable": why}
        res[mode] = r
    return res


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
                      max_position_embeddings=context + 2 * decode_steps + 128)
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
           "cache": "synthetic K/V of the context length (no prefill)",
           "reference_table11_ms_per_token_128k": {"full": 199.55, "aoh_sp0.75": 49.90,
                                                   "note": "published, hardware not stated"}}
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
    cache = make_cache(max_context=context + 2 * decode_steps + 16)
    cache.paged.reserve(context + 2 * decode_steps + 16)
    pv = cache.paged.pool_view()
    for i in range(0, pv.shape[0], 65536):
        sl = pv[i:i + 65536]
        sl.copy_((torch.randn(sl.shape, generator=gen, device=dev) * KV_SCALE).to(torch.bfloat16))
    cache.kv_seq_len = context
    ms = decode(cache)
    # the same decode step captured once as a CUDA graph (ModelDecodeGraph) and replayed per token
    from aoh_b200.hf import ModelDecodeGraph
    g = ModelDecodeGraph(model, cache, max_steps=decode_steps + 4)
    times = []
    with torch.no_grad():
        g.step(ids[:, 0])  # warm-up replay
        for t in range(decode_steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.step(ids[:, 1 + t])
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
    gms = float(np.median(times))
    g = None
    res["aoh_sp0.75"] = {"decode_ms_per_token": round(gms, 3), "eager_decode_ms_per_token": round(ms, 3),
                         "launch": "whole decode step captured as one CUDA graph (ModelDecodeGraph); eager: "
                                   "transformers' per-layer Python, the same kernels",
                         "kv_pool_gb": round(cache.paged.pool.numel() / 1e9, 3)}
    ms = gms
    assert cache.paged.device_status() == 0, "device-side check tripped"
    if full_baseline:
        res["decode_speedup_vs_full"] = round(res["full_attention"]["decode_ms_per_token"] / ms, 2)
    cache.paged.close()
    del model, cache
    torch.cuda.empty_cache()
    return res


# ----------------------------------------------------------------------------
# GPU arm: the line
# ----------------------------------------------------------------------------

def run_aoh(args):
    import torch
    import torch.distributed as dist

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
    import aoh_b200  # noqa: F401  (loads libaoh.so; fails loudly without it)

    peaks = measured_peaks()
    w = workload(args.workload, args.context, args.layers)
    main = run_decode(torch, dist, w, args, world, rank, dev, peaks, args.e2e_steps, args.gather)
    batched = None
    if not args.no_batched and w["name"] != BATCHED and args.gather == "peer":
        wb = workload(BATCHED)
        b = run_decode(torch, dist, wb, args, world, rank, dev, peaks, 0)
        batched = {"metric": wb["metric"], "value": round(b["us_layer_seq"], 3), "unit": "us/(layer*sequence)",
                   "ms_per_step": round(b["ms"], 4), "steps": args.steps, "scaling": "strong",
                   "config": line_config(wb, world),
                   "roofline_this_rank": {"bound": "hbm", "achieved": round(b["achieved"], 1), "peak": peaks["hbm"],
                                          "unit": "GB/s", "frac": round(b["achieved"] / peaks["hbm"], 4),
                                          "bytes_per_launch": b["bytes_launch"],
                                          "avg_launch_us": round(b["launch_us"], 3)},
                   "parity": b["parity"], "clocks": b["clocks"], "kv_memory": b["kv_memory"],
                   "gpu_launches": b["gpu_launches"], "layer_boundary": b["layer_boundary"]}

    extras = {}
    cpu = None
    if rank == 0 and world == 1:
        if not args.no_prefill:
            extras["prefill"] = prefill_block(torch, dev, peaks)
        if not args.no_classifier:
            extras["labels_exact"] = classifier_block(torch, dev)
        if not args.no_whole_model:
            extras["whole_model"] = whole_model(torch, dev)
        if args.cpu_calls > 0:
            r = cpu_decode_layer(w, warmup=1, steps=args.cpu_calls, budget_s=30.0)
            cpu = {"value": round(r["us"], 1), "unit": "us/layer", "cores": r["cores"], "kind": r["kind"],
                   "sample": f"{r['calls']} decode steps of one layer of one sequence at {w['context']} tokens "
                             f"({r['what']}; median, after one untimed step)"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    traffic, traffic_note = profiled_traffic(w["context"])
    line = {
        "metric": w["metric"], "value": round(main["us_layer_seq"], 3), "unit": "us/layer", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(main["ms"], 4), "higher_is_better": False,
        "scaling": "strong" if w["batch"] else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": line_config(w, world),
        "tokens_per_s": round(main["B"] / (main["ms"] / 1000.0), 2),
        "roofline": {"bound": "hbm", "achieved": round(main["achieved"], 1), "peak": peaks["hbm"], "unit": "GB/s",
                     "frac": round(main["achieved"] / peaks["hbm"], 4), "traffic": traffic,
                     "traffic_source": traffic_note, "peak_source": peaks["source"] + " (copy bandwidth)",
                     "kernel": "decode_bf16_kernel", "bytes_per_launch": main["bytes_launch"],
                     "avg_launch_us": round(main["launch_us"], 3)},
        "e2e": main["e2e"],
        "cpu_baseline": cpu,
        "parity": main["parity"],
        "gpu_launches": main["gpu_launches"],
        "launch_mode": main["launch_mode"],
        "gather": main["gather"],
        "layer_boundary": main["layer_boundary"],
        "host_enqueue_us_per_layer": round(main["host_us"], 2),
        "clocks": main["clocks"],
        "kv_memory": main["kv_memory"],
        "batched_256k": batched,
        **extras,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["aoh", "reference"], default="aoh")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-calls", type=int, default=5)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-classifier", action="store_true")
    ap.add_argument("--no-whole-model", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the 8-sequence 256K strong-scaling workload")
    ap.add_argument("--prefill-only", action="store_true", help="only the prefill sample (profiling)")
    ap.add_argument("--chunk", type=int, default=4096, choices=[256, 4096],
                    help="--prefill-only: the sample's chunk (the last chunk of the 64K prefill)")
    ap.add_argument("--whole-model", action="store_true",
                    help="only the whole-model decode ms/token (random-init Llama-3.1-8B, --context tokens)")
    ap.add_argument("--prefill-full", type=int, default=0, metavar="CHUNK",
                    help="only the full 64K chunked prefill at this chunk size")
    ap.add_argument("--classifier-only", action="store_true",
                    help="only the classifier on the Qwen2.5-7B-shaped projections (labels, timing)")
    ap.add_argument("--context", type=int, default=0, help="cached tokens (profiling cases; default: the workload's)")
    ap.add_argument("--layers", type=int, default=0, help="layers (profiling cases; default: the workload's)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=MAIN,
                    help="headline decode workload; the 256K batch-8 one also runs after it unless --no-batched")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="N > 1: output gather by peer stores from the decode kernel, or NCCL all-gather")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "aoh":
        print("note: --warmup raised to 3", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.prefill_only or args.whole_model or args.prefill_full or args.classifier_only:
        import torch
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        peaks = measured_peaks()
        if args.prefill_only:
            res = {"prefill": prefill_sample(torch, dev, peaks, args.chunk)}
        elif args.whole_model:
            res = {"whole_model": whole_model(torch, dev, context=args.context or 131072)}
        elif args.classifier_only:
            res = {"labels_exact": classifier_block(torch, dev)}
        else:
            res = {"prefill": prefill_full(torch, dev, peaks, args.prefill_full)}
        print(json.dumps(res), flush=True)
        return 0
    return run_aoh(args)


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python
"""Benchmark of the sqmix attention-mixer hot path (BASELINE.json metric).

Workload: one decode token through all 10 full-attention layers
of qwen35moe at 172032 keys per layer -- per layer the q4_0 KV append of the new
token (with fused partial RoPE) and split-KV FlashAttention over the q4_0 cache
with the sigmoid output gate.  Inputs are seeded synthetic N(0,1) tensors with the
reference's shapes (no model weights are involved in the mixer).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sqmix|reference]

N > 1 (under torchrun): the 172032 keys of every layer are split across the ranks;
each rank attends over its slice and the (O, LSE) partials are all-gathered over
NCCL and merged before the gate (strong scaling: total work fixed).

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "sqwen-moe-3090_b200"))

N_LAYERS = 10
N_KV = 172032
# DRAM bytes of one decode launch at N_KV keys, from one ncu capture
# (profiles/fa_decode_kernel_172k.txt): 99.17 MB read + 3.65 MB written.
FA_NCU_TRAFFIC = 102_818_048
HEAD_DIM = 256
N_HEAD = 16
N_HEAD_KV = 2
N_ROT = 64
FREQ_BASE = 1e7
METRIC = "attn-mixer us/token @172K ctx decode (10 full-attn layers, q4_0 KV)"
BYTES_PER_KEY = 576  # K + V q4_0 per token per layer


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the burst figure (a kernel timed alone) and its source."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def tensor_peak_sustained():
    """Dense bf16 TFLOP/s held for seconds under the power cap (a kernel timed in a long loop)."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region.

    One streaming ``nvidia-smi --query-gpu ... -lms 100`` process is started on
    entry and ``__enter__`` returns only after its first line has arrived, so the
    sampler is running before the caller starts timing.  ``mark_start`` /
    ``mark_end`` bracket the timed region on the host clock (call them after the
    synchronize on each side); the summary keeps the samples whose arrival time
    lies inside that window, and says how many there were.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 100

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []  # (host time, fields)
        self._proc = None
        self._t = None
        self._first = threading.Event()
        self.t0 = self.t1 = None

    def _read(self):
        for line in self._proc.stdout:
            line = line.strip()
            if line:
                self.samples.append((time.perf_counter(), [x.strip() for x in line.split(",")]))
                self._first.set()
        self._first.set()

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 f"-lms={self.INTERVAL_MS}"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._proc = None
            return self
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()
        self._first.wait(timeout=10)
        return self

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=10)
            except Exception:
                self._proc.kill()
            self._t.join(timeout=10)

    def summary(self):
        inside = [f for t, f in self.samples
                  if self.t0 is not None and self.t1 is not None and self.t0 <= t <= self.t1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "window_ms": None if self.t0 is None or self.t1 is None else (self.t1 - self.t0) * 1e3}
        sm = [float(s[1]) for s in inside if s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in inside if s[2].replace(".", "").isdigit()]
        power = [float(s[3]) for s in inside if s[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in inside:
            for n, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w": float(np.median(power)) if power else None, "reasons": sorted(reasons),
                "samples": len(inside), "window_ms": (self.t1 - self.t0) * 1e3}


# --------------------------------------------------------------------------- #
# CPU legs (oracle): cpu_baseline and --impl reference                          #
# --------------------------------------------------------------------------- #

def cpu_layer_inputs(n_kv: int, seed: int = 0):
    import oracle

    rng = np.random.default_rng(seed)
    k = rng.standard_normal((n_kv, 512), dtype=np.float32)
    v = rng.standard_normal((n_kv, 512), dtype=np.float32)
    kq = oracle.q4_0_quantize(k)
    vq = oracle.q4_0_quantize(v)
    q = rng.standard_normal((1, N_HEAD, HEAD_DIM), dtype=np.float32)
    gate = rng.standard_normal((1, N_HEAD, HEAD_DIM), dtype=np.float32)
    return kq, vq, q, gate


def cpu_layer(kq, vq, q, gate, n_kv):
    """One layer on the CPU restatement: dequantise the q4_0 cache, RoPE Q, attend."""
    import oracle

    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, N_HEAD_KV, HEAD_DIM)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, N_HEAD_KV, HEAD_DIM)
    qr = oracle.rope_text(q, n_kv - 1, FREQ_BASE, N_ROT)
    return oracle.attn(qr, kd, vd, gate, q_pos0=n_kv - 1, scale=1.0 / 16)


def cpu_baseline(budget_s: float = 12.0):
    import oracle

    oracle.build()
    cores = oracle.set_threads(os.cpu_count() or 1)
    kq, vq, q, gate = cpu_layer_inputs(N_KV)
    cpu_layer(kq, vq, q, gate, N_KV)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        cpu_layer(kq, vq, q, gate, N_KV)
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= N_LAYERS:
            break
    per_layer = (time.perf_counter() - t0) / n
    return {"value": per_layer * N_LAYERS * 1e6, "unit": "us/token", "cores": cores, "kind": "port",
            "sample": f"{n} layer(s) of 172032 q4_0 keys (dequant + RoPE + attention + gate), "
                      f"scaled x{N_LAYERS / n:g} to 10 layers; C restatement of the ggml CPU nodes"}


REF_BUDGET_S = 30.0


def run_reference(args, rank: int):
    if rank != 0:
        return None
    import oracle

    oracle.build()
    cores = oracle.set_threads(os.cpu_count() or 1)
    kq, vq, q, gate = cpu_layer_inputs(N_KV)
    for _ in range(min(args.warmup, 3)):
        cpu_layer(kq, vq, q, gate, N_KV)
    # A CPU layer takes ~0.1 s on 16 cores: the timed steps stop after REF_BUDGET_S so
    # that a large --steps (the GPU arm's default) still ends within a minute.
    t0 = time.perf_counter()
    n = 0
    while n < args.steps:
        cpu_layer(kq, vq, q, gate, N_KV)  # one of the 10 layers per step
        n += 1
        if time.perf_counter() - t0 > REF_BUDGET_S:
            break
    per_layer = (time.perf_counter() - t0) / n
    v = per_layer * N_LAYERS * 1e6
    sample = (f"each step = 1 of the 10 layers (172032 q4_0 keys, dequant + RoPE + attention + gate) "
              f"on {cores} threads, scaled x10; {n} of {args.steps} requested steps timed "
              f"(stopped after {REF_BUDGET_S:g} s); C restatement of the ggml CPU nodes "
              "(ggml itself is not in this image)")
    return {"metric": METRIC, "value": v, "unit": "us/token", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "timed_steps": n, "warmup": args.warmup, "ms_per_step": per_layer * 1e3,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1), seed 0",
            "config": {"workload": "config3: decode, 10 layers x 172032 q4_0 keys, 16/2 heads, d=256, n_q=1"},
            "cpu_baseline": {"value": v, "unit": "us/token", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# --------------------------------------------------------------------------- #
# GPU arm                                                                       #
# --------------------------------------------------------------------------- #

def run_gpu(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    import sqmix

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    from sqmix import split_kv

    shard = split_kv.plan(N_KV, world, rank)  # this rank's contiguous key slice
    n_local, k0 = shard.length, shard.start
    cap = shard.capacity
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)

    # ---- resident state: 10 layers of q4_0 K/V for this rank's key slice ------
    kv = sqmix.KvCache(n_layers=N_LAYERS, kv_cap=cap, device=local_rank)
    kc = [kv.k_state(l) for l in range(N_LAYERS)]
    vc = [kv.v_state(l) for l in range(N_LAYERS)]
    chunk = 16384
    for l in range(N_LAYERS):
        for a in range(0, n_local, chunk):
            n = min(chunk, n_local - a)
            kk = torch.randn((n, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
            vv = torch.randn((n, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
            rows = torch.arange(a, a + n, device=dev)
            sqmix.set_rows_q4_0(kk, vv, rows, kc[l], vc[l], cap, rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE,
                                rope_pos_offset=k0)
    # the new token is written at the last position of the last rank's slice
    pos_new = N_KV - 1
    owner = split_kv.owner(N_KV, world, pos_new)
    local_row = pos_new - split_kv.plan(N_KV, world, owner).start
    # The step's inputs share one device buffer (so that the end-to-end measurement
    # moves them with one host-to-device copy): q, gate, k_new, v_new (f32), then the
    # step scalars {n_kv, q_pos0} (i64).
    in_shapes = [(N_LAYERS, 1, N_HEAD, HEAD_DIM)] * 2 + [(N_LAYERS, 1, N_HEAD_KV, HEAD_DIM)] * 2
    in_off = [0]
    for shp in in_shapes:
        in_off.append(in_off[-1] + 4 * shp[0] * shp[1] * shp[2] * shp[3])

    def in_views(buf):
        ts = [buf[in_off[i]:in_off[i + 1]].view(torch.float32).view(shp) for i, shp in enumerate(in_shapes)]
        return ts + [buf[in_off[-1]:in_off[-1] + 16].view(torch.int64)]

    inp = torch.empty(in_off[-1] + 16, dtype=torch.uint8, device=dev)
    q, gate, k_new, v_new, step = in_views(inp)
    for t_, shp in zip((q, gate, k_new, v_new), in_shapes):
        t_.copy_(torch.randn(shp, generator=g, device=dev))
    step.copy_(torch.tensor(list(shard.local_step(N_KV, pos_new)), dtype=torch.int64, device=dev))
    out = torch.empty((N_LAYERS, 1, N_HEAD, HEAD_DIM), device=dev)
    d_nkv, d_qpos = step[0:1], step[1:2]
    d_row = torch.tensor([local_row], dtype=torch.int64, device=dev)
    n_splits = sqmix.lib().sqmix_device_sm_count(local_rank)
    ws = sqmix.new_fa_workspace(1, n_splits, dev)
    torch.cuda.synchronize()

    if world > 1:
        # (O, LSE) partials packed per layer so that one all-gather moves both
        rows = N_HEAD
        pk_loc = torch.empty((N_LAYERS, rows * (HEAD_DIM + 1)), device=dev)
        pk_all = torch.empty((world, rows * (HEAD_DIM + 1)), device=dev)
        o_loc = [pk_loc[l, :rows * HEAD_DIM].view(1, N_HEAD, HEAD_DIM) for l in range(N_LAYERS)]
        l_loc = [pk_loc[l, rows * HEAD_DIM:].view(1, N_HEAD) for l in range(N_LAYERS)]
        # default: the fused peer-memory merge (one kernel per layer, partials read
        # over NVLink); --nccl-merge: all-gather + merge kernel
        peer = None if args.nccl_merge else split_kv.PeerMerge(n_slots=N_LAYERS, rows=N_HEAD, device=dev)

    own = rank == owner  # the rank whose key slice holds the new token appends it (fused)

    def layer(l):
        if world == 1:
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, gate=gate[l], rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, rope_pos_offset=k0, out=out[l],
                                 workspace=ws, n_splits=n_splits, k_new=k_new[l], v_new=v_new[l],
                                 overlap_prev=True)
        else:
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, gate=None, rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, rope_pos_offset=k0, out=o_loc[l],
                                 lse=l_loc[l], workspace=ws, n_splits=n_splits,
                                 k_new=k_new[l] if own else None, v_new=v_new[l] if own else None,
                                 overlap_prev=True)
            if peer is not None:
                peer.merge(o_loc[l], l_loc[l], l, gate=gate[l, 0], out=out[l, 0])
            else:
                dist.all_gather_into_tensor(pk_all, pk_loc[l])
                sqmix.attn_merge_lse(pk_all[:, :rows * HEAD_DIM].view(world, rows, HEAD_DIM),
                                     pk_all[:, rows * HEAD_DIM:], gate=gate[l, 0], out=out[l, 0])

    def step_fn():
        for l in range(N_LAYERS):
            layer(l)

    stream = torch.cuda.current_stream()
    graph = None
    if not args.no_graph:  # N > 1: the NCCL all-gathers are captured too
        s = torch.cuda.Stream()
        s.wait_stream(stream)
        with torch.cuda.stream(s):
            step_fn()  # warm the launch path outside capture
        stream.wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step_fn()
        torch.cuda.synchronize()

    run = graph.replay if graph is not None else step_fn
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    sampler = ClockSampler(local_rank)
    with sampler:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        sampler.mark_start()
        e0.record()
        for _ in range(args.steps):
            run()
        e1.record()
        torch.cuda.synchronize()
        sampler.mark_end()
        ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us_per_token = ms * 1e3 / args.steps
    # per layer: decode + split merge (PDL pair), plus the cross-rank merge_lse for N > 1
    launches_per_step = N_LAYERS * (2 + (1 if world > 1 else 0))

    # ---- dominant kernel alone: flash_attn_ext over each layer in turn ---------
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    reps = max(3, args.steps)
    # (graph-captured so that host launch cost is not mistaken for kernel time)
    def fa_only():
        for l in range(N_LAYERS):
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, gate=gate[l], rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, rope_pos_offset=k0, out=out[l],
                                 workspace=ws, n_splits=n_splits, overlap_prev=True)
    s2 = torch.cuda.Stream()
    s2.wait_stream(stream)
    with torch.cuda.stream(s2):
        fa_only()
    stream.wait_stream(s2)
    torch.cuda.synchronize()
    g_fa = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_fa):
        fa_only()
    g_fa.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g_fa.replay()
    e1.record()
    torch.cuda.synchronize()
    g_fa = None
    fa_us = e0.elapsed_time(e1) * 1e3 / (reps * N_LAYERS)
    sqmix.fa_status(ws)

    # ---- MTP verify (config 3's 2-token query) over the same caches ------------
    mtp = None
    if world == 1:
        q2 = torch.randn((N_LAYERS, 2, N_HEAD, HEAD_DIM), generator=g, device=dev)
        gate2 = torch.randn((N_LAYERS, 2, N_HEAD, HEAD_DIM), generator=g, device=dev)
        out2 = torch.empty((N_LAYERS, 2, N_HEAD, HEAD_DIM), device=dev)
        step2 = torch.tensor([n_local, n_local - 2], dtype=torch.int64, device=dev)
        ws2 = sqmix.new_fa_workspace(2, n_splits, dev)

        def mtp_step():
            for l in range(N_LAYERS):
                sqmix.flash_attn_ext(q2[l], kc[l], vc[l], cap, step2[0:1], step2[1:2], gate=gate2[l],
                                     rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE, out=out2[l], workspace=ws2,
                                     n_splits=n_splits, overlap_prev=True)
        s3 = torch.cuda.Stream()
        s3.wait_stream(stream)
        with torch.cuda.stream(s3):
            mtp_step()
        stream.wait_stream(s3)
        torch.cuda.synchronize()
        g_mtp = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_mtp):
            mtp_step()
        g_mtp.replay()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            g_mtp.replay()
        e1.record()
        torch.cuda.synchronize()
        mtp_us = e0.elapsed_time(e1) * 1e3 / reps
        g_mtp = None
        sqmix.fa_status(ws2)
        mtp = {"us_per_step": mtp_us, "query_tokens": 2,
               "achieved_gbs": N_LAYERS * (n_local * BYTES_PER_KEY + 6 * N_HEAD * HEAD_DIM * 4) / mtp_us / 1e3,
               "note": "10 layers x 172032 keys, n_q = 2 (MTP verification query), CUDA graph, no append"}
    alg_bytes = n_local * BYTES_PER_KEY + 3 * N_HEAD * HEAD_DIM * 4
    hbm, peak_kind = peaks()
    achieved = alg_bytes / (fa_us * 1e-6) / 1e9

    # ---- end to end through the public API with host buffers -------------------
    h_inp = torch.empty(inp.numel(), dtype=torch.uint8).pin_memory()  # same layout as inp
    h_views = in_views(h_inp)
    for t_, shp in zip(h_views[:4], in_shapes):
        t_.copy_(torch.randn(shp))
    h_views[4].copy_(torch.tensor(list(shard.local_step(N_KV, pos_new)), dtype=torch.int64))
    h_out = torch.empty((N_LAYERS, 1, N_HEAD, HEAD_DIM)).pin_memory()
    h2d = h_inp.numel()
    d2h = h_out.numel() * 4

    def e2e_step():
        inp.copy_(h_inp, non_blocking=True)  # q, gate, k_new, v_new and the step scalars
        run()
        h_out.copy_(out, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_us = e2e_ms * 1e3 / args.steps

    used_graph = graph is not None
    graph = None  # release the captured graph before the process group goes away
    merge_kind = None
    if world > 1:
        merge_kind = "nccl all-gather + merge kernel" if peer is None else "peer-memory merge kernel (NVLink P2P)"
        if peer is not None:
            if not peer.ok():
                raise RuntimeError("peer merge: a bounded wait for a peer gave up")
            peer.close()
    if rank != 0:
        return None
    res = {
        "metric": METRIC, "value": us_per_token, "unit": "us/token", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": us_per_token / 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4_0 KV x f16 tensor-core fragments, f32 accum",
        "data": "synthetic N(0,1) K/V/Q/gate (seeded), q4_0-quantised by the append kernel",
        "config": {"workload": "config3: decode 1 token, 10 full-attn layers x 172032 q4_0 keys, "
                               "16 Q / 2 KV heads, d=256, RoPE 64/1e7, sigmoid gate",
                   "n_q": 1, "keys_per_layer": N_KV, "keys_per_gpu": n_local, "parallelism": f"split-KV x{world}",
                   "l2": "inputs larger than L2: 10 x 99 MB of KV cycled per step",
                   "cuda_graph": used_graph, "cross_gpu_merge": merge_kind},
        "tokens_per_s": 1e6 / us_per_token,
        "roofline": {"bound": "hbm",
                     "kernel": "fa_decode_kernel + fa_merge_kernel (split-KV attention, PDL-chained pair)",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": FA_NCU_TRAFFIC if n_local == N_KV else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one decode launch "
                                       "at 172032 keys (profiles/fa_decode_kernel_172k.txt)", "alg_bytes_per_launch": alg_bytes,
                     "launch_us": fa_us},
        "clocks": sampler.summary(),
        "gpu_launches": launches_per_step * args.steps,
        "e2e": {"value": e2e_us, "unit": "us/token", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
    }
    if mtp is not None:
        res["mtp_verify"] = mtp
    return res


PF_PREFIX = 32768  # config 2: pp512 and pp2048 appended onto a 32768-token q4_0 prefix


def bench_prefill(steps: int, warmup: int):
    """Config 2: one full-attention layer's prefill chunk of T tokens (append + attention
    + gate) after a 32768-token q4_0 prefix; tokens/s and tensor-core roofline."""
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    res = {}
    peak, peak_kind = tensor_peak()
    peak_sus, _ = tensor_peak_sustained()
    for T in (512, 2048):
        n_kv = PF_PREFIX + T
        cap = (n_kv + 255) // 256 * 256
        kc, vc = sqmix.new_kv_cache(cap), sqmix.new_kv_cache(cap)
        for a in range(0, PF_PREFIX, 8192):
            sqmix.set_rows_q4_0(torch.randn((8192, 2, 256), generator=g, device=dev),
                                torch.randn((8192, 2, 256), generator=g, device=dev),
                                torch.arange(a, a + 8192, device=dev), kc, vc, cap, rope_n_rot=N_ROT,
                                rope_freq_base=FREQ_BASE)
        q = torch.randn((T, N_HEAD, HEAD_DIM), generator=g, device=dev).to(torch.bfloat16)
        gate = torch.randn((T, N_HEAD, HEAD_DIM), generator=g, device=dev).to(torch.bfloat16)
        k_new = torch.randn((T, 2, 256), generator=g, device=dev)
        v_new = torch.randn((T, 2, 256), generator=g, device=dev)
        rows = torch.arange(PF_PREFIX, n_kv, device=dev)
        d = torch.tensor([n_kv, PF_PREFIX], dtype=torch.int64, device=dev)
        ws = sqmix.new_fa_prefill_workspace(T)
        out = torch.empty((T, N_HEAD, HEAD_DIM), device=dev)

        def step():
            sqmix.set_rows_q4_0(k_new, v_new, rows, kc, vc, cap, rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE)
            sqmix.flash_attn_prefill(q, kc, vc, cap, d[0:1], d[1:2], gate=gate, rope_n_rot=N_ROT,
                                     rope_freq_base=FREQ_BASE, out=out, workspace=ws)

        for _ in range(max(warmup, 3)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, steps)
        e0.record()
        for _ in range(reps):
            step()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        sqmix.fa_status(ws)
        flops = 16384 * sum(PF_PREFIX + t + 1 for t in range(T))
        tflops = flops / us / 1e6
        res[f"pp{T}"] = {"us": us, "tok_s": T / us * 1e6, "tflops": tflops,
                         "frac_of_measured_bf16_peak": tflops / peak if peak else None,
                         "frac_of_measured_bf16_sustained": tflops / peak_sus,
                         "timed_ms": us * reps / 1e3, "flops": flops}
        del kc, vc, ws
    res["config"] = "config2: 1 layer, prefix 32768 q4_0 keys, T new tokens appended (q4_0, RoPE) then " \
                    "causal GQA attention with sigmoid gate; Q bf16; flops = 4*256*16*sum_t(prefix+t+1)"
    res["peak_tflops"] = peak
    res["peak_kind"] = peak_kind
    res["peak_tflops_sustained"] = peak_sus
    res["peak_note"] = ("burst peak for a short timed loop, sustained peak (seconds of dense bf16 under the "
                        "1 kW power cap) once timed_ms reaches about a second")
    return res


GDN_STATE_BYTES = 32 * 128 * 128 * 4  # one GDN layer's recurrent state (2 MiB)


def gdn_inputs(g, dev, T: int, n_layers: int):
    """Config-1 inputs: state N(0, 0.02) [32][128][128] per layer, q/k bf16 N(0,1)
    (L2-normalised inside the kernel), v bf16 N(0,1), beta = sigmoid(N(0,1)),
    g = -exp(A_log) softplus(N(0,1) + dt_bias), A_log ~ U(0, 2.7), dt_bias ~ N(0,1)."""
    import torch

    S = torch.randn((n_layers, 1, 1, 32, 128, 128), generator=g, device=dev) * 0.02
    q = torch.randn((1, T, 16, 128), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((1, T, 16, 128), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((1, T, 32, 128), generator=g, device=dev).to(torch.bfloat16)
    a_log = torch.rand((32,), generator=g, device=dev) * 2.7
    dt_bias = torch.randn((32,), generator=g, device=dev)
    sp = torch.nn.functional.softplus(torch.randn((1, T, 32), generator=g, device=dev) + dt_bias)
    gg = (-torch.exp(a_log) * sp).contiguous()
    beta = torch.sigmoid(torch.randn((1, T, 32), generator=g, device=dev)).contiguous()
    return S, q, k, v, gg, beta


def bench_gdn(steps: int, warmup: int):
    """Config 1: GDN decode (one token per layer; the states of 96 layers, 201 MB, are
    cycled so that each layer's state comes from HBM) and a 512-token chunked prefill."""
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(13)
    res = {}
    hbm, hbm_kind = peaks()
    n_layers = 96
    S, q, k, v, gg, beta = gdn_inputs(g, dev, 1, n_layers)
    out = torch.empty((1, 1, 32, 128), device=dev)

    def decode_all():
        for l in range(n_layers):
            sqmix.gated_delta_net(q, k, v, gg, beta, S[l], l2_eps=1e-6, out=out, state_ready=True)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        decode_all()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        decode_all()
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, steps)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n_layers)
    alg = 2 * GDN_STATE_BYTES + 1 * (2 * 16 * 128 * 2 + 32 * 128 * 2 + 32 * 128 * 4 + 2 * 32 * 4)
    res["decode"] = {"us_per_layer_token": us, "alg_bytes": alg, "achieved_gbs": alg / us / 1e3,
                     "frac_of_hbm": alg / us / 1e3 / hbm, "peak_gbs": hbm, "peak_kind": hbm_kind,
                     "note": "CUDA graph of 96 single-token layer updates (states cycled through HBM)"}
    del graph, S
    # batched decode (config 4's 64 sequences, one token each): 64 x 4.2 MB per layer
    nb, n_lb = 64, 4
    Sb = torch.randn((n_lb, nb, 1, 32, 128, 128), generator=g, device=dev) * 0.02
    qb = torch.randn((nb, 1, 16, 128), generator=g, device=dev).to(torch.bfloat16)
    kb = torch.randn((nb, 1, 16, 128), generator=g, device=dev).to(torch.bfloat16)
    vb = torch.randn((nb, 1, 32, 128), generator=g, device=dev).to(torch.bfloat16)
    gb = -torch.rand((nb, 1, 32), generator=g, device=dev)
    bb = torch.rand((nb, 1, 32), generator=g, device=dev)
    ob = torch.empty((nb, 1, 32, 128), device=dev)

    def decode_batch():
        for l in range(n_lb):
            sqmix.gated_delta_net(qb, kb, vb, gb, bb, Sb[l], l2_eps=1e-6, out=ob, state_ready=True)

    for _ in range(max(warmup, 3)):
        decode_batch()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        decode_batch()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n_lb)
    algb = nb * alg
    res["decode_batch64"] = {"us_per_layer": us, "alg_bytes": algb, "achieved_gbs": algb / us / 1e3,
                             "frac_of_hbm": algb / us / 1e3 / hbm, "peak_gbs": hbm, "peak_kind": hbm_kind,
                             "note": "64 sequences x 1 token per launch (config 4 shape), 4 layer states cycled"}
    del Sb
    T = 512
    S, q, k, v, gg, beta = gdn_inputs(g, dev, T, 1)
    out = torch.empty((1, T, 32, 128), device=dev)
    ws = torch.zeros(sqmix.gdn_prefill_workspace_bytes(1, T, 32), dtype=torch.uint8, device=dev)

    def prefill():
        sqmix.gated_delta_net(q, k, v, gg, beta, S[0], l2_eps=1e-6, out=out, chunked=True, workspace=ws)

    for _ in range(max(warmup, 3)):
        prefill()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        prefill()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    flops = 2.68e9  # chunked form, 8 chunks x 32 heads (C = 64, d = 128)
    res["prefill512"] = {"us": us, "tok_s": T / us * 1e6, "tflops_chunked_form": flops / us / 1e6,
                         "note": "one layer, chunk 64, eager launches"}
    res["front_end"] = bench_gdn_front(g, dev, steps, warmup, hbm, hbm_kind)
    res["config"] = "config1: 32 value heads over 16 q/k heads, d 128, bf16 q/k/v, fused L2 norm"
    return res


def _graph_us(fn, n_calls: int, reps: int, warmup: int) -> float:
    """Device time per call of fn (n_calls launches captured in one CUDA graph)."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / (reps * n_calls)


def bench_gdn_front(g, dev, steps: int, warmup: int, hbm: float, hbm_kind: str) -> dict:
    """The GDN front end around the recurrence (config 1 shapes): short conv + SiLU + q/k
    L2 norm with the conv history (C = 8192 channels, K = 4), and norm_gated of the
    output (32 heads x 128, bf16 gate z); decode (1 token, 30 layers' buffers cycled) and
    a 512-token prefill chunk."""
    import torch

    import sqmix

    C, K, n_layers, reps = 8192, 4, 30, max(3, steps)
    res = {}
    for T in (1, 512):
        x = torch.randn((n_layers, 1, T, C), generator=g, device=dev).to(torch.bfloat16)
        w = torch.randn((n_layers, C, K), generator=g, device=dev) * 0.5
        st = torch.randn((n_layers, 1, 1, C, K - 1), generator=g, device=dev)
        out = torch.empty((1, T, C), device=dev)
        z = torch.randn((n_layers, T, 32, 128), generator=g, device=dev).to(torch.bfloat16)
        o = torch.randn((n_layers, T, 32, 128), generator=g, device=dev)
        wn = torch.randn((128,), generator=g, device=dev)
        y = torch.empty((T, 32, 128), device=dev)

        def conv_all():
            for l in range(n_layers):
                sqmix.gdn_conv(x[l], w[l], st[l], n_qk_channels=4096, l2_eps=1e-6, out=out)

        def norm_all():
            for l in range(n_layers):
                sqmix.head_norm(o[l], 1e-6, weight=wn, z=z[l], out=y)

        us_c = _graph_us(conv_all, n_layers, reps, warmup)
        us_n = _graph_us(norm_all, n_layers, reps, warmup)
        alg_c = T * C * (2 + 4) + C * K * 4 + 2 * C * (K - 1) * 4  # x bf16 in, out f32, taps, history r+w
        alg_n = T * 32 * 128 * (4 + 2 + 4) + 128 * 4  # o f32 in, z bf16 in, y f32 out
        key = "decode" if T == 1 else f"prefill{T}"
        res[key] = {
            "conv_us": us_c, "conv_alg_bytes": alg_c, "conv_frac_of_hbm": alg_c / us_c / 1e3 / hbm,
            "norm_gated_us": us_n, "norm_gated_alg_bytes": alg_n,
            "norm_gated_frac_of_hbm": alg_n / us_n / 1e3 / hbm, "peak_gbs": hbm, "peak_kind": hbm_kind}
    res["note"] = ("CUDA graphs of 30 PDL-chained launches (one per GDN layer, buffers cycled); decode is "
                   "launch/latency bound (a few hundred KB per launch)")
    return res


def bench_stack(steps: int, warmup: int, splits_per_seq: int = 0):
    """Config 4: batched hybrid mixer stack, 40 layers (3 GDN + 1 full attention, x10),
    64 sequences decoding one token each; per-sequence q4_0 KV lengths ~U[1024, 32768]
    (seeded), each sequence with its own GDN states.  Caches hold random q4_0 codes with
    fp16 scales ~U(0.05, 0.3) (filling 6 GB through the quantiser would dominate the
    run); the attention arithmetic does not depend on where the codes came from."""
    import numpy as np
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    rng = np.random.default_rng(17)
    n_seqs, n_fa, n_gdn = 64, 10, 30
    # the batch is ordered longest first, as an engine that knows its sequence lengths
    # would submit it: CTAs are scheduled in grid order, so the long splits start first
    lens = np.sort(rng.integers(1024, 32768 + 1, n_seqs))[::-1]
    caps = [int((n + 1 + 255) // 256 * 256) for n in lens]
    offs = np.concatenate([[0], np.cumsum(caps)])
    rows_total = int(offs[-1])
    unit_rows = 16  # a 4608-byte group holds 16 tokens of both heads
    kc, vc = [], []
    for _ in range(n_fa):
        for lst in (kc, vc):
            buf = torch.randint(0, 256, (rows_total * 288,), dtype=torch.uint8, generator=g, device=dev)
            units = buf.view(-1, 2304)
            sc = (torch.rand((units.shape[0], 128), generator=g, device=dev) * 0.25 + 0.05).half()
            units[:, 2048:] = sc.view(torch.uint8)
            lst.append(buf)
    i64 = lambda xs: torch.tensor([int(x) for x in xs], dtype=torch.int64, device=dev)
    kp = [i64([kc[l].data_ptr() + int(offs[s]) * 288 for s in range(n_seqs)]) for l in range(n_fa)]
    vp = [i64([vc[l].data_ptr() + int(offs[s]) * 288 for s in range(n_seqs)]) for l in range(n_fa)]
    capt = i64(caps)
    n_kv = i64([n + 1 for n in lens])
    q_pos0 = i64(list(lens))
    q = torch.randn((n_fa, n_seqs, N_HEAD, HEAD_DIM), generator=g, device=dev)
    gate = torch.randn((n_fa, n_seqs, N_HEAD, HEAD_DIM), generator=g, device=dev)
    k_new = torch.randn((n_fa, n_seqs, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
    v_new = torch.randn((n_fa, n_seqs, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
    out = torch.empty((n_fa, n_seqs, N_HEAD, HEAD_DIM), device=dev)
    ws = torch.zeros(sqmix.fa_batch_workspace_bytes(n_seqs, splits_per_seq), dtype=torch.uint8, device=dev)
    S = torch.randn((n_gdn, n_seqs, 1, 32, 128, 128), generator=g, device=dev) * 0.02
    gq = torch.randn((n_gdn, n_seqs, 1, 16, 128), generator=g, device=dev).to(torch.bfloat16)
    gk = torch.randn((n_gdn, n_seqs, 1, 16, 128), generator=g, device=dev).to(torch.bfloat16)
    gv = torch.randn((n_gdn, n_seqs, 1, 32, 128), generator=g, device=dev).to(torch.bfloat16)
    gg = -torch.rand((n_gdn, n_seqs, 1, 32), generator=g, device=dev)
    gb = torch.rand((n_gdn, n_seqs, 1, 32), generator=g, device=dev)
    go = torch.empty((n_gdn, n_seqs, 1, 32, 128), device=dev)

    def step():
        fa = gd = 0
        for layer in range(n_fa + n_gdn):
            if layer % 4 == 3:
                sqmix.flash_attn_decode_batch(q[fa], kp[fa], vp[fa], capt, n_kv, q_pos0, gate=gate[fa],
                                              rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE, out=out[fa],
                                              workspace=ws, k_new=k_new[fa], v_new=v_new[fa],
                                              splits_per_seq=splits_per_seq)
                fa += 1
            else:
                # the kernel before writes another layer's state or the KV cache, never S[gd]
                sqmix.gated_delta_net(gq[gd], gk[gd], gv[gd], gg[gd], gb[gd], S[gd], l2_eps=1e-6, out=go[gd],
                                      state_ready=True)
                gd += 1

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, steps)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    graph = None
    sqmix.fa_status(ws)
    hbm, hbm_kind = peaks()
    fa_bytes = n_fa * float(sum(int(n) + 1 for n in lens)) * BYTES_PER_KEY
    gdn_bytes = n_gdn * n_seqs * 2.0 * GDN_STATE_BYTES
    alg = fa_bytes + gdn_bytes
    return {"us_per_step": us, "tok_s": n_seqs / us * 1e6, "alg_bytes_per_step": alg,
            "achieved_gbs": alg / us / 1e3, "frac_of_hbm": alg / us / 1e3 / hbm, "peak_kind": hbm_kind,
            "kv_len_mean": float(np.mean(lens)),
            "config": "config4: 64 sequences x 1 token, 40 layers (30 GDN + 10 full attention), q4_0 KV "
                      "U[1024, 32768] per sequence, batched kernels, CUDA graph"}


def run_profile_case(case: str):
    """Small fixed workloads for ncu captures (one kernel, a few launches, ~0.3 GB)."""
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    if case == "fa":
        kc, vc = sqmix.new_kv_cache(N_KV), sqmix.new_kv_cache(N_KV)
        for a in range(0, N_KV, 16384):
            n = min(16384, N_KV - a)
            sqmix.set_rows_q4_0(torch.randn((n, 2, 256), generator=g, device=dev),
                                torch.randn((n, 2, 256), generator=g, device=dev),
                                torch.arange(a, a + n, device=dev), kc, vc, N_KV)
        q = torch.randn((1, N_HEAD, HEAD_DIM), generator=g, device=dev)
        gate = torch.randn((1, N_HEAD, HEAD_DIM), generator=g, device=dev)
        d = torch.tensor([N_KV, N_KV - 1], dtype=torch.int64, device=dev)
        ws = sqmix.new_fa_workspace(1, 0, dev)
        for _ in range(3):
            sqmix.flash_attn_ext(q, kc, vc, N_KV, d[0:1], d[1:2], gate=gate, rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, workspace=ws)
    elif case == "pf":
        P, T = 8192, 512
        n_kv = P + T
        cap = (n_kv + 255) // 256 * 256
        kc, vc = sqmix.new_kv_cache(cap), sqmix.new_kv_cache(cap)
        sqmix.set_rows_q4_0(torch.randn((n_kv, 2, 256), generator=g, device=dev),
                            torch.randn((n_kv, 2, 256), generator=g, device=dev),
                            torch.arange(n_kv, device=dev), kc, vc, cap, rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE)
        q = torch.randn((T, N_HEAD, HEAD_DIM), generator=g, device=dev).to(torch.bfloat16)
        gate = torch.randn((T, N_HEAD, HEAD_DIM), generator=g, device=dev).to(torch.bfloat16)
        d = torch.tensor([n_kv, P], dtype=torch.int64, device=dev)
        ws = sqmix.new_fa_prefill_workspace(T)
        for _ in range(3):
            sqmix.flash_attn_prefill(q, kc, vc, cap, d[0:1], d[1:2], gate=gate, rope_n_rot=N_ROT,
                                     rope_freq_base=FREQ_BASE, workspace=ws)
    elif case == "gdnp":
        S, q, k, v, gg, beta = gdn_inputs(g, dev, 512, 1)
        for _ in range(3):
            sqmix.gated_delta_net(q, k, v, gg, beta, S[0], l2_eps=1e-6, chunked=True)
    elif case == "gdn":
        S = torch.randn((1, 1, 32, 128, 128), generator=g, device=dev) * 0.02
        q = torch.nn.functional.normalize(torch.randn((1, 1, 16, 128), generator=g, device=dev), dim=-1)
        k = torch.nn.functional.normalize(torch.randn((1, 1, 16, 128), generator=g, device=dev), dim=-1)
        v = torch.randn((1, 1, 32, 128), generator=g, device=dev)
        gg = -torch.rand((1, 1, 32), generator=g, device=dev)
        b = torch.rand((1, 1, 32), generator=g, device=dev)
        for _ in range(3):
            sqmix.gated_delta_net(q, k, v, gg, b, S)
    elif case == "gdnb":  # the 64-sequence batch of config 4 (268 MB of state, > L2)
        n = 64
        S = torch.randn((n, 1, 32, 128, 128), generator=g, device=dev) * 0.02
        q = torch.nn.functional.normalize(torch.randn((n, 1, 16, 128), generator=g, device=dev), dim=-1)
        k = torch.nn.functional.normalize(torch.randn((n, 1, 16, 128), generator=g, device=dev), dim=-1)
        v = torch.randn((n, 1, 32, 128), generator=g, device=dev)
        gg = -torch.rand((n, 1, 32), generator=g, device=dev)
        b = torch.rand((n, 1, 32), generator=g, device=dev)
        for _ in range(3):
            sqmix.gated_delta_net(q, k, v, gg, b, S)
    else:
        raise SystemExit(f"unknown profile case {case}")
    torch.cuda.synchronize()
    print(f"profile case {case} done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sqmix", choices=["sqmix", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-2 prefill measurement")
    ap.add_argument("--nccl-merge", action="store_true", help="N > 1: all-gather + merge instead of the peer merge")
    ap.add_argument("--profile", default=None, help="run a small ncu case (fa | pf | gdn | gdnb | gdnp) and exit")
    args = ap.parse_args()
    if args.profile:
        run_profile_case(args.profile)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()
    res = run_gpu(args, rank, world, local_rank)
    if res is not None and world == 1 and not args.no_prefill:
        res["prefill"] = bench_prefill(args.steps, args.warmup)
        res["gdn"] = bench_gdn(args.steps, args.warmup)
        res["stack"] = bench_stack(args.steps, args.warmup)
    if res is not None:
        if cpu is not None:
            res["cpu_baseline"] = cpu
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

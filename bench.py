#!/usr/bin/env python
"""Benchmark of the sqmix attention-mixer hot path (BASELINE.json metric).

Workload: one decode token through all 10 full-attention layers
of qwen35moe at 172032 keys per layer -- per layer the q4_0 KV append of the new
token (with fused partial RoPE) and split-KV FlashAttention over the q4_0 cache
with the sigmoid output gate.  Inputs are seeded synthetic N(0,1) tensors with the
reference's shapes (no model weights are involved in the mixer).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sqmix|reference]

N > 1 (under torchrun): the 172032 keys of every layer are split across the ranks;
each rank attends over its slice and the ranks exchange their (O, LSE) partials over
NVLink peer memory and merge them before the gate, one kernel per layer (strong
scaling: total work fixed); NCCL only forms the process group and swaps the peer
buffers' IPC handles (an NCCL all-gather of the partials is kept behind --nccl-merge).
Rank 0 then checks layers 0 and 9 of the split result against a single-GPU decode over
the whole cache.  Config 4 (the 64-sequence mixer stack) is sharded by sequence.

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
# (profiles/fa_decode_kernel_172k.txt): 99.18 MB read + 3.89 MB written.
FA_NCU_TRAFFIC = 103_068_672
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
    """SM clocks, power and clock-event (throttle) reasons sampled DURING the timed region.

    A thread polls NVML (read-only queries: nvmlDeviceGetClockInfo, ...MaxClockInfo,
    ...PowerUsage, ...CurrentClocksEventReasons) about every 2 ms for the GPU this rank
    runs on (matched by UUID, so CUDA_VISIBLE_DEVICES remapping does not matter), so even
    a few-millisecond timed window holds samples.  Without NVML it falls back to one
    streaming ``nvidia-smi -lms 100``.  ``mark_start`` / ``mark_end`` bracket the timed
    region on the host clock (after the synchronize on each side); the summary keeps the
    samples taken inside that window.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    POLL_S = 0.002
    # NVML clock-event reason bits reported by name
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples = []  # (host time, sm_mhz, max_mhz, power_w, set of reasons)
        self._stop = threading.Event()
        self._t = None
        self._proc = None
        self.source = None
        self.t0 = self.t1 = None

    def _uuid(self):
        import torch

        try:
            u = str(torch.cuda.get_device_properties(self.dev).uuid)
            return u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            return None

    def _poll_nvml(self, nv, h):
        while not self._stop.is_set():
            try:
                t = time.perf_counter()
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                rs = {n for n, b in self.REASON_BITS.items() if bits & b}
                self.samples.append((t, float(sm), float(mx), pw, rs))
            except Exception:
                pass
            time.sleep(self.POLL_S)

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self._proc.stdout:
            f = [x.strip() for x in line.strip().split(",")]
            if len(f) < 9:
                continue
            try:
                rs = {n for n, v in zip(names, f[5:9]) if v.lower() == "active"}
                self.samples.append((time.perf_counter(), float(f[1]), float(f[2]), float(f[3]), rs))
            except ValueError:
                continue

    def __enter__(self):
        uuid = self._uuid()
        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByUUID(uuid) if uuid else nv.nvmlDeviceGetHandleByIndex(self.dev)
            self._t = threading.Thread(target=self._poll_nvml, args=(nv, h), daemon=True)
            self.source = "nvml"
            self._t.start()
        except Exception:
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={uuid or self.dev}", f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits", "-lms=100"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._t = threading.Thread(target=self._read_smi, daemon=True)
                self.source = "nvidia-smi"
                self._t.start()
            except Exception:
                return self
        t_wait = time.perf_counter()
        while not self.samples and time.perf_counter() - t_wait < 10:
            time.sleep(0.005)
        return self

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *exc):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=10)
            except Exception:
                self._proc.kill()
        if self._t is not None:
            self._t.join(timeout=10)

    def summary(self):
        inside = [s for s in self.samples
                  if self.t0 is not None and self.t1 is not None and self.t0 <= s[0] <= self.t1]
        window = None if self.t0 is None or self.t1 is None else (self.t1 - self.t0) * 1e3
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "window_ms": window, "source": self.source}
        reasons = set()
        for s in inside:
            reasons |= s[4]
        return {"sm_mhz": float(np.median([s[1] for s in inside])), "sm_max_mhz": max(s[2] for s in inside),
                "power_w": float(np.median([s[3] for s in inside])), "reasons": sorted(reasons),
                "samples": len(inside), "window_ms": window, "source": self.source}


def timed_window(fn, steps: int, device_index: int, world: int = 1):
    """Run fn `steps` times between CUDA events (barrier + synchronize on both sides for
    N > 1) with the clock sampler running; returns (device ms, clock summary).  The caller
    takes the maximum over ranks."""
    import torch

    sampler = ClockSampler(device_index)
    with sampler:
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        sampler.mark_start()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        sampler.mark_end()
    return e0.elapsed_time(e1), sampler.summary()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- #
# CPU legs (oracle): cpu_baseline and --impl reference                          #
# --------------------------------------------------------------------------- #

CPU_KIND = "port"
CPU_NOTE = ("C restatement of ggml-cpu's execution of these nodes (oracle/cpu_ggml.c: q8_0 Q x q4_0 K integer "
            "dots, f32 online softmax, per-key V dequant, rows split across threads); ggml itself is not in this "
            "image")


def cpu_setup():
    import oracle

    oracle.build()
    return oracle, oracle.set_threads(os.cpu_count() or 1)


def cpu_kv_rows(n_kv: int, seed: int):
    """q4_0 K and V caches in ggml row layout ([n_kv][288] bytes each) of N(0,1) values."""
    import oracle

    rng = np.random.default_rng(seed)
    kq = np.empty((n_kv, 288), dtype=np.uint8)
    vq = np.empty((n_kv, 288), dtype=np.uint8)
    for a in range(0, n_kv, 32768):
        n = min(32768, n_kv - a)
        kq[a:a + n] = oracle.q4_0_quantize(rng.standard_normal((n, 512), dtype=np.float32))
        vq[a:a + n] = oracle.q4_0_quantize(rng.standard_normal((n, 512), dtype=np.float32))
    return kq, vq


def cpu_decode_layer(oracle, kq, vq, q, gate, k_new, v_new, n_kv):
    """One full-attention decode layer of one token the way ggml-cpu runs it: the append
    (RoPE on K, quantize_row_q4_0 of the new row), RoPE on Q, flash attention over the
    q4_0 cache, sigmoid gate."""
    pos = n_kv - 1
    kq[pos] = oracle.q4_0_quantize(oracle.rope_text(k_new, pos, FREQ_BASE, N_ROT).reshape(1, 512))[0]
    vq[pos] = oracle.q4_0_quantize(v_new.reshape(1, 512))[0]
    qr = oracle.rope_text(q, pos, FREQ_BASE, N_ROT)
    return oracle.cpu_fa_q4_0(qr, kq[:n_kv], vq[:n_kv], gate, q_pos0=pos, scale=1.0 / 16)


def cpu_decode_inputs(seed: int):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((1, N_HEAD, HEAD_DIM), dtype=np.float32),
            rng.standard_normal((1, N_HEAD, HEAD_DIM), dtype=np.float32),
            rng.standard_normal((1, N_HEAD_KV, HEAD_DIM), dtype=np.float32),
            rng.standard_normal((1, N_HEAD_KV, HEAD_DIM), dtype=np.float32))


def cpu_baseline_config3(budget_s: float = 12.0):
    """Config 3 on the host cores: the 10 layers of one decode token (172032 keys each)."""
    oracle, cores = cpu_setup()
    kq, vq = cpu_kv_rows(N_KV, 0)
    q, gate, kn, vn = cpu_decode_inputs(1)
    cpu_decode_layer(oracle, kq, vq, q, gate, kn, vn, N_KV)  # warm
    t0 = time.perf_counter()
    n = 0
    while n < N_LAYERS and (n == 0 or time.perf_counter() - t0 < budget_s):
        cpu_decode_layer(oracle, kq, vq, q, gate, kn, vn, N_KV)
        n += 1
    per_layer = (time.perf_counter() - t0) / n
    return {"value": per_layer * N_LAYERS * 1e6, "unit": "us/token", "cores": cores, "kind": CPU_KIND,
            "sample": f"{n} of the 10 layers (172032 q4_0 keys: append + RoPE + attention + gate), scaled to 10 "
                      f"layers; {CPU_NOTE}"}


def cpu_baseline_config0():
    """Config 0 on the host cores: one decode layer over 4096 q4_0 keys."""
    oracle, cores = cpu_setup()
    n_kv = 4096
    kq, vq = cpu_kv_rows(n_kv, 2)
    q, gate, kn, vn = cpu_decode_inputs(3)
    cpu_decode_layer(oracle, kq, vq, q, gate, kn, vn, n_kv)
    reps, t0 = 0, time.perf_counter()
    while reps < 20 or time.perf_counter() - t0 < 1.0:
        cpu_decode_layer(oracle, kq, vq, q, gate, kn, vn, n_kv)
        reps += 1
    us = (time.perf_counter() - t0) / reps * 1e6
    return {"value": us, "unit": "us/layer-token", "cores": cores, "kind": CPU_KIND,
            "sample": f"{reps} decode layers of 4096 q4_0 keys (append + RoPE + attention + gate); {CPU_NOTE}"}


def cpu_gdn_inputs(rng, T: int):
    import oracle

    S = (rng.standard_normal((32, 128, 128)) * 0.02).astype(np.float32)
    q = oracle.l2norm(rng.standard_normal((T, 16, 128)).astype(np.float32))
    k = oracle.l2norm(rng.standard_normal((T, 16, 128)).astype(np.float32))
    v = rng.standard_normal((T, 32, 128)).astype(np.float32)
    a_log = rng.uniform(0.0, 2.7, 32)
    dt_bias = rng.standard_normal(32)
    g = (-np.exp(a_log) * np.log1p(np.exp(rng.standard_normal((T, 32)) + dt_bias))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((T, 32))))).astype(np.float32)
    return S, q, k, v, g, beta


def cpu_baseline_config1():
    """Config 1 on the host cores: GDN decode (one token) and the 512-token prefill, f32
    token by token (ggml-cpu's gated_delta_net has no chunked form)."""
    oracle, cores = cpu_setup()
    rng = np.random.default_rng(4)
    S, q, k, v, g, beta = cpu_gdn_inputs(rng, 1)
    oracle.cpu_gdn_f32(q, k, v, g, beta, S)
    reps, t0 = 0, time.perf_counter()
    while reps < 50 or time.perf_counter() - t0 < 1.0:
        oracle.cpu_gdn_f32(q, k, v, g, beta, S)
        reps += 1
    dec_us = (time.perf_counter() - t0) / reps * 1e6
    S, q, k, v, g, beta = cpu_gdn_inputs(rng, 512)
    t0 = time.perf_counter()
    oracle.cpu_gdn_f32(q, k, v, g, beta, S)
    pf_us = (time.perf_counter() - t0) * 1e6
    return {"decode": {"value": dec_us, "unit": "us/layer-token"},
            "prefill512": {"value": pf_us, "unit": "us/layer", "tok_s": 512 / pf_us * 1e6},
            "cores": cores, "kind": CPU_KIND,
            "sample": f"{reps} single-token updates of the [32][128][128] f32 state, then one 512-token pass; "
                      "C restatement of the gated delta rule in f32 (oracle/cpu_ggml.c)"}


def cpu_baseline_config2(n_sample: int = 16):
    """Config 2 on the host cores: pp512 / pp2048 after a 32768-token prefix.  A bounded
    sample of query tokens spread over the chunk (each token's cost grows with its
    position) is timed and scaled to the chunk, plus the q4_0 append of the chunk's rows."""
    oracle, cores = cpu_setup()
    res = {}
    for T in (512, 2048):
        n_kv = PF_PREFIX + T
        kq, vq = cpu_kv_rows(n_kv, 5 + T)
        rng = np.random.default_rng(6 + T)
        kn = rng.standard_normal((T, 2, 256), dtype=np.float32)
        vn = rng.standard_normal((T, 2, 256), dtype=np.float32)
        q = rng.standard_normal((T, N_HEAD, HEAD_DIM), dtype=np.float32)
        gate = rng.standard_normal((T, N_HEAD, HEAD_DIM), dtype=np.float32)
        t0 = time.perf_counter()
        kq[PF_PREFIX:] = oracle.q4_0_quantize(oracle.rope_text(kn, PF_PREFIX, FREQ_BASE, N_ROT).reshape(T, 512))
        vq[PF_PREFIX:] = oracle.q4_0_quantize(vn.reshape(T, 512))
        qr = oracle.rope_text(q, PF_PREFIX, FREQ_BASE, N_ROT)
        t_append = time.perf_counter() - t0
        picks = np.linspace(0, T - 1, n_sample).astype(int)
        t0 = time.perf_counter()
        for t in picks:
            oracle.cpu_fa_q4_0(qr[t:t + 1], kq, vq, gate[t:t + 1], q_pos0=PF_PREFIX + t, scale=1.0 / 16)
        t_attn = (time.perf_counter() - t0) / n_sample * T
        us = (t_append + t_attn) * 1e6
        res[f"pp{T}"] = {"value": us, "unit": "us/chunk", "tok_s": T / us * 1e6}
    res.update({"cores": cores, "kind": CPU_KIND,
                "sample": f"{n_sample} query tokens spread over each chunk (16 head rows each, all threads), "
                          f"scaled to the chunk, plus the chunk's append; {CPU_NOTE}"})
    return res


def cpu_baseline_config4(lens):
    """Config 4 on the host cores: one sequence of the batch (the one at the median KV
    length) through all 40 layers (10 attention decode layers + 30 GDN updates), scaled to
    the batch by the sum of KV lengths (attention) and the sequence count (GDN)."""
    oracle, cores = cpu_setup()
    L = int(np.median(lens))
    kq, vq = cpu_kv_rows(L + 1, 7)
    q, gate, kn, vn = cpu_decode_inputs(8)
    rng = np.random.default_rng(9)
    S, gq, gk, gv, gg, gb = cpu_gdn_inputs(rng, 1)
    cpu_decode_layer(oracle, kq, vq, q, gate, kn, vn, L + 1)
    t0 = time.perf_counter()
    for _ in range(10):
        cpu_decode_layer(oracle, kq, vq, q, gate, kn, vn, L + 1)
    t_fa = (time.perf_counter() - t0) / 10
    t0 = time.perf_counter()
    for _ in range(30):
        oracle.cpu_gdn_f32(gq, gk, gv, gg, gb, S)
    t_gdn = (time.perf_counter() - t0) / 30
    n_seqs = len(lens)
    us = (10 * t_fa * float(sum(int(n) + 1 for n in lens)) / (L + 1) + 30 * t_gdn * n_seqs) * 1e6
    return {"value": us, "unit": "us/step", "tok_s": n_seqs / us * 1e6, "cores": cores, "kind": CPU_KIND,
            "sample": f"one sequence (KV length {L}) through 10 attention + 30 GDN decode layers, scaled to the "
                      f"{n_seqs}-sequence batch; {CPU_NOTE}"}


REF_BUDGET_S = 30.0


def run_reference(args, rank: int):
    """--impl reference: config 3 on the host cores with the ggml-cpu restatement; each
    step is one decode token through all 10 layers (append, RoPE, attention, gate), the
    timed steps stopping after REF_BUDGET_S whatever --steps asks."""
    if rank != 0:
        return None
    oracle, cores = cpu_setup()
    kqs, vqs = [], []
    for l in range(N_LAYERS):
        kq, vq = cpu_kv_rows(N_KV, 100 + l)
        kqs.append(kq)
        vqs.append(vq)
    q, gate, kn, vn = cpu_decode_inputs(1)

    def step():
        for l in range(N_LAYERS):
            cpu_decode_layer(oracle, kqs[l], vqs[l], q, gate, kn, vn, N_KV)

    for _ in range(min(args.warmup, 3)):
        step()
    t0 = time.perf_counter()
    n = 0
    while n < args.steps:
        step()
        n += 1
        if time.perf_counter() - t0 > REF_BUDGET_S:
            break
    per_step = (time.perf_counter() - t0) / n
    v = per_step * 1e6
    sample = (f"each step = one decode token through all 10 layers (172032 q4_0 keys each: append + RoPE + "
              f"attention + gate) on {cores} threads; {n} of {args.steps} requested steps timed (stopped after "
              f"{REF_BUDGET_S:g} s); {CPU_NOTE}")
    return {"metric": METRIC, "value": v, "unit": "us/token", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "timed_steps": n, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "q4_0 KV, q8_0 Q, f32",
            "data": "synthetic N(0,1), seeded", "same_config": True,
            "config": {"workload": "config3: decode 1 token, 10 full-attn layers x 172032 q4_0 keys, 16 Q / 2 KV "
                                   "heads, d=256, RoPE 64/1e7, sigmoid gate"},
            "cpu_baseline": {"value": v, "unit": "us/token", "cores": cores, "kind": CPU_KIND, "sample": sample},
            "e2e": {"value": v, "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# --------------------------------------------------------------------------- #
# GPU arm                                                                       #
# --------------------------------------------------------------------------- #

KV_CHUNK = 1024  # keys per seeded chunk of the synthetic caches


def kv_seed(layer: int, chunk: int) -> int:
    return 1_000_003 * (layer + 1) + chunk


def fill_kv_slice(layer: int, start: int, length: int, kc, vc, cap: int, dev):
    """Rows [0, length) of the tiled caches (kc, vc) <- keys [start, start + length) of
    `layer`, N(0,1) quantised to q4_0 by the append kernel with K rotated at its absolute
    position.  Every KV_CHUNK-key chunk of the sequence has its own seed, so the slices
    held by any number of ranks are the keys of one whole-sequence cache."""
    import torch

    import sqmix

    block = 16384
    g = torch.Generator(device=dev)
    for b0 in range(start, start + length, block):
        n = min(block, start + length - b0)
        kk = torch.empty((n, N_HEAD_KV, HEAD_DIM), device=dev)
        vv = torch.empty((n, N_HEAD_KV, HEAD_DIM), device=dev)
        c = b0 // KV_CHUNK * KV_CHUNK
        while c < b0 + n:
            g.manual_seed(kv_seed(layer, c // KV_CHUNK))
            ck = torch.randn((KV_CHUNK, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
            cv = torch.randn((KV_CHUNK, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
            lo, hi = max(c, b0), min(c + KV_CHUNK, b0 + n)
            kk[lo - b0:hi - b0] = ck[lo - c:hi - c]
            vv[lo - b0:hi - b0] = cv[lo - c:hi - c]
            c += KV_CHUNK
        rows = torch.arange(b0 - start, b0 - start + n, device=dev)
        sqmix.set_rows_q4_0(kk, vv, rows, kc, vc, cap, rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE,
                            rope_pos_offset=start)


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

    # ---- resident state: 10 layers of q4_0 K/V for this rank's key slice ------
    kv = sqmix.KvCache(n_layers=N_LAYERS, kv_cap=cap, device=local_rank)
    kc = [kv.k_state(l) for l in range(N_LAYERS)]
    vc = [kv.v_state(l) for l in range(N_LAYERS)]
    for l in range(N_LAYERS):
        fill_kv_slice(l, k0, n_local, kc[l], vc[l], cap, dev)
    # the new token is written at the last position of the last rank's slice
    pos_new = N_KV - 1
    owner = split_kv.owner(N_KV, world, pos_new)
    # The step's inputs share one device buffer (so that the end-to-end measurement
    # moves them with one host-to-device copy): q, gate, k_new, v_new (f32), then the
    # step scalars {n_kv, q_pos0} (i64).  Every rank draws the same inputs.
    in_shapes = [(N_LAYERS, 1, N_HEAD, HEAD_DIM)] * 2 + [(N_LAYERS, 1, N_HEAD_KV, HEAD_DIM)] * 2
    in_off = [0]
    for shp in in_shapes:
        in_off.append(in_off[-1] + 4 * shp[0] * shp[1] * shp[2] * shp[3])

    def in_views(buf):
        ts = [buf[in_off[i]:in_off[i + 1]].view(torch.float32).view(shp) for i, shp in enumerate(in_shapes)]
        return ts + [buf[in_off[-1]:in_off[-1] + 16].view(torch.int64)]

    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    inp = torch.empty(in_off[-1] + 16, dtype=torch.uint8, device=dev)
    q, gate, k_new, v_new, step = in_views(inp)
    for t_, shp in zip((q, gate, k_new, v_new), in_shapes):
        t_.copy_(torch.randn(shp, generator=g, device=dev))
    step.copy_(torch.tensor(list(shard.local_step(N_KV, pos_new)), dtype=torch.int64, device=dev))
    out = torch.empty((N_LAYERS, 1, N_HEAD, HEAD_DIM), device=dev)
    d_nkv, d_qpos = step[0:1], step[1:2]
    n_splits = sqmix.lib().sqmix_device_sm_count(local_rank)
    ws = sqmix.new_fa_workspace(2, n_splits, dev)
    torch.cuda.synchronize()

    if world > 1:
        rows = N_HEAD
        pk_all = torch.empty((world, rows * (HEAD_DIM + 1)), device=dev)
        pk_loc = torch.empty((N_LAYERS, rows * (HEAD_DIM + 1)), device=dev)
        # default: the decode with its split merge fused to the exchange over peer memory
        # (two kernels per layer; slots 0..9 for the 1-token step, 10..19 for the MTP
        # query); --nccl-merge: decode, NCCL all-gather of the partials, merge kernel
        peer = None if args.nccl_merge else split_kv.PeerMerge(n_slots=2 * N_LAYERS, rows=N_HEAD, device=dev)

    own = rank == owner  # the rank whose key slice holds the new token appends it (fused)

    def layer(l):
        if world == 1:
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, gate=gate[l], rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, rope_pos_offset=k0, out=out[l],
                                 workspace=ws, n_splits=n_splits, k_new=k_new[l], v_new=v_new[l],
                                 overlap_prev=True)
        elif peer is not None:
            peer.decode(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, l, gate=gate[l], out=out[l], rope_n_rot=N_ROT,
                        rope_freq_base=FREQ_BASE, rope_pos_offset=k0, workspace=ws, n_splits=n_splits,
                        k_new=k_new[l] if own else None, v_new=v_new[l] if own else None, overlap_prev=True)
        else:
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, gate=None, rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, rope_pos_offset=k0,
                                 out=pk_loc[l, :rows * HEAD_DIM].view(1, N_HEAD, HEAD_DIM),
                                 lse=pk_loc[l, rows * HEAD_DIM:].view(1, N_HEAD), workspace=ws,
                                 n_splits=n_splits, k_new=k_new[l] if own else None,
                                 v_new=v_new[l] if own else None, overlap_prev=True)
            dist.all_gather_into_tensor(pk_all, pk_loc[l])
            sqmix.attn_merge_lse(pk_all[:, :rows * HEAD_DIM].view(world, rows, HEAD_DIM),
                                 pk_all[:, rows * HEAD_DIM:], gate=gate[l, 0], out=out[l, 0])

    def step_fn():
        for l in range(N_LAYERS):
            layer(l)

    stream = torch.cuda.current_stream()
    graph = None
    if not args.no_graph:  # N > 1: the merges (peer kernels or NCCL all-gathers) are captured too
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
    ms, clocks = timed_window(run, args.steps, local_rank, world)
    ms = max_over_ranks(ms, world, dev)
    us_per_token = ms * 1e3 / args.steps
    out_check = out.clone()  # the last timed step's output (parity check below)
    # per layer: decode + split merge (PDL pair; for N > 1 the merge also does the
    # exchange), plus the merge kernel after the all-gather with --nccl-merge
    launches_per_step = N_LAYERS * (2 + (1 if world > 1 and peer is None else 0))

    # ---- dominant kernel alone: flash_attn_ext over each layer in turn ---------
    reps = max(3, args.steps)

    def fa_only():
        for l in range(N_LAYERS):
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d_nkv, d_qpos, gate=gate[l], rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, rope_pos_offset=k0, out=out[l],
                                 workspace=ws, n_splits=n_splits, overlap_prev=True)

    fa_us = _graph_us(fa_only, N_LAYERS, reps, args.warmup)
    sqmix.fa_status(ws)

    # ---- MTP verify (config 3's 2-token query) over the same caches ------------
    mtp = None
    if world == 1 or peer is not None:
        q2 = torch.randn((N_LAYERS, 2, N_HEAD, HEAD_DIM), generator=g, device=dev)
        gate2 = torch.randn((N_LAYERS, 2, N_HEAD, HEAD_DIM), generator=g, device=dev)
        out2 = torch.empty((N_LAYERS, 2, N_HEAD, HEAD_DIM), device=dev)
        step2 = torch.tensor(list(shard.local_step(N_KV, N_KV - 2)), dtype=torch.int64, device=dev)

        def mtp_step():
            for l in range(N_LAYERS):
                if world == 1:
                    sqmix.flash_attn_ext(q2[l], kc[l], vc[l], cap, step2[0:1], step2[1:2], gate=gate2[l],
                                         rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE, out=out2[l], workspace=ws,
                                         n_splits=n_splits, overlap_prev=True)
                else:
                    peer.decode(q2[l], kc[l], vc[l], cap, step2[0:1], step2[1:2], N_LAYERS + l, gate=gate2[l],
                                out=out2[l], rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE, rope_pos_offset=k0,
                                workspace=ws, n_splits=n_splits, overlap_prev=True)

        mtp_us = _graph_us(mtp_step, 1, reps, args.warmup, world)
        mtp_us = max_over_ranks(mtp_us, world, dev)
        sqmix.fa_status(ws)
        mtp_bytes = N_LAYERS * (N_KV * BYTES_PER_KEY + 6 * N_HEAD * HEAD_DIM * 4)
        hbm_, _ = peaks()
        mtp = {"us_per_step": mtp_us, "query_tokens": 2, "achieved_gbs": mtp_bytes / mtp_us / 1e3,
               "frac_of_hbm_per_gpu": mtp_bytes / world / mtp_us / 1e3 / hbm_,
               "note": f"10 layers x 172032 keys split over {world} GPU(s), n_q = 2 (MTP verification query), "
                       "CUDA graph, no append"}
    alg_bytes = n_local * BYTES_PER_KEY + 3 * N_HEAD * HEAD_DIM * 4
    hbm, peak_kind = peaks()
    achieved = alg_bytes / (fa_us * 1e-6) / 1e9

    # ---- end to end through the public API with host buffers -------------------
    h_inp = torch.empty(inp.numel(), dtype=torch.uint8).pin_memory()  # same bytes as inp
    h_inp.copy_(inp)
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
    e2e_ms, _ = timed_window(e2e_step, args.steps, local_rank, world)
    e2e_ms = max_over_ranks(e2e_ms, world, dev)
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
    parity = None
    if world > 1:
        parity = split_kv_parity(rank, dev, q, gate, k_new, v_new, out_check)
        dist.barrier()
    if rank != 0:
        return None
    res = {
        "metric": METRIC, "value": us_per_token, "unit": "us/token", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": us_per_token / 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4_0 KV x f16 tensor-core fragments, f32 accum",
        "data": "synthetic N(0,1) K/V/Q/gate (seeded per 1024-key chunk, identical on every rank), q4_0-quantised "
                "by the append kernel",
        "config": {"workload": "config3: decode 1 token, 10 full-attn layers x 172032 q4_0 keys, "
                               "16 Q / 2 KV heads, d=256, RoPE 64/1e7, sigmoid gate",
                   "n_q": 1, "keys_per_layer": N_KV, "keys_per_gpu": n_local, "parallelism": f"split-KV x{world}",
                   "l2": "inputs larger than L2: 10 x 99 MB of KV cycled per step",
                   "cuda_graph": used_graph, "cross_gpu_merge": merge_kind},
        "tokens_per_s": 1e6 / us_per_token,
        "roofline": {"bound": "hbm",
                     "kernel": "fa_decode_capped_kernel + fa_merge_narrow_kernel (split-KV attention, PDL-chained pair)",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": FA_NCU_TRAFFIC if n_local == N_KV else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one decode launch "
                                       "at 172032 keys (profiles/fa_decode_kernel_172k.txt)",
                     "alg_bytes_per_launch": alg_bytes, "launch_us": fa_us},
        "clocks": clocks,
        "gpu_launches": launches_per_step * args.steps,
        "e2e": {"value": e2e_us, "unit": "us/token", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
    }
    if mtp is not None:
        res["mtp_verify"] = mtp
    if parity is not None:
        res["parity"] = parity
    return res


def split_kv_parity(rank: int, dev, q, gate, k_new, v_new, out_multi):
    """N > 1: rank 0 rebuilds layers 0 and 9 as one whole-sequence cache from the same
    per-chunk seeds, runs the single-GPU decode (fused append, RoPE, gate) over all
    172032 keys and compares it with the split-KV output of the last timed step."""
    import torch

    import sqmix

    if rank != 0:
        return None
    cap = (N_KV + 255) // 256 * 256
    kc, vc = sqmix.new_kv_cache(cap, dev), sqmix.new_kv_cache(cap, dev)
    d = torch.tensor([N_KV, N_KV - 1], dtype=torch.int64, device=dev)
    errs = {}
    for l in (0, N_LAYERS - 1):
        fill_kv_slice(l, 0, N_KV, kc, vc, cap, dev)
        ref = sqmix.flash_attn_ext(q[l], kc, vc, cap, d[0:1], d[1:2], gate=gate[l], rope_n_rot=N_ROT,
                                   rope_freq_base=FREQ_BASE, k_new=k_new[l], v_new=v_new[l])
        got = out_multi[l].double()
        errs[l] = float((got - ref.double()).abs().max() / ref.double().abs().max())
    worst = max(errs.values())
    return {"max_rel_err": worst, "tol": 2e-3, "ok": worst <= 2e-3, "layers": sorted(errs),
            "per_layer": {str(k): v for k, v in errs.items()},
            "reference": "single-GPU sqmix_fa_decode over the whole 172032-key cache built from the same seeds "
                         "(itself checked against the CPU oracle at this size by tests/test_gpu_headline.py)"}


def bench_config0(steps: int, warmup: int):
    """Config 0 on the GPU: one decode layer over 4096 q4_0 keys (append of the step's
    row, RoPE, attention, gate).  One layer's cache is 2.4 MB, so 64 layers' caches
    (151 MB, more than L2) are cycled and the time is per layer-token."""
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    n_kv, n_layers = 4096, 64
    cap = n_kv
    kc = [sqmix.new_kv_cache(cap, dev) for _ in range(n_layers)]
    vc = [sqmix.new_kv_cache(cap, dev) for _ in range(n_layers)]
    for l in range(n_layers):
        fill_kv_slice(100 + l, 0, n_kv, kc[l], vc[l], cap, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(20)
    q = torch.randn((n_layers, 1, N_HEAD, HEAD_DIM), generator=g, device=dev)
    gate = torch.randn((n_layers, 1, N_HEAD, HEAD_DIM), generator=g, device=dev)
    k_new = torch.randn((n_layers, 1, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
    v_new = torch.randn((n_layers, 1, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
    out = torch.empty((n_layers, 1, N_HEAD, HEAD_DIM), device=dev)
    d = torch.tensor([n_kv, n_kv - 1], dtype=torch.int64, device=dev)
    ws = sqmix.new_fa_workspace(1, 0, dev)

    def all_layers():
        for l in range(n_layers):
            sqmix.flash_attn_ext(q[l], kc[l], vc[l], cap, d[0:1], d[1:2], gate=gate[l], rope_n_rot=N_ROT,
                                 rope_freq_base=FREQ_BASE, out=out[l], workspace=ws, k_new=k_new[l],
                                 v_new=v_new[l], overlap_prev=True)

    us = _graph_us(all_layers, n_layers, max(3, steps // 10), warmup)
    sqmix.fa_status(ws)
    hbm, hbm_kind = peaks()
    alg = n_kv * BYTES_PER_KEY + 3 * N_HEAD * HEAD_DIM * 4
    return {"us_per_layer_token": us, "alg_bytes": alg, "achieved_gbs": alg / us / 1e3,
            "frac_of_hbm": alg / us / 1e3 / hbm, "peak_gbs": hbm, "peak_kind": hbm_kind,
            "config": "config0: 1 query token, 16/2 heads, d 256, 4096 q4_0 keys, scale 1/16, fused append, "
                      "sigmoid gate; 64 layers' caches cycled (151 MB > L2), CUDA graph",
            "note": "a 2.4 MB layer is bound by the launch and the fixed per-layer cost, not by HBM"}


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
    res["layer_decode"] = bench_gdn_layer(g, dev, steps, warmup, hbm, hbm_kind)
    res["config"] = "config1: 32 value heads over 16 q/k heads, d 128, bf16 q/k/v, fused L2 norm"
    return res


def _graph_us(fn, n_calls: int, reps: int, warmup: int, world: int = 1) -> float:
    """Device time per call of fn (n_calls launches captured in one CUDA graph).  With
    world > 1 every rank calls it (fn exchanges with the other ranks): the ranks meet at
    a barrier before the first replay."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
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


STACK_SEQS = 64


def stack_lengths():
    """Config 4's per-sequence KV lengths, ~U[1024, 32768] (seeded), longest first as an
    engine that knows its sequence lengths would submit them (CTAs are scheduled in grid
    order, so the long splits start first)."""
    rng = np.random.default_rng(17)
    return np.sort(rng.integers(1024, 32768 + 1, STACK_SEQS))[::-1]


# Mixer projections of one token through the 40 layers (n_embd 2048): (name, ggml type,
# n_in, n_out) per layer kind.  Types as a Q4_K_M model assigns them (attn_v q6_K, the
# other large matrices q4_K; the 32-row ssm_beta / ssm_alpha kept f32).
PROJ_FULL = [("attn_q", 12, 2048, 8192), ("attn_k", 12, 2048, 512), ("attn_v", 14, 2048, 512),
             ("attn_output", 12, 4096, 2048)]
PROJ_GDN = [("attn_qkv", 12, 2048, 8192), ("attn_gate", 12, 2048, 4096), ("ssm_beta", 0, 2048, 32),
            ("ssm_alpha", 0, 2048, 32), ("ssm_out", 12, 4096, 2048)]


def proj_weights(n_in, n_out, wtype, dev, seed):
    """Random rows of a GGUF format with finite f16 scales (raw quant bytes are all valid)."""
    import torch

    import sqmix

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    if wtype == 0:
        return (torch.randn((n_out, n_in), generator=g, device=dev) * 0.02).view(torch.uint8)
    rb = sqmix.mul_mat_row_bytes(wtype, n_in)
    w = torch.randint(0, 256, (n_out, rb), generator=g, dtype=torch.uint8, device=dev)
    if wtype == 12:  # d, dmin = 2^-11
        w.view(-1, 144)[:, 0:4] = torch.tensor([0, 16, 0, 16], dtype=torch.uint8, device=dev)
    elif wtype == 14:
        w.view(-1, 210)[:, 208:210] = torch.tensor([0, 16], dtype=torch.uint8, device=dev)
    return w


def bench_proj(steps: int, warmup: int) -> dict:
    """The mixer projections of one decode token (T = 1) and of an MTP verification
    step (T = 2) through all 40 layers on distinct weights (735 MB > L2), captured in a
    CUDA graph: the projections of one x go as one sqmix_mul_mat_group call (QG / K / V;
    qkv / z / beta / alpha), W_o and ssm_out alone -- 10 x 2 + 30 x 2 = 80 calls, one
    launch each.  The 190 single sqmix_mul_mat calls are timed beside it at T = 1."""
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    hbm, hbm_kind = peaks()
    layers = []  # per layer: groups of (name, wt, n_in, n_out, w) sharing x
    seed = 0
    for layer in range(40):
        groups = {}
        for name, wt, n_in, n_out in (PROJ_FULL if layer % 4 == 3 else PROJ_GDN):
            seed += 1
            groups.setdefault(n_in, []).append((name, wt, n_in, n_out, proj_weights(n_in, n_out, wt, dev, seed)))
        layers.append(list(groups.values()))
    calls = [c for groups in layers for grp in groups for c in grp]
    n_launch = sum(len(groups) for groups in layers)  # one launch per call at T <= 4
    wbytes = sum(c[4].numel() for c in calls)
    res = {"calls_per_token": sum(len(groups) for groups in layers), "launches_per_token": n_launch,
           "weight_bytes": wbytes, "peak_gbs": hbm, "peak_kind": hbm_kind}
    for T in (1, 2):
        xs = {n: torch.randn((T, n), device=dev) for n in (2048, 4096)}
        ys = {}
        for name, _, _, n_out, _ in calls:
            ys.setdefault(name, torch.empty((T, n_out), device=dev))

        def step():
            for groups in layers:
                for grp in groups:
                    if len(grp) == 1:
                        name, wt, n_in, _, w = grp[0]
                        sqmix.mul_mat(w, wt, n_in, xs[n_in], out=ys[name])
                    else:
                        sqmix.mul_mat_group([(w, wt) for _, wt, _, _, w in grp], grp[0][2], xs[grp[0][2]],
                                            outs=[ys[name] for name, *_ in grp])

        us = _graph_us(step, 1, max(3, min(steps, 200)), warmup)
        res[f"T{T}"] = {"us_per_step": us, "achieved_gbs": wbytes / us / 1e3, "frac_of_hbm": wbytes / us / 1e3 / hbm}
        if T == 1:
            def step_single():
                for name, wt, n_in, _, w in calls:
                    sqmix.mul_mat(w, wt, n_in, xs[n_in], out=ys[name])

            us = _graph_us(step_single, 1, max(3, min(steps, 200)), warmup)
            res["T1_single_calls"] = {"calls": len(calls), "us_per_step": us, "frac_of_hbm": wbytes / us / 1e3 / hbm}
    # a 512-token prefill batch through the same 80 calls: the tensor-core GEMM form
    T = 512
    xs = {n: torch.randn((T, n), device=dev) for n in (2048, 4096)}
    ys = {}
    for name, _, _, n_out, _ in calls:
        ys.setdefault(name, torch.empty((T, n_out), device=dev))

    def step_prefill():
        for groups in layers:
            for grp in groups:
                sqmix.mul_mat_group([(w, wt) for _, wt, _, _, w in grp], grp[0][2], xs[grp[0][2]],
                                    outs=[ys[name] for name, *_ in grp])

    us = _graph_us(step_prefill, 1, max(3, min(steps, 10)), warmup)
    flop = 2.0 * T * sum(n_in * n_out for _, _, n_in, n_out, _ in calls)
    res["prefill_T512"] = {"us_per_step": us, "tflops": flop / us / 1e6,
                           "frac_of_measured_bf16_peak": flop / us / 1e6 / tensor_peak()[0],
                           "note": "f32 x: tf32 tensor-core operands (half the bf16 rate)"}
    # the largest single projection, alone (QG / qkv: 2048 -> 8192 q4_K)
    x1 = torch.randn((1, 2048), device=dev)
    y1 = torch.empty((1, 8192), device=dev)
    ws = [proj_weights(2048, 8192, 12, dev, 1000 + i) for i in range(16)]

    def one():
        for wi in ws:
            sqmix.mul_mat(wi, 12, 2048, x1, out=y1)

    us1 = _graph_us(one, len(ws), max(3, min(steps, 200)), warmup)
    b1 = ws[0].numel()
    res["qkv_2048x8192_q4k"] = {"us": us1, "bytes": b1, "achieved_gbs": b1 / us1 / 1e3, "frac_of_hbm": b1 / us1 / 1e3 / hbm}
    res["note"] = ("weights: random GGUF blocks with finite scales; the roofline is the weight stream (x and y are "
                   "a few KB); a launch has a fixed cost of a few us (the wait on the kernel before, staging x), "
                   "paid once per group of projections of the same x")
    return res


def cpu_baseline_proj() -> dict:
    """The projections on the host cores with ggml-cpu's algorithm (x quantised to q8_K,
    integer dots), on a bounded sample: one attn_qkv (2048 -> 8192 q4_K) at T = 1, scaled
    by weight bytes to the 40 layers."""
    oracle, cores = cpu_setup()
    rng = np.random.default_rng(9)
    rb = oracle.row_bytes(12, 2048)
    w = rng.integers(0, 256, (8192, rb), dtype=np.uint8)
    w.reshape(-1, 144)[:, 0:4] = np.array([0, 16, 0, 16], dtype=np.uint8)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    oracle.cpu_mul_mat(w, 12, 2048, x)
    reps, t0 = 0, time.perf_counter()
    while reps < 5 or time.perf_counter() - t0 < 1.0:
        oracle.cpu_mul_mat(w, 12, 2048, x)
        reps += 1
    us = (time.perf_counter() - t0) / reps * 1e6
    total_bytes = 0
    for layer in range(40):
        for _, wt, n_in, n_out in (PROJ_FULL if layer % 4 == 3 else PROJ_GDN):
            total_bytes += oracle.row_bytes(wt, n_in) * n_out
    scale = total_bytes / w.nbytes
    # a prefill batch: the same dot products per token, 8 tokens per sample
    x8 = rng.standard_normal((8, 2048)).astype(np.float32)
    reps8, t0 = 0, time.perf_counter()
    while reps8 < 3 or time.perf_counter() - t0 < 1.0:
        oracle.cpu_mul_mat(w, 12, 2048, x8)
        reps8 += 1
    us8 = (time.perf_counter() - t0) / reps8 * 1e6
    return {"value": us * scale, "unit": "us/token", "qkv_us": us, "cores": cores, "kind": CPU_KIND,
            "prefill_T512": {"value": us8 * 64 * scale, "unit": "us per 512 tokens",
                             "sample": f"{reps8} runs of the same projection at T = 8, scaled by 64 and by weight bytes"},
            "sample": f"{reps} runs of one 2048 -> 8192 q4_K projection (T = 1), scaled by weight bytes to the 190 "
                      "projections of a token; C restatement of ggml-cpu's q4_K x q8_K integer dot products "
                      "(oracle/cpu_ggml.c)"}


def bench_gdn_layer(g, dev, steps: int, warmup: int, hbm: float, hbm_kind: str) -> dict:
    """A whole GDN mixer decode step at batch 1 (config 1 shapes): the one-launch layer
    (sqmix_gdn_layer_decode: conv + SiLU + L2 norm + gate epilogue + recurrence +
    norm_gated) against the three launches it replaces (conv, recurrence with the gate
    epilogue, norm_gated); 30 layers' buffers cycled (states 63 MB, conv planes 2.9 MB)."""
    import torch

    import sqmix

    C, K, n_layers, reps = 8192, 4, 30, max(3, steps)
    x = torch.randn((n_layers, 1, 1, C), generator=g, device=dev).to(torch.bfloat16)
    w = torch.randn((n_layers, C, K), generator=g, device=dev) * 0.5
    cst = torch.randn((n_layers, 1, 1, C, K - 1), generator=g, device=dev)
    S = torch.randn((n_layers, 1, 1, 32, 128, 128), generator=g, device=dev) * 0.02
    alpha = torch.randn((n_layers, 1, 1, 32), generator=g, device=dev)
    braw = torch.randn((n_layers, 1, 1, 32), generator=g, device=dev)
    dt = torch.randn((n_layers, 32), generator=g, device=dev)
    ssm_a = -torch.exp(torch.rand((n_layers, 32), generator=g, device=dev) * 2.7)
    z = torch.randn((n_layers, 1, 1, 32, 128), generator=g, device=dev).to(torch.bfloat16)
    wn = torch.rand((n_layers, 128), generator=g, device=dev) + 0.5
    y = torch.empty((1, 1, 32, 128), device=dev)
    conv = torch.empty((1, 1, C), device=dev)
    o = torch.empty((1, 1, 32, 128), device=dev)

    def fused():
        for l in range(n_layers):
            sqmix.gdn_layer_decode(x[l], w[l], cst[l], alpha[l], braw[l], ssm_a[l], S[l], dt_bias=dt[l], l2_eps=1e-6,
                                   z=z[l], norm_weight=wn[l], out=y, state_ready=True)

    def three():
        for l in range(n_layers):
            sqmix.gdn_conv(x[l], w[l], cst[l], n_qk_channels=4096, l2_eps=1e-6, out=conv)
            sqmix.gated_delta_net(conv[:, :, :2048].view(1, 1, 16, 128), conv[:, :, 2048:4096].view(1, 1, 16, 128),
                                  conv[:, :, 4096:].view(1, 1, 32, 128), alpha[l], braw[l], S[l], out=o,
                                  dt_bias=dt[l], ssm_a=ssm_a[l])
            sqmix.head_norm(o[0], 1e-6, weight=wn[l], z=z[l, 0], out=y[0])

    us_f = _graph_us(fused, n_layers, reps, warmup)
    us_3 = _graph_us(three, n_layers, reps, warmup)
    alg = 2 * GDN_STATE_BYTES + 2 * C * (K - 1) * 4 + C * K * 4 + C * 2 + 32 * 128 * (2 + 4) + 128 * 4
    return {"us_per_layer_token": us_f, "three_launch_us": us_3, "alg_bytes": alg,
            "achieved_gbs": alg / us_f / 1e3, "frac_of_hbm": alg / us_f / 1e3 / hbm, "peak_gbs": hbm,
            "peak_kind": hbm_kind,
            "note": "batch 1, 1 token: conv + SiLU + q/k L2 norm + beta/decay epilogue + recurrence + norm_gated; "
                    "CUDA graph of 30 layers (buffers cycled); three_launch_us = sqmix_gdn_conv + sqmix_gdn_decode + "
                    "sqmix_head_norm for the same work"}


def bench_stack(steps: int, warmup: int, rank: int = 0, world: int = 1, local_rank: int = 0,
                splits_per_seq: int = 0):
    """Config 4: batched hybrid mixer stack, 40 layers (3 GDN + 1 full attention, x10),
    64 sequences decoding one token each, each sequence with its own q4_0 KV caches
    (N(0,1) K/V quantised by the append kernel, K rotated) and its own GDN states.  With
    N ranks the sequences are sharded by sequence, round-robin over the length-sorted
    batch (rank r takes sequences r, r + N, ...): no collective on the data path; the
    aggregate is 64 tokens over the slowest rank's step time."""
    import torch

    import sqmix

    dev = torch.device("cuda", local_rank)
    lens_all = stack_lengths()
    mine = list(range(rank, STACK_SEQS, world))
    lens = lens_all[mine]
    n_seqs, n_fa, n_gdn = len(mine), 10, 30
    caps = [int((n + 1 + 255) // 256 * 256) for n in lens]
    offs = np.concatenate([[0], np.cumsum(caps)])
    rows_total = int(offs[-1])
    kc = [torch.empty(rows_total * 288, dtype=torch.uint8, device=dev) for _ in range(n_fa)]
    vc = [torch.empty(rows_total * 288, dtype=torch.uint8, device=dev) for _ in range(n_fa)]
    g = torch.Generator(device=dev)
    for l in range(n_fa):
        for i, s_glob in enumerate(mine):
            a, b = int(offs[i]) * 288, int(offs[i] + caps[i]) * 288
            kc[l][a:b].zero_()
            vc[l][a:b].zero_()
            g.manual_seed(7_000_003 * (l + 1) + s_glob)
            n = int(lens[i])
            kk = torch.randn((n, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
            vv = torch.randn((n, N_HEAD_KV, HEAD_DIM), generator=g, device=dev)
            sqmix.set_rows_q4_0(kk, vv, torch.arange(n, device=dev), kc[l][a:b], vc[l][a:b], caps[i],
                                rope_n_rot=N_ROT, rope_freq_base=FREQ_BASE)
            del kk, vv
    i64 = lambda xs: torch.tensor([int(x) for x in xs], dtype=torch.int64, device=dev)
    kp = [i64([kc[l].data_ptr() + int(offs[s]) * 288 for s in range(n_seqs)]) for l in range(n_fa)]
    vp = [i64([vc[l].data_ptr() + int(offs[s]) * 288 for s in range(n_seqs)]) for l in range(n_fa)]
    capt = i64(caps)
    n_kv = i64([n + 1 for n in lens])
    q_pos0 = i64(list(lens))
    g.manual_seed(17 + rank)
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
    reps = max(3, steps)
    ms, clocks = timed_window(graph.replay, reps, local_rank, world)
    us_local = ms * 1e3 / reps
    us = max_over_ranks(us_local, world, dev)
    graph = None
    sqmix.fa_status(ws)
    hbm, hbm_kind = peaks()
    fa_bytes = n_fa * float(sum(int(n) + 1 for n in lens)) * BYTES_PER_KEY
    gdn_bytes = n_gdn * n_seqs * 2.0 * GDN_STATE_BYTES
    alg = fa_bytes + gdn_bytes
    all_bytes = n_fa * float(sum(int(n) + 1 for n in lens_all)) * BYTES_PER_KEY + \
        n_gdn * STACK_SEQS * 2.0 * GDN_STATE_BYTES
    return {"us_per_step": us, "tok_s": STACK_SEQS / us * 1e6, "n_gpus": world, "seqs_per_gpu": n_seqs,
            "alg_bytes_per_step": all_bytes, "aggregate_gbs": all_bytes / us / 1e3,
            "rank0_alg_bytes": alg, "rank0_us": us_local, "rank0_frac_of_hbm": alg / us_local / 1e3 / hbm,
            "peak_kind": hbm_kind, "kv_len_mean": float(np.mean(lens_all)), "clocks": clocks,
            "scaling": "strong", "parallelism": f"sequences sharded x{world} (round-robin), no collective",
            "config": "config4: 64 sequences x 1 token, 40 layers (30 GDN + 10 full attention), q4_0 KV of N(0,1) "
                      "(append kernel) with lengths U[1024, 32768] per sequence, batched kernels, CUDA graph; "
                      "tok_s = 64 / the slowest rank's step time"}


def run_profile_case(case: str):
    """Small fixed workloads for ncu captures (one kernel, a few launches, ~0.3 GB)."""
    import torch

    import sqmix

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    if case in ("fa", "fa2"):  # decode at 172K keys; fa2: the n_q = 2 MTP verification
        nq = 2 if case == "fa2" else 1
        kc, vc = sqmix.new_kv_cache(N_KV), sqmix.new_kv_cache(N_KV)
        for a in range(0, N_KV, 16384):
            n = min(16384, N_KV - a)
            sqmix.set_rows_q4_0(torch.randn((n, 2, 256), generator=g, device=dev),
                                torch.randn((n, 2, 256), generator=g, device=dev),
                                torch.arange(a, a + n, device=dev), kc, vc, N_KV)
        q = torch.randn((nq, N_HEAD, HEAD_DIM), generator=g, device=dev)
        gate = torch.randn((nq, N_HEAD, HEAD_DIM), generator=g, device=dev)
        d = torch.tensor([N_KV, N_KV - nq], dtype=torch.int64, device=dev)
        ws = sqmix.new_fa_workspace(nq, 0, dev)
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
    elif case == "gdnl":  # the one-launch GDN decode layer, batch 1 (4.6 MB per launch)
        C = 8192
        x = torch.randn((1, 1, C), generator=g, device=dev).to(torch.bfloat16)
        w = torch.randn((C, 4), generator=g, device=dev) * 0.5
        cst = torch.randn((1, 1, C, 3), generator=g, device=dev)
        S = torch.randn((1, 1, 32, 128, 128), generator=g, device=dev) * 0.02
        alpha = torch.randn((1, 1, 32), generator=g, device=dev)
        braw = torch.randn((1, 1, 32), generator=g, device=dev)
        ssm_a = -torch.exp(torch.rand((32,), generator=g, device=dev) * 2.7)
        z = torch.randn((1, 1, 32, 128), generator=g, device=dev).to(torch.bfloat16)
        wn = torch.rand((128,), generator=g, device=dev) + 0.5
        for _ in range(3):
            sqmix.gdn_layer_decode(x, w, cst, alpha, braw, ssm_a, S, l2_eps=1e-6, z=z, norm_weight=wn)
    elif case == "mm":  # a GDN layer's input projections as one group, T = 1 (14.7 MB per launch)
        x = torch.randn((1, 2048), generator=g, device=dev)
        groups = [[(proj_weights(n_in, n_out, wt, dev, 10 * i + j), wt)
                   for j, (_, wt, n_in, n_out) in enumerate(PROJ_GDN[:4])] for i in range(3)]
        for grp in groups:
            sqmix.mul_mat_group(grp, 2048, x)
    elif case == "mmp":  # the same group at a 512-token prefill batch (the tensor-core GEMM form)
        x = torch.randn((512, 2048), generator=g, device=dev)
        groups = [[(proj_weights(n_in, n_out, wt, dev, 10 * i + j), wt)
                   for j, (_, wt, n_in, n_out) in enumerate(PROJ_GDN[:4])] for i in range(3)]
        for grp in groups:
            sqmix.mul_mat_group(grp, 2048, x)
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
    ap.add_argument("--headline-only", action="store_true",
                    help="config 3 only (skip configs 0, 1, 2 and 4)")
    ap.add_argument("--nccl-merge", action="store_true", help="N > 1: all-gather + merge instead of the peer merge")
    ap.add_argument("--profile", default=None, help="run a small ncu case (fa | fa2 | pf | gdn | gdnb | gdnp | gdnl | mm | mmp) and exit")
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
    cpu_on = rank == 0 and world == 1 and not args.no_cpu_baseline
    cpu = cpu_baseline_config3() if cpu_on else None
    res = run_gpu(args, rank, world, local_rank)
    if not args.headline_only:
        if world == 1:
            res["config0"] = bench_config0(args.steps, args.warmup)
            res["prefill"] = bench_prefill(args.steps, args.warmup)
            res["gdn"] = bench_gdn(args.steps, args.warmup)
            res["proj"] = bench_proj(args.steps, args.warmup)
        stack = bench_stack(args.steps, args.warmup, rank, world, local_rank)  # every rank (sharded)
        if res is not None:
            res["stack"] = stack
        if cpu_on:
            res["config0"]["cpu_baseline"] = cpu_baseline_config0()
            res["gdn"]["cpu_baseline"] = cpu_baseline_config1()
            res["proj"]["cpu_baseline"] = cpu_baseline_proj()
            res["prefill"]["cpu_baseline"] = cpu_baseline_config2()
            res["stack"]["cpu_baseline"] = cpu_baseline_config4(stack_lengths())
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

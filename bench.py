#!/usr/bin/env python
"""Benchmark of the backend-cuda hot path: Llama-3-8B-shaped INT4 decode.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload: llama-dense, 32 layers, hidden 4096, 32/8
heads x 128, FFN 14336, vocab 128256, RoPE theta 5e5, weights N(0, 0.02)
quantized to symmetric INT4 group 128 (generated on the device), f32
activations and KV cache, a 1024-token random prompt (prefill, untimed), then
greedy decode. One timed step = one decode token per sequence through
Engine::step (slc_llama_step): every command of the decode program goes
through slc_dispatch; with command capture the step replays as one CUDA
graph, and at batch 1 on one GPU its 32 layers run as one persistent kernel
(decode_layers_kernel). With N > 1 (torchrun) the model is tensor-parallel
over N GPUs (all-reduce after o/down, all-gather of the logits); the total
work is fixed, so scaling is "strong".

Reported: `value` = decode tok/s from the device time of the steps (CUDA
events on the device stream, max over ranks); `e2e` = the same through the
public API with host buffers (ids/positions uploaded, logits downloaded every
step, host wall clock, max over ranks); `roofline` = the dominant kernel:
the persistent decode-layer kernel, timed on the device every timed step
by its own global-timer stamps at start (first CTA) and end (last CTA to
exit) (where it does not run: the quantized
decode GEMVs measured live on the model's own weights); `cpu_baseline` = the
CPU oracle (the restated reference kernels) on this host's cores. The
weights streamed per step (~4 GB) exceed the 126 MB L2, so no flush is
needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
METRIC = "decode tok/s (Llama-3-8B-shaped llama-dense, INT4 g128)"
METRIC_70B = "decode tok/s (Llama-2-70B-shaped llama-dense, INT8 g128)"
TRAFFIC_PROFILE = os.path.join(ROOT, "profiles", "gemv_imma_int4_28672x4096_m1.md")
FUSED_PROFILE = os.path.join(ROOT, "profiles", "decode_layers_8b_int4_4layers.md")


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences (default: 1 for 8b, 16 for 70b, as BASELINE configs[3], [4])")
    ap.add_argument("--prompt", type=int, default=None,
                    help="prompt tokens, prefilled before the timed decode (default: 1024 for "
                         "8b, 2048 for 70b)")
    ap.add_argument("--layers", type=int, default=32, help="(testing only) fewer layers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="8b: Llama-3-8B shape INT4 g128 (default workload); 70b: Llama-2-70B "
                         "shape INT8 g128 (BASELINE configs[4])")
    ap.add_argument("--synthetic-kv", action="store_true",
                    help="fill the KV cache with N(0,1) values instead of running the prefill "
                         "(decode cost does not depend on the cached values)")
    ap.add_argument("--sweep", action="store_true",
                    help="per-operator and GEMV sweeps of BASELINE configs[1] and [2]")
    ap.add_argument("--gemv", type=str, default=None, metavar="N,K,M",
                    help="profiling aid: only run one quantized MatMulNT shape (INT4 g128, "
                         "random codes) --steps times and print its time")
    args = ap.parse_args(argv)
    if args.batch is None:
        args.batch = 16 if args.model == "70b" else 1
    if args.prompt is None:
        args.prompt = 2048 if args.model == "70b" else 1024
    return args


# ---------------------------------------------------------------- helpers --

def hbm_peak():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def bf16_peak():
    """Measured dense bf16 burst peak (TFLOP/s) for the prefill GEMM fraction."""
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def profile_traffic_ratio(path=TRAFFIC_PROFILE):
    """DRAM bytes / algorithmic bytes of a kernel, from its committed ncu
    summary (the traffic_ratio line)."""
    try:
        for line in open(path):
            if line.strip().startswith("traffic_ratio:"):
                return float(line.split(":", 1)[1].strip().split()[0])
    except Exception:
        pass
    return None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of this rank's GPU during
    the timed region, from two sources read together: NVML polled from a
    thread every 10 ms (a timed region of tens of milliseconds still gets
    several samples) and `nvidia-smi -lms 200`. Reads only: no clock or other
    setting of the GPU is changed."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    PERIOD_S = 0.010

    def __init__(self, index: int):
        # NVML and nvidia-smi number the GPUs physically; map this process's
        # CUDA ordinal through CUDA_VISIBLE_DEVICES when it lists indices.
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.index = int(vis[index]) if index < len(vis) and vis[index].isdigit() else index
        self.proc = self.path = self.thread = None
        self.rows = []  # (sm_mhz, max_mhz, {reason: bool})

    def _nvml_sample(self, nv, h):
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        try:
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception:
            return False
        self.rows.append((sm, mx, {n: bool(r & b) for n, b in zip(self.NAMES, bits)}))
        return True

    def _nvml_loop(self, nv, h, stop):
        while not stop.is_set():
            self._nvml_sample(nv, h)
            stop.wait(self.PERIOD_S)

    def start(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self._nv, self._h = nv, h
            self._stop = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h, self._stop),
                                           daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def _smi_rows(self):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) >= 9 and p[1].replace(".", "").isdigit() and p[2].replace(".", "").isdigit():
                self.rows.append((float(p[1]), float(p[2]),
                                  {n: v.lower() == "active" for n, v in zip(self.NAMES, p[5:9])}))
        os.unlink(self.path)

    def stop(self):
        n_nvml = 0
        if self.thread:
            # One sample as the region ends, taken here: the thread's own
            # samples can be few when the region lasts only tens of ms.
            self._nvml_sample(self._nv, self._h)
            self._stop.set()
            self.thread.join(timeout=5)
            n_nvml = len(self.rows)
        if self.proc:
            self._smi_rows()
        rows = self.rows
        if not rows:
            return None
        mx = max(r[1] for r in rows)
        reasons = sorted({n for r in rows for n, v in r[2].items() if v})
        loaded = [r[0] for r in rows if r[0] > 0.5 * mx] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows),
                "source": f"{n_nvml} NVML samples every 10 ms, "
                          f"{len(rows) - n_nvml} nvidia-smi samples every 200 ms"}


class Dist:
    """One process per GPU; gloo for host plumbing (ids broadcast, timing max)."""

    def __init__(self, gpus: int):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.pg = dist
        if self.world != gpus and gpus != 1:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def broadcast_bytes(self, data: bytes | None, n: int) -> bytes:
        if not self.pg:
            return data
        import torch
        t = torch.zeros(n, dtype=torch.uint8)
        if self.rank == 0:
            t[:] = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        self.pg.broadcast(t, 0)
        return bytes(t.numpy().tobytes())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def emit(line: dict):
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- CPU (oracle) arm --

def oracle_decode_sample(batch: int, prompt: int, threads: int):
    """Per-token time of the CPU reference path for the 8B decode step, from a
    bounded sample: one decoder layer's kernels (7 matmul_nt against f32
    weights, the reference's dequantize-then-matmul path; causal_attention over
    the prompt; 2 rms_norm, rope, add) timed once and multiplied by 32 layers,
    plus matmul_nt against an 8192-row slice of lm_head scaled to 128256 rows.
    Returns (seconds per token, description)."""
    from oracle import pyoracle as orc
    orc.set_threads(threads)
    H, Hq, Hkv, D, I, V = 4096, 32, 8, 128, 14336, 128256
    rng = np.random.default_rng(0)
    x = rng.standard_normal((batch, H), dtype=np.float32)
    shapes = [(Hq * D, H), (Hkv * D, H), (Hkv * D, H), (H, Hq * D), (I, H), (I, H), (H, I)]
    ws = [(rng.standard_normal(n * k, dtype=np.float32) * 0.02) for n, k in shapes]
    max_seq = prompt + 1
    cache = rng.standard_normal(batch * 1 * 2 * max_seq * Hkv * D, dtype=np.float32)
    q = rng.standard_normal(batch * Hq * D, dtype=np.float32)
    kv = rng.standard_normal(batch * Hkv * D, dtype=np.float32)
    head = rng.standard_normal(8192 * H, dtype=np.float32) * 0.02
    g = np.ones(H, np.float32)
    t0 = time.perf_counter()
    for (n, k), w in zip(shapes, ws):
        xi = x if k == H else rng.standard_normal((batch, k), dtype=np.float32)
        orc.matmul_nt(xi, w, 1, batch, k, n)
    orc.causal_attention(q, kv, kv, cache, batch, 1, 0, Hq, Hkv, 1, prompt, D, max_seq,
                         1.0 / np.sqrt(D))
    for _ in range(2):
        orc.rms_norm(x, g, batch, H, 1e-5)
    orc.rope(q, np.full(batch, prompt, np.uint32), batch, Hq, 1, D, 500000.0)
    orc.add(x, x, batch * H)
    layer = time.perf_counter() - t0
    t1 = time.perf_counter()
    orc.matmul_nt(x, head, 1, batch, H, 8192)
    head_t = (time.perf_counter() - t1) * (V / 8192)
    per_token = 32 * layer + head_t
    desc = (f"one 8B decoder layer (7 matmul_nt, causal_attention over {prompt} keys, norms, "
            f"rope, add) x 32 + lm_head slice 8192/128256 rows scaled; batch {batch}; "
            f"restated reference kernels, {threads} OpenMP threads")
    return per_token, desc


def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return 0
    threads = os.cpu_count() or 1
    samples = []
    for _ in range(max(args.warmup, 0)):
        oracle_decode_sample(args.batch, args.prompt, threads)
    for _ in range(args.steps):
        t, desc = oracle_decode_sample(args.batch, args.prompt, threads)
        samples.append(t)
    per_token = statistics.mean(samples)
    value = args.batch / per_token
    emit({"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_token * 1e3,
          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
          "data": "synthetic", "impl": "reference",
          "config": {"workload": "llama3-8b-int4-decode", "batch": args.batch,
                     "prompt": args.prompt, "parallelism": "cpu"},
          "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                           "sample": desc},
          "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                  "d2h_bytes_per_step": 0}})
    return 0


# ------------------------------------------------------------ GPU arm ------

def fused_layer_bytes(cfg, past):
    """Algorithmic HBM bytes of one layer of the persistent decode kernel at
    one token, on one rank: the seven quantized matrices (codes + one f32
    scale per group; q/k/v/gate/up rows and o/down columns split over the
    tensor-parallel ranks), the rank's cached keys and values at positions
    [0, past) read once and the new position's written, and the two norm
    weights."""
    D, w_ = cfg.head_dim, max(1, cfg.tp_world)
    hq, hkv, inter = cfg.heads // w_, cfg.kv_heads // w_, cfg.inter // w_
    mats = [(hq * D, cfg.hidden), (hkv * D, cfg.hidden), (hkv * D, cfg.hidden),
            (cfg.hidden, hq * D), (inter, cfg.hidden), (inter, cfg.hidden), (cfg.hidden, inter)]
    int4 = int(cfg.quant) == 0
    w = sum((n * k // 2 if int4 else n * k) + 4 * n * (k // cfg.group_size) for n, k in mats)
    kv = 2 * past * hkv * D * 4 + 2 * hkv * D * 4
    return w + kv + 2 * cfg.hidden * 4


def streamed_weight_bytes(cfg):
    """Quantized weight bytes one decode step streams, per GPU (the layers'
    matrices and the vocabulary projection, split over the TP ranks)."""
    w_ = max(1, cfg.tp_world)
    per_layer = (fused_layer_bytes(cfg, 0) - 2 * (cfg.kv_heads // w_) * cfg.head_dim * 4
                 - 2 * cfg.hidden * 4)
    return cfg.layers * per_layer + model_lm_bytes(cfg) / w_


def model_lm_bytes(cfg):
    """Vocabulary projection (quantized) and final norm bytes of one step."""
    int4 = int(cfg.quant) == 0
    n, k = cfg.vocab, cfg.hidden
    return (n * k // 2 if int4 else n * k) + 4 * n * (k // cfg.group_size) + 4 * k


def fused_roofline(cfg, fused_ms, pasts, peak):
    """Roofline of the persistent decode-layer kernel (one launch = every
    layer of one decode step), timed by the kernel's own device global-timer
    stamps (start of CTA 0, end of the last CTA to exit) in every timed step."""
    launch_s = statistics.mean(fused_ms) / 1e3
    per_launch = statistics.mean(cfg.layers * fused_layer_bytes(cfg, p) for p in pasts)
    achieved = per_launch / launch_s / 1e9
    ratio = profile_traffic_ratio(FUSED_PROFILE)
    return {"bound": "hbm", "achieved": achieved, "peak": peak[0], "unit": "GB/s",
            "frac": achieved / peak[0],
            "traffic": ratio * per_launch if ratio is not None else None,
            "kernel": ("decode_layers_kernel (persistent, all %d layers of a decode step%s)"
                       % (cfg.layers, ", this rank's shard, o/down all-reduced in the kernel"
                          if cfg.tp_world > 1 else "")),
            "algorithmic_bytes_per_launch": per_launch, "launch_us": launch_s * 1e6,
            "launches_timed": len(fused_ms), "peak_source": peak[1],
            "traffic_source": ("ncu dram bytes of a 4-layer launch per algorithmic byte, "
                               "scaled to this launch" if ratio is not None else None)}


def _gemv_roofline(dev, model, cfg, batch, peak):
    """Live measurement of the INT4 decode GEMV (MatMulNT, M = batch) on the
    model's own quantized weights, every layer in turn (working set ~4 GB, cold
    in L2). Algorithmic bytes per launch: N*K/2 codes + 4*N*K/128 scales +
    4*M*(K+N) activations."""
    import torch
    from starlight_b200.device import BufferRef, Op, OpCode, Value
    stream = torch.cuda.ExternalStream(dev.stream())
    roles = ["q", "k", "v", "o", "gate", "up", "down"]
    launches = []
    xbufs = {}
    for role in roles + ["lm_head"]:
        ref, val = model.weight_ref(role, 0)
        n, k = val.shape
        if k not in xbufs:
            b = dev.allocate_f32(batch * k)
            dev.upload_f32(b, np.random.default_rng(k).standard_normal(batch * k, dtype=np.float32))
            xbufs[k] = b
    outs = {}
    for role in roles + ["lm_head"]:
        _, val = model.weight_ref(role, 0)
        n = val.shape[0]
        if n not in outs:
            outs[n] = dev.allocate_f32(batch * n)
    for layer in range(cfg.layers):
        for role in roles:
            launches.append(model.weight_ref(role, layer))
    launches.append(model.weight_ref("lm_head", 0))

    def run_all():
        for ref, val in launches:
            n, k = val.shape
            dev.dispatch(Op(OpCode.MatMulNT), [BufferRef(xbufs[k], 0, batch * k), ref],
                         [Value.f32((batch, k)), val], [BufferRef(outs[n], 0, batch * n)],
                         [Value.f32((batch, n))])

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3

    def timed(segment):
        # With capture on, the third and later runs of the same segment are
        # one CUDA-graph replay. The segment is recorded (host work, nothing
        # submitted) before the start event; the flush submits the replay, so
        # the events bracket device work only.
        for _ in range(3):
            segment()
            dev.flush()
            dev.synchronize()
        total = 0.0
        for _ in range(reps):
            segment()
            t0.record(stream)
            dev.flush()
            t1.record(stream)
            dev.synchronize()
            t1.synchronize()
            total += t0.elapsed_time(t1)
        return total

    ms = timed(run_all)

    def algo_bytes(val):
        n, k = val.shape
        code_bytes = n * k // 2 if int(val.quant_format) == 0 else n * k
        return code_bytes + 4 * n * (k // 128) + 4 * batch * (k + n)

    total_bytes = sum(algo_bytes(val) for _, val in launches)
    n_launch = len(launches)
    per_launch_bytes = total_bytes / n_launch
    per_launch_s = ms / 1e3 / (reps * n_launch)
    achieved = per_launch_bytes / per_launch_s / 1e9
    # Per weight shape: every layer's matrix of one role in turn.
    shapes = {}
    for role in roles + ["lm_head"]:
        subset = [lv for lv in launches if lv[1].shape == model.weight_ref(role, 0)[1].shape]
        key = "x".join(str(d) for d in subset[0][1].shape)
        if key in shapes:
            continue

        def run_subset():
            for ref, val in subset:
                n, k = val.shape
                dev.dispatch(Op(OpCode.MatMulNT), [BufferRef(xbufs[k], 0, batch * k), ref],
                             [Value.f32((batch, k)), val], [BufferRef(outs[n], 0, batch * n)],
                             [Value.f32((batch, n))])
        us = timed(run_subset) * 1e3 / (reps * len(subset))
        b = algo_bytes(subset[0][1])
        shapes[key] = {"launch_us": round(us, 2), "gbs": round(b / us / 1e3, 1),
                       "frac": round(b / us / 1e3 / peak[0], 3), "launches": len(subset)}
    # ncu traffic of one full-size launch, scaled to this mix's average launch
    # (traffic grows with the bytes streamed: each weight byte is read once).
    ratio = profile_traffic_ratio()
    traffic = ratio * per_launch_bytes if ratio is not None else None
    return {"bound": "hbm", "achieved": achieved, "peak": peak[0], "unit": "GB/s",
            "frac": achieved / peak[0], "traffic": traffic,
            "kernel": ("quantized MatMulNT, M=%d (qgemv_lane / qgemv_imma) over one decode step's "
                       "weight mix" % batch),
            "algorithmic_bytes_per_launch": per_launch_bytes, "launch_us": per_launch_s * 1e6,
            "peak_source": peak[1], "by_shape_NxK": shapes}


def rmsnorm_gbs(dev, peak):
    """RMSNorm over [4096, 4096] f32 (64 MiB in, 64 MiB out), 8 distinct
    inputs rotated so that every launch reads from HBM."""
    import torch
    from starlight_b200.device import BufferRef, Op, OpCode, Value, ValueRole
    rows, h = 4096, 4096
    stream = torch.cuda.ExternalStream(dev.stream())
    xs = [dev.allocate_f32(rows * h) for _ in range(8)]
    rng = np.random.default_rng(3)
    for b in xs:
        dev.upload_f32(b, rng.standard_normal(rows * h, dtype=np.float32))
    w = dev.allocate_f32(h)
    dev.upload_f32(w, 1.0 + 0.1 * rng.standard_normal(h, dtype=np.float32))
    outs = [dev.allocate_f32(rows * h) for _ in range(2)]
    op = Op(OpCode.RmsNorm, eps=1e-5)

    def one(i):
        dev.dispatch(op, [BufferRef(xs[i % 8], 0, rows * h), BufferRef(w, 0, h)],
                     [Value.f32((rows, h)), Value.f32((h,), ValueRole.Param)],
                     [BufferRef(outs[i % 2], 0, rows * h)], [Value.f32((rows, h))])

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 32

    def segment():
        for i in range(reps):
            one(i)

    for _ in range(3):  # eager, captured, replayed (with capture on)
        segment()
        dev.flush()
        dev.synchronize()
    segment()  # recorded only; the flush below submits the replay
    t0.record(stream)
    dev.flush()
    t1.record(stream)
    dev.synchronize()
    t1.synchronize()
    s = t0.elapsed_time(t1) / 1e3 / reps
    bytes_ = 8 * rows * h + 4 * h
    return {"shape": [rows, h], "achieved_gbs": bytes_ / s / 1e9,
            "frac": bytes_ / s / 1e9 / peak[0], "launch_us": s * 1e6}


def run_ours(args, dist: Dist):
    import torch
    from starlight_b200.device import CudaDevice, comm_unique_id
    from starlight_b200.engine import DECODE, PREFILL, LLAMA2_70B, LLAMA3_8B, Llama, LlamaConfig

    world, rank = dist.world, dist.rank
    torch.cuda.set_device(dist.local)
    dev = CudaDevice(dist.local)
    # Command capture: repeated decode steps replay as one CUDA graph each
    # (at batch 1 without tensor parallelism the layers of a step run as one
    # persistent kernel, which stamps its own start and end on the device).
    dev.set_capture(True)
    peer = None
    if world > 1:
        uid = comm_unique_id() if rank == 0 else None
        uid = dist.broadcast_bytes(uid, 128)
        dev.comm_init(uid, rank, world)
        peer = dev.peer_status()
        if not (peer["peer_allreduce"] and peer["decode_fusion"]) and rank == 0:
            print("bench: ERROR peer-memory paths off at %d ranks (%s): all-reduces fall back "
                  "to NCCL" % (world, peer), file=sys.stderr, flush=True)
    B, T = args.batch, args.prompt
    base = LLAMA3_8B if args.model == "8b" else LLAMA2_70B
    layers = base.layers if args.layers == 32 else args.layers
    max_seq = T + args.warmup + args.steps + 8
    cfg = LlamaConfig(**{**base.__dict__, "batch": B, "prefill_len": T, "max_seq": max_seq,
                         "layers": layers, "tp_rank": rank, "tp_world": world})
    model = Llama(dev, cfg)
    model.init_random(seed=8, std=0.02)
    V = cfg.vocab
    rng = np.random.default_rng(1234)
    synthetic_kv = args.synthetic_kv
    prefill_ms = None
    if synthetic_kv:
        # The decode step's cost does not depend on the cached keys/values:
        # fill the cache instead of running the prefill (--synthetic-kv).
        from starlight_b200.device import BufferRef
        kb, kn = model.kv_buffer()
        dev.fill_normal(BufferRef(kb, 0, kn), seed=99, mean=0.0, std=1.0)
        ids = rng.integers(0, V, size=B, dtype=np.uint32)
    else:
        prompt = rng.integers(0, V, size=B * T, dtype=np.uint32)
        pos = np.tile(np.arange(T, dtype=np.uint32), B)
        logits = model.step(PREFILL, prompt, pos, T, 0)
        prefill_ms = dist.max(model.last_step_ms())  # device time, untimed by the bench clock
        ids = logits.argmax(axis=1).astype(np.uint32)
    past = T
    for _ in range(args.warmup):
        logits = model.step(DECODE, ids, np.full(B, past, np.uint32), 1, past)
        ids = logits.argmax(axis=1).astype(np.uint32)
        past += 1

    sampler = ClockSampler(dist.local)
    sampler.start()
    launches0 = dev.launch_count()
    dist.barrier()
    dev.synchronize()
    device_ms = 0.0
    fused_ms, pasts = [], []
    wall = 0.0
    # NVTX range (a no-op without a profiler) so a launch list can select the
    # timed decode steps: ncu --nvtx --nvtx-include "decode/".
    torch.cuda.nvtx.range_push("decode")
    for _ in range(args.steps):
        # Host clock around the public call and the greedy pick (the step
        # returns the logits in host memory); the kernel-timing query below
        # stays outside it.
        w0 = time.perf_counter()
        logits = model.step(DECODE, ids, np.full(B, past, np.uint32), 1, past)
        ids = logits.argmax(axis=1).astype(np.uint32)
        wall += time.perf_counter() - w0
        device_ms += model.last_step_ms()
        fs = dev.decode_fusion_stats()
        if fs["last_ms"] > 0:
            fused_ms.append(fs["last_ms"])
            pasts.append(past)
        past += 1
    dev.synchronize()
    torch.cuda.nvtx.range_pop()
    dist.barrier()
    launches = dev.launch_count() - launches0
    clocks = sampler.stop()
    device_ms = dist.max(device_ms)
    wall = dist.max(wall)

    result = None
    if rank == 0:
        peak = hbm_peak()
        if len(fused_ms) == args.steps:
            roof = fused_roofline(cfg, fused_ms, pasts, peak)
            roof["step"] = {"achieved": (cfg.layers * statistics.mean(
                                fused_layer_bytes(cfg, p) for p in pasts)
                                + model_lm_bytes(cfg) / max(1, world))
                            / (device_ms / args.steps / 1e3) / 1e9,
                            "note": "whole decode step: fused layers + final norm + "
                                    "vocabulary projection bytes over the step time"}
            roof["step"]["frac"] = roof["step"]["achieved"] / peak[0]
        else:
            roof = _gemv_roofline(dev, model, cfg, B, peak) if world == 1 else None
        norm = rmsnorm_gbs(dev, peak) if world == 1 else None
        value = B * args.steps / (device_ms / 1e3)
        e2e = B * args.steps / wall
        result = {
            "metric": METRIC if args.model == "8b" else METRIC_70B, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": device_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 activations, %s weights" % ("int4" if args.model == "8b" else "int8"),
            "data": "synthetic" + (" (KV cache filled, no prefill)" if synthetic_kv else ""),
            "config": {"workload": ("llama3-8b-int4-decode" if args.model == "8b"
                                    else "llama2-70b-int8-decode"),
                       "model": "llama-dense %s shape" % args.model.upper(),
                       "batch": B, "prompt": T, "layers": cfg.layers,
                       "quant": "int4 g128" if args.model == "8b" else "int8 g128",
                       "global_batch": B, "seq_len": T,
                       "parallelism": f"tp{world}" if world > 1 else "single",
                       "l2": "no flush: %.2f GB of quantized weights streamed per step per "
                             "GPU (> 126 MB L2)" % (streamed_weight_bytes(cfg) / 1e9),
                       "commands_per_step": model.command_count(DECODE)},
            "clocks": clocks,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 2 * 4 * B,
                    "d2h_bytes_per_step": 4 * B * V},
            "gpu_launches": launches,
            "launches_per_step": launches / args.steps,
            "prefill": None if prefill_ms is None else {
                "tokens": B * T, "ms": prefill_ms, "tok_s": B * T / (prefill_ms / 1e3),
                "note": "one prefill step (untimed warm-up of the decode bench), device time, "
                        "max over ranks; first execution (no graph)"},
            "peer_paths": peer,
            "capture": dev.capture_stats(),
            "roofline": roof,
            "norm": norm,
            "weight_bytes_per_rank": model.weight_bytes(),
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            per_token, desc = oracle_decode_sample(B, T, threads)
            one, _ = oracle_decode_sample(B, T, 1)  # the reference's kernels are single-threaded
            result["cpu_baseline"] = {"value": B / per_token, "unit": "tok/s", "cores": threads,
                                      "kind": "port", "sample": desc,
                                      "single_thread": {"value": B / one, "unit": "tok/s",
                                                        "cores": 1}}
    model.close()
    dev.close()
    return result


def run_sweep(args):
    """BASELINE configs[1] and [2]: per-operator sweeps (RMSNorm, softmax,
    SiLU, Mul, residual Add, residual Add + broadcast bias, RoPE at T in
    {1, 16, 256, 4096, 16384}) and the
    quantized matmul sweep (decode GEMV at M in {1, 4, 16}, prefill at M in
    {512, 2048}; INT4 and INT8, group 128). Every case is one captured
    segment of launches over enough distinct input copies to exceed 2x L2,
    timed as a CUDA-graph replay (device time only). Prints one JSON line."""
    import torch
    from starlight_b200.device import (BufferRef, CudaDevice, Op, OpCode, QuantFormat, Value,
                                       ValueRole)
    dev = CudaDevice(0)
    dev.set_capture(True)
    stream = torch.cuda.ExternalStream(dev.stream())
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    peak = hbm_peak()[0]
    rng = np.random.default_rng(7)
    L2x2 = 252 << 20

    def timed(segment, reps=3):
        # Third and later runs are graph replays; each is recorded on the host
        # first and only its submission is bracketed by the events.
        for _ in range(3):
            segment()
            dev.flush()
            dev.synchronize()
        total = 0.0
        for _ in range(reps):
            segment()
            t0.record(stream)
            dev.flush()
            t1.record(stream)
            dev.synchronize()
            t1.synchronize()
            total += t0.elapsed_time(t1)
        return total / reps  # ms per segment

    def f32buf(n, fill=None):
        b = dev.allocate_f32(n)
        if fill is not None:
            dev.upload_f32(b, fill)
        return b

    ops = []
    for T in (1, 16, 256, 4096, 16384):
        cases = []
        H = 4096
        cases.append(("rms_norm", [T, H], 8 * T * H + 4 * H))
        if T <= 4096:
            cases.append(("softmax", [32 * T, 2048], 8 * 32 * T * 2048))
        cases.append(("silu", [T, 14336], 8 * T * 14336))
        cases.append(("mul", [T, 14336], 12 * T * 14336))
        cases.append(("add", [T, H], 12 * T * H))
        cases.append(("add_bias", [T, H], 12 * T * H + 4 * H))
        cases.append(("rope", [T, 32, 128], 8 * T * 4096 + 4 * T))
        for name, shape, algo in cases:
            n = int(np.prod(shape))
            copies = max(1, min(16, -(-L2x2 // max(1, algo))))
            data = rng.standard_normal(n, dtype=np.float32)
            ins = [f32buf(n, data) for _ in range(copies)]
            outs = [f32buf(n) for _ in range(2)]
            extra = None
            if name == "rms_norm":
                extra = f32buf(H, (1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
            elif name in ("mul", "add"):
                extra = f32buf(n, rng.standard_normal(n, dtype=np.float32))
            elif name == "add_bias":
                extra = f32buf(n + H, rng.standard_normal(n + H, dtype=np.float32))
            elif name == "rope":
                extra = dev.allocate_u32(T)
                dev.upload_u32(extra, np.arange(T, dtype=np.uint32))

            def one(i, name=name, shape=shape, n=n, ins=ins, outs=outs, extra=extra):
                x = BufferRef(ins[i % len(ins)], 0, n)
                o = BufferRef(outs[i % 2], 0, n)
                if name == "rms_norm":
                    dev.dispatch(Op(OpCode.RmsNorm, eps=1e-5), [x, BufferRef(extra, 0, H)],
                                 [Value.f32(shape), Value.f32((H,), ValueRole.Param)], [o],
                                 [Value.f32(shape)])
                elif name == "softmax":
                    dev.dispatch(Op(OpCode.Softmax), [x], [Value.f32(shape)], [o], [Value.f32(shape)])
                elif name == "silu":
                    dev.dispatch(Op(OpCode.Silu), [x], [Value.f32(shape)], [o], [Value.f32(shape)])
                elif name in ("mul", "add"):
                    code = OpCode.Mul if name == "mul" else OpCode.Add
                    dev.dispatch(Op(code), [x, BufferRef(extra, 0, n)],
                                 [Value.f32(shape), Value.f32(shape)], [o], [Value.f32(shape)])
                elif name == "add_bias":  # residual add plus broadcast [H] bias (extension op)
                    dev.dispatch(Op(OpCode.AddBias),
                                 [x, BufferRef(extra, 0, n), BufferRef(extra, n, H)],
                                 [Value.f32(shape), Value.f32(shape),
                                  Value.f32((H,), ValueRole.Param)], [o], [Value.f32(shape)])
                else:
                    dev.dispatch(Op(OpCode.Rope, theta=500000.0), [x, BufferRef(extra, 0, T)],
                                 [Value.f32((1, 32, T, 128)), Value.u32((1, T))], [o],
                                 [Value.f32((1, 32, T, 128))])

            reps_in = max(copies, 4)
            ms = timed(lambda: [one(i) for i in range(reps_in)])
            us = ms * 1e3 / reps_in
            ops.append({"op": name, "shape": shape, "us": round(us, 2),
                        "gbs": round(algo / us / 1e3, 1), "frac": round(algo / us / 1e3 / peak, 3)})
            for b in ins + outs:
                dev.release(b)
            if extra is not None:
                dev.release(extra)

    gemv, prefill = [], []
    tc_peak = bf16_peak()
    for fmt in (QuantFormat.Int4, QuantFormat.Int8):
        for k, n in ((4096, 4096), (4096, 14336), (14336, 4096), (4096, 128256)):
            row_bytes = k // 2 if fmt == QuantFormat.Int4 else k
            words = n * row_bytes // 4
            wbytes = n * row_bytes + 4 * n * (k // 128)
            copies = max(2, min(32, -(-L2x2 // wbytes)))
            codes = rng.integers(0, 2**32, size=words, dtype=np.uint64).astype(np.uint32)
            scales = (rng.random(n * (k // 128), dtype=np.float32) * 0.01).astype(np.float32)
            mats = []
            for _ in range(copies):
                cb = dev.allocate_u32(words)
                dev.upload_u32(cb, codes)
                sb = f32buf(n * (k // 128), scales)
                dev.bind_quant(cb, sb, fmt, 128)
                mats.append((cb, sb))
            for m in (1, 4, 16, 512, 2048):
                if m >= 512 and k * n > 4096 * 14336:
                    continue  # the vocabulary projection is not a prefill matmul per token block
                xb = f32buf(m * k, rng.standard_normal(m * k, dtype=np.float32))
                ob = f32buf(m * n)

                def seg(m=m, xb=xb, ob=ob, mats=mats, k=k, n=n, words=words, fmt=fmt):
                    for cb, _ in (mats if m < 512 else mats[:1]):
                        dev.dispatch(Op(OpCode.MatMulNT),
                                     [BufferRef(xb, 0, m * k), BufferRef(cb, 0, words)],
                                     [Value.f32((m, k)), Value.quantized((n, k), fmt, 128)],
                                     [BufferRef(ob, 0, m * n)], [Value.f32((m, n))])

                launches = len(mats) if m < 512 else 1
                us = timed(seg, reps=3 if m < 512 else 2) * 1e3 / launches
                if m < 512:
                    algo = wbytes + 4 * m * (k + n)
                    gemv.append({"fmt": fmt.name, "K": k, "N": n, "M": m, "us": round(us, 2),
                                 "gbs": round(algo / us / 1e3, 1),
                                 "frac": round(algo / us / 1e3 / peak, 3)})
                else:
                    flop = 2.0 * m * n * k
                    prefill.append({"fmt": fmt.name, "K": k, "N": n, "M": m, "us": round(us, 1),
                                    "tflops": round(flop / us / 1e6, 2),
                                    "frac": round(flop / us / 1e6 / tc_peak[0], 3)})
                dev.release(xb)
                dev.release(ob)
            for cb, sb in mats:
                dev.release(cb)
                dev.release(sb)
    emit({"sweep": "configs[1] ops, configs[2] quantized matmul", "hbm_peak_gbs": peak,
          "bf16_peak_tflops": tc_peak[0], "peak_source": tc_peak[1],
          "prefill_note": "frac = algorithmic 2MNK flops / measured bf16 burst peak; the tcgen05 "
                          "GEMM executes twice that (bf16 hi + lo activation planes)",
          "timing": "CUDA-graph replay of one captured segment; inputs rotated over >= 2x L2",
          "ops": ops, "gemv": gemv, "prefill": prefill})
    dev.close()
    return 0


def run_gemv_only(args):
    """One quantized MatMulNT shape, `--steps` launches after `--warmup`, on
    16 distinct weight matrices in turn (so that the launches read HBM, not
    L2): a small, self-contained case for kernel profiles."""
    import torch
    from starlight_b200.device import BufferRef, CudaDevice, Op, OpCode, QuantFormat, Value
    n, k, m = (int(v) for v in args.gemv.split(","))
    dev = CudaDevice(0)
    rng = np.random.default_rng(0)
    words = n * (k // 2) // 4
    mats = []
    for i in range(16):
        cb = dev.allocate_u32(words)
        dev.upload_u32(cb, rng.integers(0, 2**32, size=words, dtype=np.uint64).astype(np.uint32))
        sb = dev.allocate_f32(n * (k // 128))
        dev.upload_f32(sb, (rng.random(n * (k // 128), dtype=np.float32) * 0.01))
        dev.bind_quant(cb, sb, QuantFormat.Int4, 128)
        mats.append(cb)
    xb = dev.allocate_f32(m * k)
    dev.upload_f32(xb, rng.standard_normal(m * k, dtype=np.float32))
    ob = dev.allocate_f32(m * n)
    stream = torch.cuda.ExternalStream(dev.stream())

    def one(i):
        dev.dispatch(Op(OpCode.MatMulNT), [BufferRef(xb, 0, m * k), BufferRef(mats[i % 16], 0, words)],
                     [Value.f32((m, k)), Value.quantized((n, k), QuantFormat.Int4, 128)],
                     [BufferRef(ob, 0, m * n)], [Value.f32((m, n))])

    for i in range(args.warmup):
        one(i)
    dev.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        one(i)
    t1.record(stream)
    dev.synchronize()
    t1.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / max(1, args.steps)
    algo = n * k // 2 + 4 * n * (k // 128) + 4 * m * (k + n)
    emit({"gemv": [n, k, m], "launch_us": us, "algorithmic_bytes": algo,
          "gbs": algo / us / 1e3, "note": "stream launches from Python; host-bound below ~20 us"})
    dev.close()
    return 0


def main(argv=None):
    args = parse_args(argv)
    if args.gemv:
        return run_gemv_only(args)
    if args.sweep:
        return run_sweep(args)
    dist = Dist(args.gpus)
    try:
        if args.impl == "reference":
            return run_reference(args, dist)
        result = run_ours(args, dist)
        if result is not None:
            emit(result)
        return 0
    finally:
        dist.close()


if __name__ == "__main__":
    sys.exit(main())

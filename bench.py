"""Benchmark of the quantized-weight decode GEMV (the reference's headline path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mlq|reference]

Workload: one Qwen2-7B-shaped layer plus lm_head
in q4_0 -- QKV 4608x3584, O 3584x3584, gate/up 18944x3584, down 3584x18944,
lm_head 152064x3584 -- decoded at batch 1 with fp32 activations.  A step is
one pass over the six matrices (437,649,408 bytes of packed weights, larger
than the 126 MB L2, so no L2 flush is needed between steps).  Weights are
seeded N(0, 0.02) fp32 quantized by the library's reference-exact q4_0
quantizer; activations are seeded N(0, 1).

Metric: effective weight GB/s = packed weight bytes / time.  One JSON line on
stdout (rank 0).  --impl reference times the reference's own CPU
implementation (src/quant.cc linearQ40 through ThreadPool, compiled from
the reference's sources into oracle/_ref/) on this machine's host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "mini-llama_b200"
MB = 1_000_000

# The bench line's workload is BASELINE configs[1]; --workload picks one of
# the other decode configs for scaling studies (configs[4]: 70B-shaped shards).
WORKLOADS = {
    "qwen7b": {
        "name": "qwen2-7b-layer+lm_head q4_0 decode (BASELINE configs[1])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Qwen2-7B layer + lm_head, batch 1)",
        "fmt": "q4_0",
        "rows": 1,
        "matrices": [("qkv", 4608, 3584), ("o", 3584, 3584), ("gate", 18944, 3584),
                     ("up", 18944, 3584), ("down", 3584, 18944), ("lm_head", 152064, 3584)],
    },
    # The same layer through the fused entry points: the q/k/v bias added in
    # the QKV launch's store (mlq_linear_bias) and gate/up as one SwiGLU-pair
    # launch writing silu(gate) * up (mlq_linear_swiglu); same weight bytes.
    "qwen7b-fused": {
        "name": "qwen2-7b-layer+lm_head q4_0 decode, fused bias + SwiGLU (BASELINE configs[1])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Qwen2-7B layer + lm_head, batch 1)",
        "fmt": "q4_0",
        "rows": 1,
        "matrices": [("qkv", 4608, 3584), ("o", 3584, 3584), ("gate", 18944, 3584),
                     ("up", 18944, 3584), ("down", 3584, 18944), ("lm_head", 152064, 3584)],
        "fused": {"bias": ["qkv"], "pair": ["gate", "up"]},
    },
    "llama70b": {
        "name": "llama-3-70b FFN + lm_head q4_0 decode shards, batch 1 (BASELINE configs[4])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Llama-3-70B FFN + lm_head, batch 1)",
        "fmt": "q4_0",
        "rows": 1,
        "matrices": [("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672),
                     ("lm_head", 128256, 8192)],
    },
    "prefill-q4_1": {
        "name": "llama-3-8b FFN prefill q4_1, 512 rows of x (BASELINE configs[2])",
        "metric": "effective weight GB/s (q4_1 prefill GEMM, Llama-3-8B FFN, 512 rows)",
        "fmt": "q4_1",
        "rows": 512,
        "matrices": [("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)],
    },
    "llama70b-b8": {
        "name": "llama-3-70b FFN + lm_head q4_0 decode shards, batch 8 (BASELINE configs[4])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Llama-3-70B FFN + lm_head, batch 8)",
        "fmt": "q4_0",
        "rows": 8,
        "matrices": [("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672),
                     ("lm_head", 128256, 8192)],
    },
}
WORKLOAD = WORKLOADS["qwen7b"]
METRIC = WORKLOAD["metric"]
UNIT = "GB/s"


def load_pkg():
    spec = importlib.util.spec_from_file_location(
        "mini_llama_b200", PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mini_llama_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def weight_bytes(fmt, out_f, in_f):
    bs = {"q8_0": 34, "q4_0": 18, "q4_1": 20}[fmt]
    return out_f * ((in_f + 31) // 32) * bs


def bf16_peak():
    """Measured dense bf16 TFLOP/s (burst: each GEMM launch is timed alone)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, the data nvidia-smi reports)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period_s
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self.REASONS.items():
                    if mask & bit and k != "gpu_idle":
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": len(self.samples)}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU path (oracle/_ref), all host threads
# ---------------------------------------------------------------------------
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_has_avx2():
    try:
        return "avx2" in Path("/proc/cpuinfo").read_text()
    except Exception:
        return False


class ReferenceCPU:
    """The reference's CPU linearQ80/Q40/Q41 (oracle/_ref, built from its
    sources) over row samples of the workload's matrices, all host threads."""

    def __init__(self):
        sys.path.insert(0, str(ROOT))
        from oracle.oracle import Oracle, Reference  # checker / CPU baseline only
        variant = "avx2" if (cpu_has_avx2() and Reference.available("avx2")) else "scalar"
        if not Reference.available(variant):
            raise FileNotFoundError("oracle/_ref was not built")
        self.ref = Reference(variant)
        self.variant = f"libref_{variant}.so"
        self.cores = host_cores()
        self.ref.set_threads(self.cores)
        self.orc = Oracle()
        self.handles = []

    def load(self, pkg, frac):
        """Quantize the first ceil(frac*out) rows of every matrix (seeded)."""
        self.release()
        fmt = WORKLOAD["fmt"]
        self.parts = []
        for i, (name, out_f, in_f) in enumerate(WORKLOAD["matrices"]):
            rows = min(out_f, max(16 * self.cores, int(np.ceil(out_f * frac))))
            w = pkg.synth.normal((rows, in_f), seed=1000 + i, std=0.02)
            h = self.ref.hold(fmt, self.orc.quantize(fmt, w))
            x = pkg.synth.normal((WORKLOAD["rows"], in_f), seed=2000 + i)
            self.parts.append((h, x, rows, in_f, np.zeros((WORKLOAD["rows"], rows), np.float32)))
            self.handles.append(h)
        self.bytes = sum(weight_bytes(fmt, r, i) for _, _, r, i, _ in self.parts)

    def step(self):
        t0 = time.perf_counter()
        for h, x, rows, in_f, y in self.parts:
            self.ref.linear_held(WORKLOAD["fmt"], x, h, rows, y)
        return time.perf_counter() - t0

    def release(self):
        for h in self.handles:
            self.ref.release(WORKLOAD["fmt"], h)
        self.handles = []

    def calibrate(self, pkg):
        """Seconds for one full pass over the workload, from a 1/32 sample."""
        self.load(pkg, 1 / 32)
        self.step()
        t = min(self.step() for _ in range(2))
        return t * (sum(weight_bytes(WORKLOAD["fmt"], o, i) for _, o, i in WORKLOAD["matrices"])
                    / self.bytes)


def reference_cpu_baseline(pkg, seconds):
    """Bounded sample (~`seconds` of CPU work) of the workload on the
    reference's CPU path; returns the cpu_baseline dict."""
    try:
        rc = ReferenceCPU()
    except FileNotFoundError as e:
        return {"unavailable": str(e)}
    t_pass = rc.calibrate(pkg)
    frac = min(1.0, seconds / 4 / t_pass)
    rc.load(pkg, frac)
    rc.step()
    total, steps = 0.0, 0
    while total < seconds and steps < 1000:
        total += rc.step()
        steps += 1
    gbs = rc.bytes * steps / total / 1e9
    rc.release()
    return {"value": round(gbs, 3), "unit": UNIT, "kind": "reference", "cores": rc.cores,
            "sample": f"{steps} passes of linearQ40 over the first {frac:.1%} of every matrix's "
                      f"rows ({rc.bytes / MB:.1f} MB/pass), {total:.1f} s, "
                      f"ThreadPool threads = {rc.cores}, {rc.variant}"}


# ---------------------------------------------------------------------------
# Placement of the workload's matrices on N GPUs (north_star: large
# matrices row-sharded, small ones on one GPU).  A sharded call costs ~8 us
# more than a local one (fused all-gather epilogue + cross-GPU completion
# handshake), so a matrix is sharded only from SHARD_MIN_BYTES of packed
# weights on (every 70B-shaped matrix; the 7B layer's lm_head, not its
# 38 MB FFN matrices).  "local0": rank 0 computes, no gather (its consumer
# runs on rank 0); "shard": rows split across all ranks, fused all-gather.
SHARD_MIN_BYTES = 100 * MB


def gemv_passes(rows):
    """Streaming-GEMV launches for `rows` rows of x (passes of 8, 4, 2, 1
    tokens: gemv_tokens_per_pass in csrc/mlq_gemv.cu)."""
    n = 0
    while rows > 0:
        rows -= min(rows, 8 if rows >= 5 else 4 if rows >= 3 else 2 if rows == 2 else 1)
        n += 1
    return n


def launches_per_call(mlq, rows, out_f, in_f, local, pair):
    """Kernel launches of one library call in this bench (all shapes here are
    aligned for every kernel): the GEMM is an x-split launch plus the GEMM
    (per matrix of a pair, plus the SwiGLU pass); the GEMV one launch per pass."""
    if local and mlq.takes_gemm(rows, out_f, in_f):
        return 5 if pair else 2
    return gemv_passes(rows)


def placement(world):
    if world == 1:
        return {name: "shard" for name, _, _ in WORKLOAD["matrices"]}
    return {name: ("shard" if weight_bytes(WORKLOAD["fmt"], o, i) >= SHARD_MIN_BYTES else "local0")
            for name, o, i in WORKLOAD["matrices"]}


def make_inputs(torch, pkg, device, world=1, rank=0):
    """Quantized weights on the device (this rank's rows) and x vectors."""
    import importlib
    sh = importlib.import_module("mini_llama_b200.sharding")
    fmt = WORKLOAD["fmt"]
    g = torch.Generator(device=device)
    ws, xs_dev, xs_host, ranges = [], [], [], []
    for i, (name, out_f, in_f) in enumerate(WORKLOAD["matrices"]):
        place = placement(world)[name]
        rg = sh.shard_rows(out_f, world, owners=[0] if place in ("local0", "bcast0") else None)
        b, e = rg[rank]
        ranges.append(rg)
        g.manual_seed(1000 + i)
        w32 = torch.randn((out_f, in_f), generator=g, device=device, dtype=torch.float32) * 0.02
        ws.append(pkg.mlq.quantize(fmt, w32[b:e].contiguous()) if e > b else None)
        del w32
        torch.cuda.empty_cache()  # keep only the packed weights resident
        x = pkg.synth.normal((WORKLOAD["rows"], in_f), seed=2000 + i)
        xs_host.append(x)
        xs_dev.append(torch.from_numpy(x).to(device))
    torch.cuda.synchronize(device)
    return ws, xs_dev, xs_host, ranges


def run_mlq(args):
    import importlib

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    pkg = load_pkg()
    mlq = pkg.mlq
    sh = importlib.import_module("mini_llama_b200.sharding")
    fmt = WORKLOAD["fmt"]
    mats = WORKLOAD["matrices"]
    rows = WORKLOAD["rows"]
    ws, xs, xs_host, ranges = make_inputs(torch, pkg, device, world, rank)
    bytes_step = sum(weight_bytes(fmt, o, i) for _, o, i in mats)
    stream = torch.cuda.Stream(device)
    sh_stream = stream.cuda_stream
    L = mlq.lib()
    fid = mlq.FORMATS[fmt]

    # per matrix: a callable launching this rank's share of it
    calls, ybufs, launches_per_step = [], [], 0
    fused = WORKLOAD.get("fused", {})
    pair = fused.get("pair")
    if pair and world > 1 and any(placement(world)[n] != "local0" for n in pair):
        raise SystemExit("bench: a SwiGLU pair is launched on one GPU (placement local0)")
    group = None
    if world > 1:
        group = sh.PeerGroup(mlq, dist, rank, world)
        flags = group.alloc(mlq.flag_bytes())
    epoch = [0]
    for j, (name, out_f, in_f) in enumerate(mats):
        b, e = ranges[j][rank]
        if world == 1 or placement(world)[name] == "local0":
            if e == b:
                calls.append(None)
                ybufs.append(None)
                continue
            if pair and name == pair[1]:
                # the up projection streams inside the gate's pair launch
                calls.append(None)
                ybufs.append(None)
                continue
            y = torch.empty((rows, out_f), dtype=torch.float32, device=device)
            nb = ws[j].numel() // mlq.BLOCK_BYTES[fmt]
            if pair and name == pair[0]:
                ju = [m[0] for m in mats].index(pair[1])

                def call(j=j, ju=ju, out_f=out_f, in_f=in_f, y=y, nb=nb):
                    st = L.mlq_linear_swiglu(fid, ws[j].data_ptr(), ws[ju].data_ptr(), nb, out_f, in_f,
                                             xs[j].data_ptr(), rows, y.data_ptr(), sh_stream)
                    if st != 0:
                        raise RuntimeError(L.mlq_last_error().decode())
                    return y.data_ptr()
            elif name in fused.get("bias", ()):
                bias = torch.from_numpy(pkg.synth.normal((out_f,), seed=3000 + j, std=0.02)).to(device)

                def call(j=j, out_f=out_f, in_f=in_f, y=y, nb=nb, bias=bias):
                    st = L.mlq_linear_bias(fid, ws[j].data_ptr(), nb, out_f, in_f, xs[j].data_ptr(), rows,
                                           bias.data_ptr(), y.data_ptr(), sh_stream)
                    if st != 0:
                        raise RuntimeError(L.mlq_last_error().decode())
                    return y.data_ptr()
            else:
                def call(j=j, out_f=out_f, in_f=in_f, y=y, nb=nb):
                    st = L.mlq_linear(fid, ws[j].data_ptr(), nb, out_f, in_f, xs[j].data_ptr(), rows,
                                      y.data_ptr(), sh_stream)
                    if st != 0:
                        raise RuntimeError(L.mlq_last_error().decode())
                    return y.data_ptr()
            calls.append(call)
            ybufs.append(lambda y=y: y.data_ptr())
        else:
            lin = sh.ShardedLinear(mlq, fmt, out_f, in_f, rows, ranges[j], rank, group, flags)

            def call(j=j, lin=lin):
                epoch[0] += 1
                return lin(ws[j].data_ptr() if ws[j] is not None else 0, xs[j].data_ptr(), epoch[0],
                           sh_stream)
            calls.append(call)
            ybufs.append(lambda lin=lin: lin.y_ptr(epoch[0]))
        on_one_gpu = world == 1 or placement(world)[name] == "local0"
        launches_per_step += launches_per_call(mlq, rows, out_f, in_f, on_one_gpu,
                                               bool(pair) and name == pair[0])

    def step(events=None):
        for j, call in enumerate(calls):
            if call is None:
                continue
            if events is not None:
                events[j][0].record(stream)
            call()
            if events is not None:
                events[j][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
    torch.cuda.synchronize(device)

    # ---- headline: K steps on the device, inputs resident in HBM ----
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                step()
        t1.record(stream)
        t1.synchronize()
    ms = t0.elapsed_time(t1)
    if world > 1:
        tm = torch.tensor([ms], device=device)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    torch.cuda.synchronize(device)
    value = bytes_step * args.steps / (ms / 1e3) / 1e9

    # ---- per-launch durations (CUDA events on the launching stream) ----
    k2 = max(20, min(args.steps, 400))
    evs = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
            for _ in mats] for _ in range(k2)]
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(stream):
        for k in range(k2):
            step(evs[k])
    torch.cuda.synchronize(device)
    per = {name: statistics.mean(evs[k][j][0].elapsed_time(evs[k][j][1]) for k in range(k2))
           for j, (name, _, _) in enumerate(mats) if calls[j] is not None}
    peak, peak_kind = hbm_peak()
    # dominant launch: the largest share of weight bytes on this rank
    def local_bytes(j):
        b, e = ranges[j][rank]
        nbytes = weight_bytes(fmt, e - b, mats[j][2])
        return 2 * nbytes if pair and mats[j][0] == pair[0] else nbytes  # a pair launch reads both
    dj = max((j for j in range(len(mats)) if calls[j] is not None), key=local_bytes)
    dom, dom_bytes = mats[dj][0], local_bytes(dj)
    achieved = dom_bytes / (per[dom] / 1e3) / 1e9
    kernel_sum_ms = sum(per.values())
    # the dominant matrix alone, R launches back to back between two events
    # (consecutive launches overlap as in the step; the isolated per-launch
    # figure above includes each launch's ramp and drain)
    rb = 50
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        b0.record(stream)
        for _ in range(rb):
            calls[dj]()
        b1.record(stream)
    b1.synchronize()
    b2b_ms = b0.elapsed_time(b1) / rb
    if world > 1:
        tm = torch.tensor([b2b_ms], device=device)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        b2b_ms = float(tm.item())
    traffic = read_traffic() if world == 1 and WORKLOAD["name"] == WORKLOADS["qwen7b"]["name"] and dom == "lm_head" else None

    # ---- e2e: host x / host y around every call, copies inside the timed region ----
    e2e = None
    if not args.no_e2e:
        xh = [torch.from_numpy(x).pin_memory() for x in xs_host]
        yh = [torch.empty((rows, o), dtype=torch.float32).pin_memory() for _, o, _ in mats]
        ke = max(3, min(args.steps, 300))

        def e2e_step():
            if world == 1 and not fused:
                for j, (name, out_f, in_f) in enumerate(mats):
                    st = L.mlq_linear_host(fid, ws[j].data_ptr(), ws[j].numel() // mlq.BLOCK_BYTES[fmt],
                                           out_f, in_f, xh[j].data_ptr(), rows, None,
                                           yh[j].data_ptr(), local, sh_stream)
                    if st != 0:
                        raise RuntimeError(L.mlq_last_error().decode())
                return
            with torch.cuda.stream(stream):
                for j, (name, out_f, in_f) in enumerate(mats):
                    if calls[j] is None:
                        continue
                    xs[j].copy_(xh[j], non_blocking=True)
                    yp = calls[j]()
                    yh[j].copy_(sh.device_view(yp, (rows, out_f)), non_blocking=True)
                stream.synchronize()
        for _ in range(3):
            e2e_step()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(ke):
            e2e_step()
        e1.record(stream)
        e1.synchronize()
        ems = e0.elapsed_time(e1)
        if world > 1:
            tm = torch.tensor([ems], device=device)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ems = float(tm.item())
        h2d = sum(4 * rows * i for j, (_, _, i) in enumerate(mats) if calls[j] is not None)
        d2h = sum(4 * rows * o for j, (_, o, _) in enumerate(mats) if calls[j] is not None)
        e2e = {"value": round(bytes_step * ke / (ems / 1e3) / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": ke,
               "path": ("mlq_linear_host (device weights, pinned host x/y)" if world == 1 and not fused else
                        "pinned x H2D + the step's device call + y D2H, per launch")}

    err = mlq.device_error(local)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = reference_cpu_baseline(pkg, args.cpu_seconds)

    # the dominant launch's kernel: sharded calls always stream; local calls
    # follow the library's routing rule (MLQ_GEMM_ROWS_RULE)
    dom_local = world == 1 or placement(world)[dom] == "local0"
    dom_gemm = dom_local and mlq.takes_gemm(rows, mats[dj][1], mats[dj][2])
    kernel = (f"gemv_stream_kernel<{fmt}, MT={rows}, integer mode>" if rows == 1 else
              f"gemv_stream_kernel<{fmt}, MT={min(rows, 8)}, fp32 mode>" if not dom_gemm else
              f"gemm_tc_kernel<{fmt}>") + f" ({dom} launch, rank 0)"
    roof = {"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
            "traffic": traffic, "algorithmic_bytes_per_launch": dom_bytes,
            "launch_ms": round(per[dom], 5),
            "launch_ms_back_to_back": round(b2b_ms, 5),
            "achieved_back_to_back": round(dom_bytes / (b2b_ms / 1e3) / 1e9, 1),
            "all_launches_GBps": round(sum(local_bytes(j) for j in range(len(mats)) if calls[j] is not None)
                                       / (kernel_sum_ms / 1e3) / 1e9, 1),
            "per_launch_ms": {k: round(v, 5) for k, v in per.items()}}
    if dom_gemm:
        # the GEMM is tensor-bound: algorithmic flops of the dominant launch
        # (2 * rows * its rows of W * in) against the measured bf16 peak
        b_, e_ = ranges[dj][rank]
        flops = 2.0 * rows * (e_ - b_) * mats[dj][2]
        tpk, tpk_kind = bf16_peak()
        tach = flops / (per[dom] / 1e3) / 1e12
        roof.update({"bound": "tensor", "achieved": round(tach, 1), "peak": tpk, "unit": "TFLOP/s",
                     "frac": round(tach / tpk, 4), "peak_kind": tpk_kind,
                     "algorithmic_flops_per_launch": flops,
                     "achieved_back_to_back": round(flops / (b2b_ms / 1e3) / 1e12, 1),
                     "note": "three bf16 MMAs per K-step (x and W split into hi/lo): executed flops are ~3x"})
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": f"fp32 activations x {fmt} weights",
            "data": f"synthetic (seeded N(0,0.02) weights quantized to {fmt}; N(0,1) x)",
            "config": {"workload": WORKLOAD["name"], "format": fmt, "batch": rows,
                       "matrices": {n: [o, i] for n, o, i in mats},
                       "weight_bytes_per_step": bytes_step,
                       **({"fused": fused} if fused else {}),
                       "placement": placement(world) if world > 1 else "all on one GPU",
                       "l2": f"inputs larger than L2 ({bytes_step / 1e6:.1f} MB per step vs 126 MB L2); no flush"},
            "roofline": roof,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks.summary(), "device_error": err,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        group.close()
        dist.destroy_process_group()


def read_traffic():
    """DRAM bytes per lm_head launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "gemv_q4_0_lm_head.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def run_reference(args):
    """--impl reference: the reference's own CPU implementation of the path
    (oracle/_ref) on this host's cores; each step is a row sample of the
    workload sized so the whole run stays within ~2.5 minutes."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # single-process CPU code: only rank 0 runs and prints
    pkg = load_pkg()
    fmt = WORKLOAD["fmt"]
    base = {"impl": "reference", "metric": METRIC, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"fp32 activations x {fmt} weights",
            "data": f"synthetic (seeded N(0,0.02) weights quantized to {fmt}; N(0,1) x)",
            "config": {"workload": WORKLOAD["name"], "format": fmt, "batch": WORKLOAD["rows"]}}
    try:
        rc = ReferenceCPU()
    except FileNotFoundError as e:
        print(json.dumps({"impl": "reference", "unavailable": str(e)}), flush=True)
        return
    t_pass = rc.calibrate(pkg)
    budget = 150.0
    frac = min(1.0, budget / (max(1, args.steps + args.warmup) * t_pass))
    rc.load(pkg, frac)
    for _ in range(max(1, args.warmup)):
        rc.step()
    total = sum(rc.step() for _ in range(args.steps))
    value = rc.bytes * args.steps / total / 1e9
    rc.release()
    sample = (f"each step: linearQ40 over the first {frac:.2%} of every matrix's rows "
              f"({rc.bytes / MB:.1f} MB), ThreadPool threads = {rc.cores}, {rc.variant}")
    line = dict(base)
    line.update({
        "value": round(value, 3), "ms_per_step": round(total / args.steps * 1e3, 3),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "kind": "reference",
                         "cores": rc.cores, "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="mlq", choices=["mlq", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--only", default=None,
                    help="run one matrix of the workload (qkv/o/gate/up/down/lm_head), for profiling")
    ap.add_argument("--workload", default="qwen7b", choices=sorted(WORKLOADS),
                    help="qwen7b (default, the bench line) or a 70B-shaped scaling study")
    args = ap.parse_args()
    global WORKLOAD, METRIC
    WORKLOAD = dict(WORKLOADS[args.workload])
    METRIC = WORKLOAD["metric"]
    if args.only:
        WORKLOAD["matrices"] = [m for m in WORKLOAD["matrices"] if m[0] == args.only]
        if not WORKLOAD["matrices"]:
            ap.error(f"--only: no matrix named {args.only!r}")
        args.no_cpu_baseline = True
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mlq(args)


if __name__ == "__main__":
    main()

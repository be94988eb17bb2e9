"""Benchmark of the quantized-weight decode GEMV (the reference's headline path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mlq|reference]

Headline workload: one Qwen2-7B-shaped layer plus
lm_head in q4_0 -- QKV 4608x3584, O 3584x3584, gate/up 18944x3584, down
3584x18944, lm_head 152064x3584 -- decoded at batch 1 with fp32 activations.
A step is one pass over the six matrices (437,649,408 bytes of packed
weights, larger than the 126 MB L2, so no L2 flush is needed between steps),
launched as one batch (mlq_linear_batch).  Weights are seeded N(0, 0.02) fp32
drawn by mini-llama_b200/synth.py (the same numbers the CPU arm draws) and
quantized by the library's reference-exact quantizer; activations are seeded
N(0, 1).

Metric: effective weight GB/s = packed weight bytes / time.  One JSON line on
stdout (rank 0).  The line also carries, under "extra", the other BASELINE
configs measured in the same run (config 1 q8_0 with rotating weight copies,
config 3 prefill, config 4 batched decode, config 5 70B shards at batch 1
and 8) and per-format decode fractions ("formats").

--impl reference times the reference's own CPU implementation (src/quant.cc
linearQ40 through ThreadPool, compiled from the reference's sources into
oracle/_ref/) on this machine's host cores.
"""
from __future__ import annotations

import argparse
import importlib
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


def llama8b_layers():
    """Config 4: 32 Llama-3-8B layers (Q, K, V, O, gate, up, down) + lm_head."""
    mats = []
    for l in range(32):
        mats += [(f"l{l}.q", 4096, 4096), (f"l{l}.k", 1024, 4096), (f"l{l}.v", 1024, 4096),
                 (f"l{l}.o", 4096, 4096), (f"l{l}.gate", 14336, 4096), (f"l{l}.up", 14336, 4096),
                 (f"l{l}.down", 4096, 14336)]
    return mats + [("lm_head", 128256, 4096)]


def llama8b_shared_x():
    """K and V read Q's x, up reads gate's x (src/forward.cc:425-435, 574-582)."""
    share = {}
    for l in range(32):
        share.update({f"l{l}.k": f"l{l}.q", f"l{l}.v": f"l{l}.q", f"l{l}.up": f"l{l}.gate"})
    return share


QWEN7B = [("qkv", 4608, 3584), ("o", 3584, 3584), ("gate", 18944, 3584), ("up", 18944, 3584),
          ("down", 3584, 18944), ("lm_head", 152064, 3584)]
LLAMA70B = [("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672), ("lm_head", 128256, 8192)]

# At N > 1 the matrices named in "shard" are row-sharded across every GPU
# (fused all-gather); the others run on rank 0 (north_star: FFN and lm_head
# sharded, small matrices on one GPU).  "share_x": matrices that read another
# matrix's x, as in the model (the library runs consecutive batched-decode
# matrices on one x as one grouped launch).
WORKLOADS = {
    "qwen7b": {
        "name": "qwen2-7b-layer+lm_head q4_0 decode (BASELINE configs[1])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Qwen2-7B layer + lm_head, batch 1)",
        "fmt": "q4_0", "rows": 1, "matrices": QWEN7B,
        # qkv and o stay whole on rank 0: a sharded launch has a fixed cost
        # (stores to every rank, the system-scope release) that outweighs
        # half of a 5-9 MB matrix
        "shard": {"gate", "up", "down", "lm_head"},
    },
    # The same layer through the fused entry points: the q/k/v bias added in
    # the QKV launch's store and gate/up as one SwiGLU-pair launch writing
    # silu(gate) * up (mlq_linear_swiglu); same weight bytes.  One GPU.
    "qwen7b-fused": {
        "name": "qwen2-7b-layer+lm_head q4_0 decode, fused bias + SwiGLU (BASELINE configs[1])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Qwen2-7B layer + lm_head, batch 1)",
        "fmt": "q4_0", "rows": 1, "matrices": QWEN7B, "shard": set(),
        "fused": {"bias": ["qkv"], "pair": ["gate", "up"]},
    },
    "config1-q8_0": {
        "name": "qwen2-0.5b FFN-up q8_0 decode, 4864x896 (BASELINE configs[0])",
        "metric": "effective weight GB/s (q8_0 decode GEMV, 4864x896, batch 1)",
        "fmt": "q8_0", "rows": 1, "matrices": [("up", 4864, 896)], "shard": set(),
        # 4.6 MB fits in L2: every step reads the next of 64 copies (296 MB)
        "rotate": 64,
    },
    "prefill-q4_1": {
        "name": "llama-3-8b FFN prefill q4_1, 512 rows of x (BASELINE configs[2])",
        "metric": "effective weight GB/s (q4_1 prefill GEMM, Llama-3-8B FFN, 512 rows)",
        "fmt": "q4_1", "rows": 512,
        "matrices": [("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)],
        "shard": set(),
    },
    "llama8b-b16": {
        "name": "llama-3-8b 32 layers + lm_head q8_0 batched decode, batch 16 (BASELINE configs[3])",
        "metric": "effective weight GB/s (q8_0 batched decode, Llama-3-8B, batch 16)",
        "fmt": "q8_0", "rows": 16, "matrices": llama8b_layers(), "share_x": llama8b_shared_x(),
        "shard": {n for n, _, _ in llama8b_layers() if n.split(".")[-1] in ("gate", "up", "down", "lm_head")},
    },
    "llama70b": {
        "name": "llama-3-70b FFN + lm_head q4_0 decode shards, batch 1 (BASELINE configs[4])",
        "metric": "effective weight GB/s (q4_0 decode GEMV, Llama-3-70B FFN + lm_head, batch 1)",
        "fmt": "q4_0", "rows": 1, "matrices": LLAMA70B, "shard": {"gate", "up", "down", "lm_head"},
    },
    "llama70b-b8": {
        "name": "llama-3-70b FFN + lm_head q4_0 decode shards, batch 8 (BASELINE configs[4])",
        "metric": "effective weight GB/s (q4_0 decode, Llama-3-70B FFN + lm_head, batch 8)",
        "fmt": "q4_0", "rows": 8, "matrices": LLAMA70B, "shard": {"gate", "up", "down", "lm_head"},
        "share_x": {"up": "gate"},
    },
    # one matrix per format at one row, for per-format profiles of the GEMV
    "gemv-q8_0": {
        "name": "llama-3-8b FFN gate q8_0 decode, 14336x4096, batch 1",
        "metric": "effective weight GB/s (q8_0 decode GEMV, 14336x4096, batch 1)",
        "fmt": "q8_0", "rows": 1, "matrices": [("gate", 14336, 4096)], "shard": set(), "rotate": 8,
    },
    "gemv-q4_1": {
        "name": "llama-3-8b FFN gate q4_1 decode, 14336x4096, batch 1",
        "metric": "effective weight GB/s (q4_1 decode GEMV, 14336x4096, batch 1)",
        "fmt": "q4_1", "rows": 1, "matrices": [("gate", 14336, 4096)], "shard": set(), "rotate": 8,
    },
}
# measured after the headline in the default run (extra key of the line)
EXTRAS_N1 = ["config1-q8_0", "prefill-q4_1", "llama8b-b16", "llama70b", "llama70b-b8"]
EXTRAS_NGT1 = ["llama8b-b16", "llama70b", "llama70b-b8"]
UNIT = "GB/s"


def load_pkg():
    if "mini_llama_b200" in sys.modules:
        return sys.modules["mini_llama_b200"]
    spec = importlib.util.spec_from_file_location(
        "mini_llama_b200", PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mini_llama_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def weight_bytes(fmt, out_f, in_f):
    bs = {"q8_0": 34, "q4_0": 18, "q4_1": 20}[fmt]
    return out_f * ((in_f + 31) // 32) * bs


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return None


def hbm_peak():
    pk = _peaks()
    return (float(pk["hbm_gbs"]), "measured") if pk else (6650.0, "fallback")


def bf16_peak():
    """Measured dense bf16 TFLOP/s (burst: each GEMM launch is timed alone)."""
    pk = _peaks()
    return (float(pk["bf16_tflops"]), "measured") if pk else (1590.0, "fallback")


def config_of(wl, world):
    """The config dict both arms print (same keys, same values)."""
    return {"workload": wl["name"], "format": wl["fmt"], "batch": wl["rows"],
            "matrices": {n: [o, i] for n, o, i in wl["matrices"]} if len(wl["matrices"]) <= 8
            else f"{len(wl['matrices'])} matrices",
            "weight_bytes_per_step": sum(weight_bytes(wl["fmt"], o, i) for _, o, i in wl["matrices"]),
            "sharded_at_n_gt_1": sorted(wl["shard"]) if len(wl["shard"]) <= 8 else "FFN + lm_head",
            "placement": "all on one GPU" if world == 1 else "listed matrices row-sharded, others on rank 0",
            "l2": "inputs larger than L2 (no flush)" if not wl.get("rotate")
            else f"{wl['rotate']} rotating weight copies per pass (> 2x L2)"}


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
        med = statistics.median(self.samples) if self.ok and self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


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
    sources) over the first rows of the workload's matrices (the same seeded
    weights and x as the GPU arm), all host threads."""

    def __init__(self, wl):
        sys.path.insert(0, str(ROOT))
        from oracle.oracle import Oracle, Reference  # checker / CPU baseline only
        variant = "avx2" if (cpu_has_avx2() and Reference.available("avx2")) else "scalar"
        if not Reference.available(variant):
            raise FileNotFoundError("oracle/_ref was not built")
        self.wl = wl
        self.ref = Reference(variant)
        self.variant = f"libref_{variant}.so"
        self.cores = host_cores()
        self.ref.set_threads(self.cores)
        self.orc = Oracle()
        self.handles = []

    def load(self, pkg, frac):
        """Quantize the first ceil(frac*out) rows of every matrix."""
        self.release()
        fmt = self.wl["fmt"]
        self.parts = []
        for i, (name, out_f, in_f) in enumerate(self.wl["matrices"]):
            rows = min(out_f, max(16 * self.cores, int(np.ceil(out_f * frac))))
            w = pkg.synth.normal((rows, in_f), seed=1000 + i, std=0.02)
            h = self.ref.hold(fmt, self.orc.quantize(fmt, w))
            x = pkg.synth.normal((self.wl["rows"], in_f), seed=2000 + i)
            self.parts.append((h, x, rows, in_f, np.zeros((self.wl["rows"], rows), np.float32)))
            self.handles.append(h)
        self.bytes = sum(weight_bytes(fmt, r, i) for _, _, r, i, _ in self.parts)

    def step(self):
        t0 = time.perf_counter()
        for h, x, rows, in_f, y in self.parts:
            self.ref.linear_held(self.wl["fmt"], x, h, rows, y)
        return time.perf_counter() - t0

    def release(self):
        for h in self.handles:
            self.ref.release(self.wl["fmt"], h)
        self.handles = []

    def calibrate(self, pkg):
        """Seconds for one full pass over the workload, from a 1/32 sample."""
        self.load(pkg, 1 / 32)
        self.step()
        t = min(self.step() for _ in range(2))
        return t * (sum(weight_bytes(self.wl["fmt"], o, i) for _, o, i in self.wl["matrices"])
                    / self.bytes)


def reference_cpu_baseline(pkg, wl, seconds):
    """Bounded sample (~`seconds` of CPU work) of the workload on the
    reference's CPU path; returns the cpu_baseline dict."""
    try:
        rc = ReferenceCPU(wl)
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
            "sample": f"{steps} passes of linearQ{wl['fmt'][1]}{wl['fmt'][3]} over the first {frac:.1%} of "
                      f"every matrix's rows ({rc.bytes / MB:.1f} MB/pass), {total:.1f} s, "
                      f"ThreadPool threads = {rc.cores}, {rc.variant}"}


# ---------------------------------------------------------------------------
# the GPU arm
# ---------------------------------------------------------------------------
def gemm_split(out_f, in_f, rows, sms):
    """gemm_split of csrc/mlq_gemm.cu (launch counting only)."""
    nt = 16 if rows <= 16 else 32 if rows <= 32 else 64 if rows <= 64 else 128
    tiles = -(-out_f // 128) * -(-rows // nt)
    chunks = -(-in_f // 256)
    if tiles >= sms or chunks < 2:
        return 1
    s = max(1, min(sms // tiles, 8, chunks))
    per = -(-chunks // s)
    return -(-chunks // per)


def launches_of(mlq, rows, out_f, in_f, gemm_ok, pair, sms):
    """Kernel launches of one library call: the batched-decode GEMM is an
    x-split launch and the GEMM; the bf16 GEMM an x-split launch, the GEMM
    and (split-K) a reduction; per matrix of a pair plus the SwiGLU pass; the
    GEMV one launch per pass of <= 8 rows (pairs stream together)."""
    if gemm_ok and mlq.takes_bgemm(rows, out_f, in_f):
        return 5 if pair else 2  # x split, GEMM (per matrix of a pair, plus SwiGLU)
    if gemm_ok and mlq.takes_gemm(rows, out_f, in_f):
        per = 2 + (gemm_split(out_f, in_f, rows, sms) > 1)
        return 2 * per + 1 if pair else per
    n = 0
    while rows > 0:
        rows -= min(rows, 8 if rows >= 5 else 4 if rows >= 3 else 2 if rows == 2 else 1)
        n += 1
    return n


class Ctx:
    """Process-wide state of the GPU arm (one process per GPU)."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.device)
        self.pkg = load_pkg()
        self.mlq = self.pkg.mlq
        self.sh = importlib.import_module("mini_llama_b200.sharding")
        self.stream = torch.cuda.Stream(self.device)
        self.sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.group = self.flags = None
        if self.world > 1:
            self.group = self.sh.PeerGroup(self.mlq, dist, self.rank, self.world)
            self.flags = self.group.alloc(self.mlq.flag_bytes())
        self.tok = torch.zeros(1, device=self.device)
        self.epoch = 0  # last epoch published on self.flags (every workload continues it)

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, fn):
        """ms of fn()'s GPU work on the bench stream, CUDA events, max over
        ranks.  At N > 1 the ranks first meet in an NCCL all-reduce on the
        bench stream, so every rank's start event fires after the same device
        rendezvous (not after a host barrier, which releases ranks at
        different times)."""
        torch = self.torch
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            self.dist.barrier()
            with torch.cuda.stream(self.stream):
                self.dist.all_reduce(self.tok)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(self.stream)
        fn()
        t1.record(self.stream)
        t1.synchronize()
        return self.max_over_ranks(t0.elapsed_time(t1))

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.group.close()
            self.dist.destroy_process_group()


class Step:
    """One workload on this rank: resident packed weights (this rank's rows),
    x, y, and the batches that launch a whole step with one library call."""

    def __init__(self, ctx, wl):
        torch, mlq, sh, pkg = ctx.torch, ctx.mlq, ctx.sh, ctx.pkg
        self.ctx, self.wl = ctx, wl
        fmt, rows, mats = wl["fmt"], wl["rows"], wl["matrices"]
        self.fmt, self.rows = fmt, rows
        # epochs continue the sequence of every earlier workload on ctx.flags
        self.plan = sh.StepPlan(mats, ctx.world, ctx.rank, shard=wl["shard"], epoch0=ctx.epoch)
        fused = wl.get("fused", {})
        pair = fused.get("pair")
        if pair and ctx.world > 1:
            raise SystemExit("bench: the fused workload runs on one GPU")
        self.keep = []
        self.w, self.x, self.y = {}, {}, {}
        self.bytes_step = sum(weight_bytes(fmt, o, i) for _, o, i in mats)
        # packed weights of this rank's rows, drawn row chunk by row chunk
        for i, (name, out_f, in_f) in enumerate(mats):
            b, e = self.plan.rows(name)
            if not self.plan.active(name) or e == b:
                self.w[name] = None
            else:
                self.w[name] = self._weights(i, b, e, in_f)
            src = wl.get("share_x", {}).get(name)
            if src is not None:
                self.x[name] = self.x[src]  # the model's shared input (defined earlier in the list)
            else:
                self.x[name] = torch.from_numpy(pkg.synth.normal((rows, in_f), seed=2000 + i)).to(ctx.device)
        torch.cuda.empty_cache()
        # per op (call order): the matrix, the launch count, the ops of both y parities
        shard_names = self.plan.sharded
        self.slab = None
        if shard_names:
            self.slab = sh.GatherSlab(ctx.group, [4 * rows * dict((n, o) for n, o, _ in mats)[n]
                                                  for n in shard_names])
        self.gathers = [[], []]
        self.names, self.op_bytes, self.launches = [], [], []
        self.one_run = False  # every op of the step in one run launch (set below)
        # A step whose ops all join one run launch (one row each, at most
        # RUN_MAX_OPS of them) publishes once, at the end of that launch: its
        # gathers wait there too (defer_wait 0), with no separate wait kernel.
        # Otherwise every gathered op only publishes and the step ends with
        # one mlq_gather_wait.
        active = [(n, i) for n, _, i in mats if self.plan.active(n) and not (pair and n == pair[1])]
        one_launch = (rows == 1 and not pair and 2 <= len(active) <= mlq.RUN_MAX_OPS
                      and all(mlq.joins_run(fmt, rows, i) for _, i in active))
        ops = [[], []]
        grp = None  # (x pointer, matrices) of the open batched-decode group
        for i, (name, out_f, in_f) in enumerate(mats):
            if not self.plan.active(name) or (pair and name == pair[1]):
                continue
            b, e = self.plan.rows(name)
            wp = self.w[name].data_ptr() if self.w[name] is not None else 0
            if self.plan.place[name] == "shard":
                grp = None  # a gathered op is never grouped
                k = shard_names.index(name)
                for p in (0, 1):
                    g = mlq.make_gather(ctx.world, ctx.rank, b, e, self.slab.peer_ptrs(p, k),
                                        ctx.flags.peers, epoch=1, defer_wait=not one_launch)
                    self.gathers[p].append(g)
                    ops[p].append(mlq.linear_op(fmt, wp, out_f, in_f, self.x[name].data_ptr(), rows,
                                                self.slab.local_ptr(p, k), gather=g))
                # a shard takes the batched-decode GEMM or the streaming GEMV
                # (the sharded call has no bf16 GEMM route)
                self.launches.append(launches_of(mlq, rows, e - b, in_f, mlq.takes_bgemm(rows, e - b, in_f), False,
                                                 ctx.sms))
            else:
                y = torch.empty((rows, out_f), dtype=torch.float32, device=ctx.device)
                self.y[name] = y
                w_up = bias = None
                if pair and name == pair[0]:
                    w_up = self.w[pair[1]].data_ptr()
                if name in fused.get("bias", ()):
                    bt = torch.from_numpy(pkg.synth.normal((out_f,), seed=3000 + i, std=0.02)).to(ctx.device)
                    self.keep.append(bt)
                    bias = bt.data_ptr()
                op = mlq.linear_op(fmt, wp, out_f, in_f, self.x[name].data_ptr(), rows, y.data_ptr(),
                                   w_up_ptr=w_up, bias_ptr=bias)
                ops[0].append(op)
                ops[1].append(op)
                n_l = launches_of(mlq, rows, out_f, in_f, True, w_up is not None, ctx.sms)
                # the library runs consecutive batched-decode ops on one x as
                # one grouped launch (up to 4 matrices): no launches of their own
                xp = self.x[name].data_ptr()
                if w_up is None and mlq.takes_bgemm(rows, out_f, in_f):
                    if grp is not None and grp[0] == xp and grp[1] < 4:
                        grp = (xp, grp[1] + 1)
                        n_l = 0
                    else:
                        grp = (xp, 1)
                else:
                    grp = None
                self.launches.append(n_l)
            self.names.append(name)
            nb = weight_bytes(fmt, e - b, in_f)
            self.op_bytes.append(2 * nb if (pair and name == pair[0]) else nb)
        self.ops = ops
        # How the library launches the step (mlq_linear_batch): consecutive
        # one-row ops that join a run (local or gathered) take two launches
        # per 8 ops -- the x slicing and the persistent run kernel -- instead
        # of one launch each; other runs of local one-launch GEMVs end with
        # the library's join launch.
        seq = [(n, o, i) for n, o, i in mats if self.plan.active(n) and not (pair and n == pair[1])]

        def member(n, i):
            return rows == 1 and mlq.joins_run(fmt, rows, i) and not (pair and n == pair[0])

        def one_gemv(n, o, i):
            return (self.plan.place[n] != "shard" and rows <= 2 and not mlq.takes_bgemm(rows, o, i)
                    and not mlq.takes_gemm(rows, o, i))
        k = 0
        while k < len(seq):
            j = k
            while j < len(seq) and member(seq[j][0], seq[j][2]):
                j += 1
            if j - k >= 2:
                self.launches.append(2 * -(-(j - k) // mlq.RUN_MAX_OPS) - (j - k))
                self.one_run = j - k == len(seq)
                k = j
                continue
            j = k
            while j < len(seq) and one_gemv(*seq[j]):
                j += 1
            if j - k >= 2:
                self.launches.append(1)
            k = max(j, k + 1)
        # the step's one cross-rank wait: every rank's highest epoch of the step
        self.waiter = (mlq.make_gather(ctx.world, ctx.rank, 0, 0, [0] * ctx.world, ctx.flags.peers, epoch=1)
                       if shard_names and not one_launch else None)
        if self.waiter is not None and ctx.world > 1:
            self.launches.append(1)  # mlq_gather_wait's kernel, once per step
        self.batch = [mlq.Batch(ops[0]), mlq.Batch(ops[1])]
        self.single = [[mlq.Batch([op]) for op in ops[p]] for p in (0, 1)]
        # rotating copies (an L2-sized matrix): one batch per copy
        self.rot = None
        if wl.get("rotate"):
            name = mats[0][0]
            copies = [self.w[name]] + [self.w[name].clone() for _ in range(wl["rotate"] - 1)]
            self.keep += copies
            rops = []
            for c in copies:
                op = mlq.LinearOp.from_buffer_copy(ops[0][0])
                op.w = c.data_ptr()
                rops.append(op)
            self.rot = mlq.Batch(rops)
        self.steps_run = 0
        torch.cuda.synchronize(ctx.device)

    def _weights(self, i, b, e, in_f):
        """Packed blocks of rows [b, e) of matrix i: N(0, 0.02) from seed
        1000 + i (synth.normal_torch at the rows' offset), quantized on the GPU."""
        torch, mlq, pkg = self.ctx.torch, self.ctx.mlq, self.ctx.pkg
        rb = ((in_f + 31) // 32) * mlq.BLOCK_BYTES[self.fmt]
        out = torch.empty((e - b) * rb, dtype=torch.uint8, device=self.ctx.device)
        chunk = max(8, (1 << 26) // in_f // 8 * 8)
        for r0 in range(b, e, chunk):
            r1 = min(e, r0 + chunk)
            w32 = pkg.synth.normal_torch((r1 - r0, in_f), seed=1000 + i, std=0.02, device=self.ctx.device,
                                         offset=r0 * in_f)
            out[(r0 - b) * rb:(r1 - b) * rb] = mlq.quantize(self.fmt, w32)
            del w32
        return out

    def _set_epochs(self, parity, epochs):
        for g, ep in zip(self.gathers[parity], epochs):
            g.epoch = ep
        if self.waiter is not None and epochs:
            self.waiter.epoch = max(epochs)

    def _wait(self, stream):
        """The deferred wait of the step's sharded ops (their y complete here)."""
        if self.waiter is not None:
            self.ctx.mlq.gather_wait(self.waiter, stream)

    def step(self):
        """One pass over the workload: one library call."""
        if self.rot is not None:
            self.rot.run(self.ctx.stream.cuda_stream)
            return
        parity, epochs = self.plan.next_step()
        self._set_epochs(parity, epochs)
        self.batch[parity].run(self.ctx.stream.cuda_stream)
        self._wait(self.ctx.stream.cuda_stream)
        self.steps_run += 1

    def step_host(self, host_batches):
        parity, epochs = self.plan.next_step()
        self._set_epochs(parity, epochs)
        host_batches[parity].run_host(self.ctx.local, self.ctx.stream.cuda_stream)

    def per_launch_ms(self, rounds):
        """Mean CUDA-event time of each op launched on its own (events around
        every op of a step, `rounds` steps).  Each round is queued behind a
        ~1 ms sleep kernel, so the host has launched the whole round before
        the GPU reaches it and no event pair spans GPU idle time."""
        torch, s = self.ctx.torch, self.ctx.stream
        n = len(self.names)
        evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(n)] for _ in range(rounds)]
        for r in range(rounds):
            parity, epochs = self.plan.next_step()
            self._set_epochs(parity, epochs)
            with torch.cuda.stream(s):
                torch.cuda._sleep(2_000_000)
            for j in range(n):
                evs[r][j][0].record(s)
                self.single[parity][j].run(s.cuda_stream)
                evs[r][j][1].record(s)
            self._wait(s.cuda_stream)  # outside the events: the ranks stay in step
        torch.cuda.synchronize(self.ctx.device)
        return [statistics.mean(evs[r][j][0].elapsed_time(evs[r][j][1]) for r in range(rounds))
                for j in range(n)]

    def back_to_back_ms(self, j, reps):
        """One local op launched `reps` times in a row between two events (the
        launches overlap as inside a step).  None for a sharded op: its calls
        are tied to the peers' calls."""
        torch, s = self.ctx.torch, self.ctx.stream
        if self.plan.place[self.names[j]] == "shard":
            return None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(self.ctx.device)
        e0.record(s)
        for _ in range(reps):
            self.single[0][j].run(s.cuda_stream)
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    def parity_check(self):
        """Every sharded matrix: the gathered y of its last call on this rank
        against one local mlq_linear of the whole matrix (regenerated from
        its seed) on the same x; max relative L2 error of an output row."""
        torch, mlq = self.ctx.torch, self.ctx.mlq
        worst, where = 0.0, None
        for k, name in enumerate(self.plan.sharded):
            i, (_, out_f, in_f) = next((i, m) for i, m in enumerate(self.wl["matrices"]) if m[0] == name)
            parity = (self.plan.calls[name] - 1) & 1
            got = self.ctx.sh.device_view(self.slab.local_ptr(parity, k), (self.rows, out_f)).clone()
            full = self._weights(i, 0, out_f, in_f)
            ref = mlq.linear(self.fmt, full, out_f, in_f, self.x[name])
            torch.cuda.synchronize(self.ctx.device)
            err = (torch.linalg.norm((got - ref).double(), dim=1) /
                   torch.linalg.norm(ref.double(), dim=1).clamp_min(1e-30)).max().item()
            if err > worst:
                # the shard (writing rank) whose rows differ most
                shard_err = []
                for r, (b, e) in enumerate(self.plan.ranges[name]):
                    d = (got[:, b:e] - ref[:, b:e]).double().norm().item() if e > b else 0.0
                    shard_err.append(round(d / max(ref[:, b:e].double().norm().item(), 1e-30), 4) if e > b else 0.0)
                worst, where = err, {"matrix": name, "rank": self.ctx.rank, "shard_rel_l2": shard_err}
            del full, ref, got
        torch.cuda.empty_cache()
        if where is not None and worst > 1e-3:
            print(f"bench: parity of {where}: {worst:.3e}", file=sys.stderr, flush=True)
        return self.ctx.max_over_ranks(worst)


def run_workload(ctx, wl, steps, warmup, full=False, args=None):
    """Times `steps` steps of a workload (after `warmup`); with `full`, also the
    per-launch roofline, the back-to-back dominant launch, the e2e path and
    (N > 1) the parity gate.  Returns a dict (on every rank)."""
    torch, mlq = ctx.torch, ctx.mlq
    st = Step(ctx, wl)
    for _ in range(max(3, warmup)):
        st.step()
    torch.cuda.synchronize(ctx.device)
    res = {}
    if ctx.world > 1 and st.plan.sharded:
        res["parity_max_rel_l2"] = st.parity_check()
    clocks = ClockSampler(ctx.local)
    with clocks:
        ms = ctx.timed(lambda: [st.step() for _ in range(steps)])
    per_step_bytes = st.bytes_step * (1 if not wl.get("rotate") else wl["rotate"])
    res.update({"value": round(per_step_bytes * steps / (ms / 1e3) / 1e9, 2),
                "ms_per_step": round(ms / steps, 5), "steps": steps, "clocks": clocks.summary(),
                "gpu_launches_per_step": sum(st.launches) * (wl.get("rotate") or 1)})
    # the dominant op of this rank and its roofline
    rounds = max(5, min(steps, 200)) if full else 5
    if wl.get("rotate"):
        per_launch = ms / steps / wl["rotate"]
        res["roofline"] = _roof(st.op_bytes[0], per_launch, None, wl, ctx, st, 0)
    else:
        per = st.per_launch_ms(rounds)
        dj = max(range(len(st.names)), key=lambda j: st.op_bytes[j])
        b2b = st.back_to_back_ms(dj, 50) if full else None
        res["roofline"] = _roof(st.op_bytes[dj], per[dj], b2b, wl, ctx, st, dj)
        res["roofline"]["per_launch_ms"] = {n: round(v, 5) for n, v in zip(st.names, per)}
        res["roofline"]["all_launches_GBps"] = round(sum(st.op_bytes) / (sum(per) / 1e3) / 1e9, 1)
        if st.one_run:
            # the step is one run launch (all ops local, one row each): that
            # kernel is the timed region's dominant kernel; the single-op
            # figures stay beside it
            single = res["roofline"]
            step_ms = ms / steps
            ach = sum(st.op_bytes) / (step_ms / 1e3) / 1e9
            peak, kind = hbm_peak()
            res["roofline"] = {
                "bound": "hbm",
                "kernel": f"gemv_run_kernel<{wl['fmt']}> (the step's {len(st.names)} products in one persistent "
                          f"launch, after its x-slicing launch; rank {ctx.rank})",
                "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "peak_kind": peak_kind_text(kind), "traffic": None,
                "algorithmic_bytes_per_launch": sum(st.op_bytes), "launch_ms": round(step_ms, 5),
                "single_op_launches": single}
    if full and not (args and args.no_e2e):
        res["e2e"] = _e2e(ctx, st, steps)
    ctx.epoch = st.plan.epoch
    del st
    torch.cuda.empty_cache()
    return res


def _roof(nbytes, launch_ms, b2b_ms, wl, ctx, st, j):
    mlq = ctx.mlq
    peak, kind = hbm_peak()
    name = st.names[j]
    out_f, in_f = next((o, i) for n, o, i in wl["matrices"] if n == name)
    b, e = st.plan.rows(name)
    local = st.plan.place[name] != "shard"
    bgemm = mlq.takes_bgemm(wl["rows"], e - b, in_f) if e > b else False
    gemm = bgemm or (local and mlq.takes_gemm(wl["rows"], out_f, in_f))
    kernel = (f"bgemm_kernel<{wl['fmt']}> (batched decode)" if bgemm else
              f"gemm_tc_kernel<{wl['fmt']}>" if gemm else
              f"gemv_stream_kernel<{wl['fmt']}, MT={min(wl['rows'], 8)}, "
              f"{'integer' if wl['rows'] == 1 else 'fp32'} mode>") + f" ({name} launch, rank {ctx.rank})"
    ach = nbytes / (launch_ms / 1e3) / 1e9
    r = {"bound": "hbm", "kernel": kernel, "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
         "frac": round(ach / peak, 4), "peak_kind": peak_kind_text(kind),
         "traffic": None, "algorithmic_bytes_per_launch": nbytes, "launch_ms": round(launch_ms, 5)}
    if b2b_ms:
        r["launch_ms_back_to_back"] = round(b2b_ms, 5)
        r["achieved_back_to_back"] = round(nbytes / (b2b_ms / 1e3) / 1e9, 1)
        r["frac_back_to_back"] = round(nbytes / (b2b_ms / 1e3) / 1e9 / peak, 4)
    if gemm:
        flops = 2.0 * wl["rows"] * (e - b) * in_f
        tpk, tkind = bf16_peak()
        tach = flops / (launch_ms / 1e3) / 1e12
        r.update({"bound": "tensor" if wl["rows"] >= 64 else "hbm",
                  "tensor_achieved_TFLOPs": round(tach, 1), "tensor_peak_TFLOPs": tpk,
                  "tensor_frac": round(tach / tpk, 4), "algorithmic_flops_per_launch": flops})
        if wl["rows"] >= 64:
            r.update({"achieved": round(tach, 1), "peak": tpk, "unit": "TFLOP/s", "frac": round(tach / tpk, 4),
                      "peak_kind": peak_kind_text(tkind)})
    return r


def peak_kind_text(kind):
    return "of measured (MEASURED_PEAKS.json)" if kind == "measured" else "of fallback"


def _e2e(ctx, st, steps):
    """The same step through mlq_linear_batch_host: pinned host x and y, the
    copies and one synchronisation inside every step."""
    torch, mlq = ctx.torch, ctx.mlq
    # every op's host x, and every host y, back to back in one pinned buffer
    # each (op order): the library then moves each direction in one copy
    shape = {n: (i, o) for n, o, i in st.wl["matrices"]}
    # ops that read one device x (share_x) read one host slice too
    owner = {}
    for name in st.names:
        owner[name] = next((m for m in owner if st.x[m] is st.x[name]), name)
    nx = sum(st.rows * shape[n][0] for n in st.names if owner[n] == n)
    ny = sum(st.rows * shape[n][1] for n in st.names)
    xbuf = torch.empty(nx, dtype=torch.float32).pin_memory()
    ybuf = torch.empty(ny, dtype=torch.float32).pin_memory()
    hx, hy, host_batches = {}, {}, []
    xoff = yoff = 0
    for name in st.names:
        i_f, o_f = shape[name]
        if owner[name] == name:
            hx[name] = xbuf[xoff:xoff + st.rows * i_f].view(st.rows, i_f)
            hx[name].copy_(st.x[name].cpu().view(st.rows, i_f))
            xoff += st.rows * i_f
        else:
            hx[name] = hx[owner[name]]
        hy[name] = ybuf[yoff:yoff + st.rows * o_f].view(st.rows, o_f)
        yoff += st.rows * o_f
    for p in (0, 1):
        hops = []
        for op, name in zip(st.ops[p], st.names):
            h = mlq.LinearOp.from_buffer_copy(op)
            h.x, h.y = hx[name].data_ptr(), hy[name].data_ptr()
            hops.append(h)
        host_batches.append(mlq.Batch(hops))
    ke = max(3, min(steps, 300))
    for _ in range(3):
        st.step_host(host_batches)
    ms = ctx.timed(lambda: [st.step_host(host_batches) for _ in range(ke)])
    bytes_step = st.bytes_step
    h2d = sum(4 * st.rows * next(i for n, _, i in st.wl["matrices"] if n == name) for name in st.names)
    d2h = sum(4 * st.rows * next(o for n, o, _ in st.wl["matrices"] if n == name) for name in st.names)
    return {"value": round(bytes_step * ke / (ms / 1e3) / 1e9, 2), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": ke,
            "path": "mlq_linear_batch_host: the step's ops in one call, pinned host x and y "
                    "(each back to back in one buffer: one copy per direction), one stream "
                    "synchronisation per step"}


def ref_gpu_baseline(ctx, wl, steps):
    """The REFERENCE's own CUDA kernels (q80/q40/q41LinearKernel of
    src/cuda_quant.cu, compiled for sm_100a into oracle/_ref/libref_gpu.so)
    timed on this GPU on the same workload: the same seeded weights
    (quantized on the device) and x, each step one launch per matrix with
    the reference's own grid, CUDA events around the steps.  Also the
    largest relative L2 difference of an output row between the reference's
    kernel and this library on the last matrix (a cross-check on identical
    device inputs)."""
    torch, mlq, pkg = ctx.torch, ctx.mlq, ctx.pkg
    sys.path.insert(0, str(ROOT))
    try:
        from oracle.oracle import ReferenceGpu  # baseline only, never the measured path
        ref = ReferenceGpu()
    except (FileNotFoundError, OSError) as e:
        return {"unavailable": str(e)}
    fmt, rows = wl["fmt"], wl["rows"]
    s = ctx.stream.cuda_stream
    mats = []
    for i, (name, out_f, in_f) in enumerate(wl["matrices"]):
        w32 = pkg.synth.normal_torch((out_f, in_f), seed=1000 + i, std=0.02, device=ctx.device)
        w = mlq.quantize(fmt, w32)
        del w32
        x = torch.from_numpy(pkg.synth.normal((rows, in_f), seed=2000 + i)).to(ctx.device)
        y = torch.empty((rows, out_f), device=ctx.device)
        mats.append((name, out_f, in_f, w, x, y))
    torch.cuda.empty_cache()

    def step():
        for name, out_f, in_f, w, x, y in mats:
            ref.linear(fmt, x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, in_f, out_f, s)

    step()
    k = max(3, min(steps, 10))
    ms = ctx.timed(lambda: [step() for _ in range(k)]) / k
    bytes_step = sum(weight_bytes(fmt, o, i) for _, o, i in wl["matrices"])
    name, out_f, in_f, w, x, y = mats[-1]
    mine = mlq.linear(fmt, w, out_f, in_f, x)
    torch.cuda.synchronize(ctx.device)
    diff = (torch.linalg.norm((mine - y).double(), dim=1) / torch.linalg.norm(y.double(), dim=1).clamp_min(1e-30)).max()
    out = {"value": round(bytes_step / (ms / 1e3) / 1e9, 2), "unit": UNIT, "ms_per_step": round(ms, 4),
           "steps": k, "kernels": f"reference q{fmt[1]}{fmt[3]}LinearKernel, src/cuda_quant.cu (sm_100a build)",
           "max_rel_l2_vs_this_library": float(diff)}
    del mats, mine
    torch.cuda.empty_cache()
    return out


def formats_probe(ctx):
    """Decode (batch 1) weight GB/s of one large matrix per format against
    the measured HBM peak: q8_0 and q4_1 at the Llama-3-8B FFN shape
    14336x4096 (configs 4 and 3), q4_0 at the Qwen2-7B lm_head 152064x3584
    (config 2).  The products cycle through copies of the matrix totalling
    at least 300 MB (more than L2), so every one reads its weights from HBM.
    Two figures: products writing one y (each waits for the one before it:
    launches back to back), and products with a y each (independent: run
    eight at a time in one persistent launch)."""
    torch, mlq, pkg = ctx.torch, ctx.mlq, ctx.pkg
    peak, _ = hbm_peak()
    out = {}
    for fmt, (o, i) in [("q8_0", (14336, 4096)), ("q4_0", (152064, 3584)), ("q4_1", (14336, 4096))]:
        w32 = pkg.synth.normal_torch((o, i), seed=4242, std=0.02, device=ctx.device)
        w = mlq.quantize(fmt, w32)
        del w32
        ncopy = max(1, -(-300 * MB // weight_bytes(fmt, o, i)))
        ws = [w] + [w.clone() for _ in range(ncopy - 1)]
        x = torch.from_numpy(pkg.synth.normal((1, i), seed=4243)).to(ctx.device)
        y = torch.empty((1, o), device=ctx.device)
        n_ops = 20 * ncopy
        b = mlq.Batch([mlq.linear_op(fmt, ws[k % ncopy].data_ptr(), o, i, x.data_ptr(), 1, y.data_ptr())
                       for k in range(n_ops)])
        for _ in range(3):
            b.run(ctx.stream.cuda_stream)
        ms = ctx.timed(lambda: [b.run(ctx.stream.cuda_stream) for _ in range(10)]) / (10 * n_ops)
        gbs = weight_bytes(fmt, o, i) / (ms / 1e3) / 1e9
        # the same products with a y each (8 apart): independent, so the
        # batch runs them eight at a time in one persistent run launch
        ys = [torch.empty((1, o), device=ctx.device) for _ in range(mlq.RUN_MAX_OPS)]
        br = mlq.Batch([mlq.linear_op(fmt, ws[k % ncopy].data_ptr(), o, i, x.data_ptr(), 1,
                                      ys[k % mlq.RUN_MAX_OPS].data_ptr()) for k in range(n_ops)])
        for _ in range(3):
            br.run(ctx.stream.cuda_stream)
        ms_r = ctx.timed(lambda: [br.run(ctx.stream.cuda_stream) for _ in range(10)]) / (10 * n_ops)
        gbs_r = weight_bytes(fmt, o, i) / (ms_r / 1e3) / 1e9
        out[fmt] = {"matrix": [o, i], "copies": ncopy, "launch_ms_back_to_back": round(ms, 5),
                    "GBps": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
                    "run_ms_per_product": round(ms_r, 5), "run_GBps": round(gbs_r, 1),
                    "run_frac_of_measured_hbm": round(gbs_r / peak, 4)}
        del w, ws, x, y, ys, b, br
    torch.cuda.empty_cache()
    return out


def run_mlq(args):
    ctx = Ctx()
    wl = dict(WORKLOADS[args.workload])
    if args.only:
        wl["matrices"] = [m for m in wl["matrices"] if m[0] == args.only]
    head = run_workload(ctx, wl, args.steps, args.warmup, full=True, args=args)
    if ctx.world == 1 and args.workload == "qwen7b" and not args.only:
        roof = head["roofline"]
        if "gemv_run_kernel" in roof["kernel"]:
            roof["traffic"] = read_traffic("gemv_run_q4_0_decode_step.txt")
            roof["single_op_launches"]["traffic"] = read_traffic("gemv_q4_0_lm_head.txt")
        elif "lm_head" in roof["kernel"]:
            roof["traffic"] = read_traffic("gemv_q4_0_lm_head.txt")
    extra, formats = {}, None
    if not args.no_extra and not args.only and args.workload == "qwen7b":
        for name in (EXTRAS_N1 if ctx.world == 1 else EXTRAS_NGT1):
            ew = WORKLOADS[name]
            r = run_workload(ctx, ew, min(args.steps, 10 if name != "llama8b-b16" else 5), 3)
            extra[name] = {"workload": ew["name"], "metric": ew["metric"], "value": r["value"], "unit": UNIT,
                           "ms_per_step": r["ms_per_step"], "steps": r["steps"],
                           "frac_of_measured_hbm": round(r["value"] / hbm_peak()[0], 4),
                           "roofline": r["roofline"], "clocks": r["clocks"],
                           **({"parity_max_rel_l2": r["parity_max_rel_l2"]} if "parity_max_rel_l2" in r else {})}
        if ctx.world == 1:
            formats = formats_probe(ctx)
    cpu = refgpu = None
    if ctx.world == 1 and not args.no_cpu_baseline and not args.only:
        refgpu = ref_gpu_baseline(ctx, wl, args.steps)
        cpu = reference_cpu_baseline(ctx.pkg, wl, args.cpu_seconds)
    parity = [v.get("parity_max_rel_l2") for v in [head, *extra.values()] if "parity_max_rel_l2" in v]
    dev_err = ctx.mlq.device_error(ctx.local)  # any kernel of the whole run that gave up
    if ctx.rank == 0:
        line = {
            "metric": wl["metric"], "value": head["value"], "unit": UNIT, "n_gpus": ctx.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"fp32 activations x {wl['fmt']} weights",
            "data": f"synthetic (seeded N(0,0.02) weights quantized to {wl['fmt']}; N(0,1) x)",
            "config": config_of(wl, ctx.world),
            "roofline": head["roofline"], "cpu_baseline": cpu, "ref_gpu_baseline": refgpu, "e2e": head.get("e2e"),
            "gpu_launches": args.steps * head["gpu_launches_per_step"],
            "clocks": head["clocks"], "device_error": dev_err,
        }
        if "parity_max_rel_l2" in head:
            line["parity_max_rel_l2"] = head["parity_max_rel_l2"]
        if extra:
            line["extra"] = extra
        if formats:
            line["formats"] = formats
        print(json.dumps(line), flush=True)
    ctx.close()
    if dev_err or any(p is None or p > 1e-3 for p in parity):
        raise SystemExit(f"bench: device error {dev_err} or sharded results differ from the one-GPU "
                         f"results (max rel L2 {parity})")


def read_traffic(summary):
    """DRAM bytes per launch from a committed ncu summary under profiles/
    (its traffic_bytes_per_launch line), if any."""
    p = ROOT / "profiles" / summary
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
    wl = WORKLOADS[args.workload]
    fmt = wl["fmt"]
    base = {"impl": "reference", "metric": wl["metric"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"fp32 activations x {fmt} weights",
            "data": f"synthetic (seeded N(0,0.02) weights quantized to {fmt}; N(0,1) x)",
            "config": config_of(wl, world)}
    try:
        rc = ReferenceCPU(wl)
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
    sample = (f"each step: linearQ{fmt[1]}{fmt[3]} over the first {frac:.2%} of every matrix's rows "
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
    ap.add_argument("--no-extra", action="store_true", help="headline workload only")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--only", default=None,
                    help="run one matrix of the workload (qkv/o/gate/up/down/lm_head), for profiling")
    ap.add_argument("--workload", default="qwen7b", choices=sorted(WORKLOADS),
                    help="qwen7b (default, the bench line) or another BASELINE config")
    args = ap.parse_args()
    if args.only and not any(m[0] == args.only for m in WORKLOADS[args.workload]["matrices"]):
        ap.error(f"--only: no matrix named {args.only!r}")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mlq(args)


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark of the DIAL quantized-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload w8a16_gemv|gguf_sweep]

Prints ONE JSON line on rank 0.

Workloads (seeded synthetic inputs with the shapes and distributions of the
benchmark configurations; no dataset is involved):
  w8a16_gemv  W8A16 decode linear: x f16 [1,4096] ~N(0,1), W [12288,4096]
              ~N(0,0.02) quantised per row to int8 with an f16 scale (Qwen3-8B
              MLP up-proj).  Metric: dequant-GEMV HBM GB/s.
  gguf_sweep  GGUF QMatMul over the 7 linears of an 8B decoder layer (q, k, v,
              o, gate, up, down) for Q4_0 and Q8_0 at M in {1, 8}, f32
              activations.  Metric: dequant-GEMV HBM GB/s over the sweep.
A step is one pass of the workload.  Inputs: rotating copies of the weights
whose total exceeds the 126 MB L2, so every step reads its weights from HBM.

Multi-GPU: a single linear does not shard (replicas only): under torchrun
every rank runs the same workload on its own GPU, the timed region is the max
over ranks, and `value` is the sum of all ranks' bytes over that time.

--impl reference times the CPU restatement of the reference's path (the C
oracle, OpenMP over all host threads) on the same workload and prints the
same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "dial-8b-orin_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED = 299792458
L2_BYTES = 126 * 2**20
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

LAYER_SHAPES = [  # (name, out N, in K) of one 8B decoder layer (Qwen3-8B / config 2)
    ("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
    ("gate", 12288, 4096), ("up", 12288, 4096), ("down", 4096, 12288),
]


def peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", FALLBACK_BF16_TFLOPS)), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ distributed
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, local, world


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ workloads
class W8A16Gemv:
    name = "w8a16_gemv"
    desc = "W8A16 decode GEMV x f16 [1,4096] . W int8 [12288,4096]^T (f16 row scale)"

    def __init__(self, torch, D):
        self.torch, self.D = torch, D
        self.M, self.N, self.K = 1, 12288, 4096
        g = torch.Generator(device="cuda").manual_seed(SEED)
        per = self.N * self.K + 2 * self.N
        self.copies = max(2, -(-3 * L2_BYTES // per))  # rotate past the L2
        self.lins = []
        for _ in range(self.copies):
            w = torch.randn((self.N, self.K), generator=g, device="cuda", dtype=torch.float32) * 0.02
            self.lins.append(D.W8A16Linear.from_linear("up", w, scale_dtype=torch.float16))
            del w
        self.x = (torch.randn((self.M, self.K), generator=g, device="cuda")).half()
        self.y = torch.empty((self.M, self.N), dtype=torch.float16, device="cuda")
        self.i = 0
        self.bytes_per_step = self.N * self.K + 2 * self.N + 2 * self.M * self.K + 2 * self.M * self.N
        self.flops_per_step = 2 * self.M * self.N * self.K
        self.kernel_bytes = self.bytes_per_step  # one launch per step
        self.launches_per_step = 1
        self.h_x = torch.empty_like(self.x, device="cpu").pin_memory()
        self.h_x.copy_(self.x.cpu())
        self.h_y = torch.empty_like(self.y, device="cpu").pin_memory()
        self.config = {"workload": self.name, "M": 1, "N": self.N, "K": self.K,
                       "weight": "int8 per-row, f16 scale", "activation": "f16",
                       "l2": f"{self.copies} rotating weight copies "
                             f"({self.copies * per / 1e6:.0f} MB > 126 MB L2)"}

    def step(self):
        lin = self.lins[self.i % self.copies]
        self.i += 1
        lin.forward(self.x, out=self.y)

    def step_e2e(self):
        self.x.copy_(self.h_x, non_blocking=True)
        self.step()
        self.h_y.copy_(self.y, non_blocking=True)
        return self.h_x.numel() * 2, self.h_y.numel() * 2

    # CPU baseline: the oracle on the same shape
    def cpu_setup(self, np, O):
        rng = np.random.default_rng(SEED)
        w = rng.normal(0, 0.02, (self.N, self.K)).astype(np.float32)
        self.c_q, self.c_s32, _ = O.w8a16_quantize(w)
        self.c_x = rng.normal(0, 1, (1, self.K)).astype(np.float16)

    def cpu_step(self, O):
        O.w8a16_linear_f32(self.c_x, self.c_q, self.c_s32)


class GgufSweep:
    name = "gguf_sweep"
    desc = "GGUF QMatMul over the 7 linears of an 8B layer, Q4_0 and Q8_0, M in {1, 8}, f32 x"

    def __init__(self, torch, D, ms=(1, 8)):
        self.torch, self.D, self.ms = torch, D, tuple(ms)
        g = torch.Generator(device="cuda").manual_seed(SEED)
        layer = []
        per_layer = 0
        for qt in (D.Q4_0, D.Q8_0):
            for name, N, K in LAYER_SHAPES:
                w = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float32) * 0.02
                lin = D.GgufLinear.quantize(w, qt, name)
                del w
                layer.append(lin)
                per_layer += lin.weight_bytes
        self.copies = max(2, -(-3 * L2_BYTES // per_layer))
        self.layers = [layer]
        for _ in range(self.copies - 1):
            cp = []
            for lin in layer:
                cp.append(D.GgufLinear(lin.qs.clone(), lin.d.clone(), lin.qtype, lin.in_dim,
                                       lin.out_dim, lin.name))
            self.layers.append(cp)
        maxk = max(k for _, _, k in LAYER_SHAPES)
        maxn = max(n for _, n, _ in LAYER_SHAPES)
        self.xs = {m: torch.randn((m, maxk), generator=g, device="cuda") for m in self.ms}
        self.ys = {m: torch.empty((m, maxn), device="cuda") for m in self.ms}
        self.i = 0
        b = 0
        for m in self.ms:
            for lin in layer:
                b += lin.weight_bytes + 4 * m * lin.in_dim + 4 * m * lin.out_dim
        self.bytes_per_step = b
        self.kernel_bytes = None
        self.launches_per_step = 2 * len(layer) * len(self.ms)
        self.flops_per_step = sum(2 * m * lin.in_dim * lin.out_dim for m in self.ms for lin in layer)
        self.config = {"workload": self.name, "M": list(self.ms), "types": ["Q4_0", "Q8_0"],
                       "shapes": [f"{n}:{k}->{N}" for n, N, k in LAYER_SHAPES], "activation": "f32",
                       "l2": f"{self.copies} rotating layer copies "
                             f"({self.copies * per_layer / 1e6:.0f} MB > 126 MB L2)"}

    def step(self):
        layer = self.layers[self.i % self.copies]
        self.i += 1
        for m in self.ms:
            for lin in layer:
                x = self.xs[m][:, : lin.in_dim]
                if not x.is_contiguous():
                    x = x.contiguous()
                lin.forward(x, out=self.ys[m][:, : lin.out_dim].contiguous())

    def step_e2e(self):
        raise NotImplementedError

    def cpu_setup(self, np, O):
        rng = np.random.default_rng(SEED)
        self.c = []
        for qt in (O.Q4_0, O.Q8_0):
            for _, N, K in LAYER_SHAPES:
                w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
                self.c.append((O.gguf_quantize(w, qt), qt, N, K))
        self.c_x = {m: rng.normal(0, 1, (m, 12288)).astype(np.float32) for m in self.ms}

    def cpu_step(self, O):
        for m in self.ms:
            for blocks, qt, N, K in self.c:
                O.gguf_linear_candle(self.c_x[m][:, :K], blocks, qt, N)


WORKLOADS = {"w8a16_gemv": W8A16Gemv, "gguf_sweep": GgufSweep}


# ------------------------------------------------------------------ CPU legs
def cpu_measure(wl_cls, budget_s: float):
    import numpy as np

    import oracle as O
    wl = wl_cls.__new__(wl_cls)
    wl_cls_init_cpu(wl)
    wl.cpu_setup(np, O)
    wl.cpu_step(O)  # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        wl.cpu_step(O)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    return dt, n, O.num_threads()


def wl_cls_init_cpu(wl):
    if isinstance(wl, W8A16Gemv):
        wl.M, wl.N, wl.K = 1, 12288, 4096
        wl.bytes_per_step = wl.N * wl.K + 2 * wl.N + 2 * wl.M * wl.K + 2 * wl.M * wl.N
    elif isinstance(wl, GgufSweep):
        wl.ms = (1, 8)
        b = 0
        for m in wl.ms:
            for qt_bytes in (18, 34):
                for _, N, K in LAYER_SHAPES:
                    b += N * K // 32 * qt_bytes + 4 * m * K + 4 * m * N
        wl.bytes_per_step = b


def run_reference(args, rank, world):
    if rank != 0:
        return
    wl_cls = WORKLOADS[args.workload]
    dts = []
    n_total = 0
    for _ in range(args.warmup):
        cpu_measure(wl_cls, 0.0)
    per_step_budget = max(1.0, min(20.0, 60.0 / max(args.steps, 1)))
    threads = 1
    for _ in range(args.steps):
        dt, n, threads = cpu_measure(wl_cls, per_step_budget)
        dts.append(dt)
        n_total += n
    wl = wl_cls.__new__(wl_cls)
    wl_cls_init_cpu(wl)
    dt = statistics.median(dts)
    value = wl.bytes_per_step / dt / 1e9
    line = {
        "impl": "reference", "metric": "dequant-GEMV HBM GB/s", "value": round(value, 3),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xf16" if args.workload == "w8a16_gemv" else "q4_0/q8_0 x f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": args.workload},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{n_total} calls of the oracle over {args.steps} steps of "
                                   f"~{per_step_budget:.0f}s"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU leg
def run_ours(args, rank, local, world):
    import torch

    import dial_cuda as D
    torch.cuda.set_device(local)
    wl = WORKLOADS[args.workload](torch, D)
    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()

    # ---- device-timed region: K steps, events around every step on the launching stream
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    launches0 = D.launch_count()
    with ClockSampler(local) as clocks:
        t_begin.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            wl.step()
            ends[i].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    launches = D.launch_count() - launches0
    total_ms = max_over_ranks(t_begin.elapsed_time(t_end), world)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]

    # ---- end-to-end: host buffers, H2D + call + D2H inside the timed region
    e2e = None
    if hasattr(wl, "h_x"):
        for _ in range(3):
            wl.step_e2e()
        torch.cuda.synchronize()
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d = d2h = 0
        for _ in range(args.steps):
            h2d, d2h = wl.step_e2e()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
        e2e = {"value": round(wl.bytes_per_step * world * args.steps / (e2e_ms / 1e3) / 1e9, 3),
               "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(e2e_ms / args.steps, 5)}

    hbm_peak, tf_peak, peak_src = peaks()
    value = wl.bytes_per_step * world * args.steps / (total_ms / 1e3) / 1e9
    avg_step_ms = statistics.mean(step_ms)
    kernel_bytes = wl.kernel_bytes if wl.kernel_bytes else wl.bytes_per_step / wl.launches_per_step
    kernel_ms = avg_step_ms / (1 if wl.kernel_bytes else wl.launches_per_step)
    achieved = kernel_bytes / (kernel_ms / 1e3) / 1e9
    line = {
        "metric": "dequant-GEMV HBM GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xf16" if args.workload == "w8a16_gemv" else "q4_0/q8_0 x f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": dict(wl.config, parallelism=f"replicas x{world}"),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "traffic": None,
                     "peak_source": peak_src, "kernel": "w8a16_skinny_kernel<1>"
                     if args.workload == "w8a16_gemv" else "gguf_skinny_kernel (mean per linear)"},
        "e2e": e2e, "gpu_launches": launches, "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, n, threads = cpu_measure(WORKLOADS[args.workload], args.cpu_budget)
        line["cpu_baseline"] = {"value": round(wl.bytes_per_step / dt / 1e9, 3), "unit": "GB/s",
                                "cores": threads, "kind": "port",
                                "sample": f"{n} calls of the C oracle in ~{args.cpu_budget:.0f}s"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="w8a16_gemv")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank, local, world = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, local, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark of the DIAL quantized-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Prints ONE JSON line on rank 0.

Workloads (seeded synthetic inputs with the shapes and distributions of the
benchmark configurations; no dataset is involved):
  w8a16_gemv    W8A16 decode linear: x f16 [1,4096] ~N(0,1), W [12288,4096]
                ~N(0,0.02) quantised per row to int8 with an f16 scale
                (Qwen3-8B MLP up-proj).  Metric: dequant-GEMV HBM GB/s.
  gguf_sweep    GGUF QMatMul over the 7 linears of an 8B decoder layer (q, k,
                v, o, gate, up, down) for Q4_0 and Q8_0 at M in {1, 8}, f32
                activations.  Metric: dequant-GEMV HBM GB/s over the sweep.
  gguf_sweep_m32  The same sweep at M = 32 (between decode and prefill; still
                HBM-bound).  Metric: HBM GB/s over the sweep.
  gguf_prefill  The same sweep at M = 512 (the prefill point of the GGUF
                sweep).  Metric: dequant-GEMM TFLOP/s (tensor roofline).
  w8a16_prefill The 4 fused linears of a Qwen3-8B layer (QKV 6144x4096, O
                4096x4096, gate_up 24576x4096, down 4096x12288) at M = 512
                (a 512-token prompt), f16.  Metric: dequant-GEMM TFLOP/s.
  gguf_k_prefill  The same layer's 7 linears in Q4_K and Q6_K at M = 512 (a
                prompt), f16.  Metric: dequant-GEMM TFLOP/s.
  gguf_k_sweep  The 7 linears of a Llama-3-8B layer in Q4_K and Q6_K (the
                types of a Q4_K_M file) at M = 1, f16 activations.  Metric:
                dequant-GEMV HBM GB/s over the sweep.
  qwen3_decode / qwen3_decode_bf16 / qwen3_generate / llama_gguf_decode /
  attention_batched: whole-model decode (the default, qwen3_decode: f16, the
                reference's W8A16 dtype) and the batched decode attention;
                their docstrings give the shapes.  --split even|planner picks
                the layer split of the pipeline workloads; --head vocab
                splits their output head over the stages by vocabulary rows
                (each stage a share that evens out the stages' weight bytes)
                instead of running it on the last stage.
A step is one pass of the workload.  Multi-linear steps are captured once in
a CUDA graph and replayed.  Inputs: rotating copies of the weights whose total
exceeds the 126 MB L2, so every step reads its weights from HBM.

Multi-GPU: a single linear does not shard (replicas only): under torchrun
every rank runs the same workload on its own GPU, the timed region is the max
over ranks, and `value` is the sum of all ranks' work over that time.

--impl reference times the CPU restatement of the reference's path (the C
oracle, OpenMP over all host threads) on the same workload and prints the
same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "dial-8b-orin_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SEED = 299792458
DATA = "synthetic (seeded N(0,0.02) weights, N(0,1) activations)"
L2_BYTES = 126 * 2**20
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

LAYER_SHAPES = [  # (name, out N, in K) of one 8B decoder layer (Qwen3-8B shapes)
    ("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
    ("gate", 12288, 4096), ("up", 12288, 4096), ("down", 4096, 12288),
]
GGUF_BLOCK_BYTES = {"Q4_0": 18, "Q8_0": 34}


def peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in FALLBACK}, "measured"
    except Exception:
        return dict(FALLBACK), "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and throttle reasons, sampled with NVML every ~2 ms in a thread."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch, device_index: int):
        self.samples = []
        self.stop = threading.Event()
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            props = torch.cuda.get_device_properties(device_index)
            bus = getattr(props, "pci_bus_id", None)
            if bus is not None:
                dom = getattr(props, "pci_domain_id", 0)
                dev = getattr(props, "pci_device_id", 0)
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0")
            else:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.handle is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.handle is not None:
            self.thread.join(timeout=2)

    def summary(self, t0=None, t1=None):
        sel = [s for s in self.samples if t0 is None or (t0 <= s[0] <= t1)]
        window = "timed region"
        if not sel:
            sel, window = self.samples, "warm-up + timed region"
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, _, rs in sel:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in sel), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sel), "window": window}


# ------------------------------------------------------------------ distributed
def dist_setup():
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


def sum_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ workloads (GPU)
def build_copy_graphs(wl):
    """One CUDA graph per weight copy, captured on a side stream that was warmed
    first (kernel attributes, the tensor-map entry point, that stream's linear
    workspace), so the graphs hold the kernels only."""
    torch = wl.torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for li in range(wl.copies):
            wl.run_copy(li)
    torch.cuda.synchronize()
    wl.graphs = []
    for li in range(wl.copies):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            wl.run_copy(li)
        wl.graphs.append(gr)
    torch.cuda.synchronize()


class W8A16Gemv:
    """One W8A16 decode linear per step (the Qwen3-8B up-proj shape)."""
    metric, unit, bound, dtype = "dequant-GEMV HBM GB/s", "GB/s", "hbm", "int8 x f16"
    kernel = "w8a16_gemv_kernel<NT=1>"
    M, N, K = 1, 12288, 4096
    graph = True
    # DRAM read + write bytes of one w8a16_gemv_kernel launch of this shape, from
    # an ncu capture of this workload
    traffic = 50_430_464 + 256

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        self.torch = torch
        g = torch.Generator(device="cuda").manual_seed(SEED)
        per = self.N * self.K + 2 * self.N
        self.copies = max(2, -(-3 * L2_BYTES // per))  # rotate past the L2
        self.lins = []
        for _ in range(self.copies):
            w = torch.randn((self.N, self.K), generator=g, device="cuda", dtype=torch.float32) * 0.02
            self.lins.append(D.W8A16Linear.from_linear("up", w, scale_dtype=torch.float16))
            del w
        self.x = torch.randn((self.M, self.K), generator=g, device="cuda").half()
        self.y = torch.empty((self.M, self.N), dtype=torch.float16, device="cuda")
        self.i = 0
        self.work_per_step = self.bytes()  # GB/s metric: bytes
        self.kernel_work = self.work_per_step
        self.h_x = self.x.cpu().pin_memory()
        self.h_y = torch.empty(self.y.shape, dtype=self.y.dtype).pin_memory()
        self.config = self.describe()

    @classmethod
    def describe(cls, world: int = 1):
        per = cls.N * cls.K + 2 * cls.N
        copies = max(2, -(-3 * L2_BYTES // per))
        return {"workload": "w8a16_gemv", "M": 1, "N": cls.N, "K": cls.K,
                "weight": "int8 per-row, f16 scale", "activation": "f16",
                "l2": f"{copies} rotating weight copies ({copies * per / 1e6:.0f} MB > 126 MB L2)",
                "launch": f"CUDA graph of {cls.chain} consecutive GEMVs (PDL between them)"}

    @classmethod
    def bytes(cls):
        return cls.N * cls.K + 2 * cls.N + 2 * cls.M * cls.K + 2 * cls.M * cls.N

    chain = 16  # GEMVs per chained graph (steps per replay)

    def run_copy(self, li):
        self.lins[li].forward(self.x, out=self.y)

    def build_graphs(self):
        """Per-copy graphs, plus one graph of `chain` consecutive GEMVs cycling
        through the copies, so that a Python-side replay per 25 us GEMV does not
        starve the GPU: a step is still one GEMV over a weight copy not in L2."""
        build_copy_graphs(self)
        torch = self.torch
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.run_copy(0)  # the stream's linear workspace
        torch.cuda.synchronize()
        self.chain_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.chain_graph, stream=side):
            for k in range(self.chain):
                self.run_copy(k % self.copies)
        torch.cuda.synchronize()

    def step(self):
        self.graphs[self.i % self.copies].replay()
        self.i += 1

    def run_steps(self, n):
        """n steps: whole chains, then single GEMVs for the remainder."""
        for _ in range(n // self.chain):
            self.chain_graph.replay()
        for _ in range(n % self.chain):
            self.step()

    def step_e2e(self):
        """Through the public API with host buffers: H2D x, linear, D2H y."""
        self.x.copy_(self.h_x, non_blocking=True)
        self.lins[self.i % self.copies].forward(self.x, out=self.y)
        self.i += 1
        self.h_y.copy_(self.y, non_blocking=True)
        return self.h_x.numel() * 2, self.h_y.numel() * 2


class GgufSweep:
    """GGUF decode sweep: 7 shapes x {Q4_0, Q8_0} x M in {1, 8}."""
    metric, unit, bound, dtype = "dequant-GEMV HBM GB/s", "GB/s", "hbm", "q4_0/q8_0 x f32"
    kernel = "gguf_gemv_kernel (whole tiles; Q8_0 staging fused at M = 1) (whole sweep)"
    ms = (1, 8)
    graph = True

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        self.torch, self.D = torch, D
        g = torch.Generator(device="cuda").manual_seed(SEED)
        layer, per_layer = [], 0
        for qt in (D.Q4_0, D.Q8_0):
            for name, N, K in LAYER_SHAPES:
                w = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float32) * 0.02
                lin = D.GgufLinear.quantize(w, qt, name)
                del w
                layer.append(lin)
                per_layer += lin.weight_bytes
        self.copies = max(2, -(-3 * L2_BYTES // per_layer))
        self.layers = [layer] + [[D.GgufLinear(l.qs.clone(), l.d.clone(), l.qtype, l.in_dim,
                                               l.out_dim, l.name) for l in layer]
                                 for _ in range(self.copies - 1)]
        self.calls = []
        for li, lay in enumerate(self.layers):
            for m in self.ms:
                for lin in lay:
                    x = torch.randn((m, lin.in_dim), generator=g, device="cuda")
                    y = torch.empty((m, lin.out_dim), device="cuda")
                    lin.workspace(m)
                    self.calls.append((li, lin, x, y))
        self.i = 0
        self.work_per_step = self.bytes()
        self.kernel_work = None
        self.config = self.describe()

    name = "gguf_sweep"

    @classmethod
    def describe(cls, world: int = 1):
        per_layer = sum(N * (K // 32) * bb for bb in GGUF_BLOCK_BYTES.values() for _, N, K in LAYER_SHAPES)
        copies = max(2, -(-3 * L2_BYTES // per_layer))
        return {"workload": cls.name, "M": list(cls.ms), "types": ["Q4_0", "Q8_0"],
                "shapes": [f"{n}:{k}->{N}" for n, N, k in LAYER_SHAPES], "activation": "f32",
                "l2": f"{copies} rotating layer copies ({copies * per_layer / 1e6:.0f} MB > 126 MB L2)",
                "launch": "CUDA graph per layer copy"}

    @classmethod
    def bytes(cls):
        b = 0
        for m in cls.ms:
            for bb in GGUF_BLOCK_BYTES.values():
                for _, N, K in LAYER_SHAPES:
                    b += N * (K // 32) * bb + 4 * m * K + 4 * m * N
        return b

    def run_copy(self, li):
        for lj, lin, x, y in self.calls:
            if lj == li:
                lin.forward(x, out=y)

    def build_graphs(self):
        build_copy_graphs(self)

    def step(self):
        self.graphs[self.i % self.copies].replay()
        self.i += 1


LLAMA_SHAPES = [  # (name, out N, in K) of one Llama-3-8B decoder layer
    ("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
    ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336),
]
K_BLOCK_BYTES = {"Q4_K": 144, "Q6_K": 210}


class GgufKSweep:
    """GGUF K-quant decode sweep: the 7 linears of a Llama-3-8B layer in Q4_K and
    in Q6_K (the two types of a Q4_K_M file) at M = 1, f16 activations, the
    file's native super-blocks read by the decode linear."""
    metric, unit, bound, dtype = "dequant-GEMV HBM GB/s", "GB/s", "hbm", "q4_k/q6_k x f16"
    kernel = "kq4_gemv_kernel + kq6_gemv_kernel (whole sweep)"
    data = "synthetic (seeded random Q4_K/Q6_K super-blocks with N(0,1e-4) f16 scales, N(0,1) activations)"
    ms = (1,)
    types = ("Q4_K", "Q6_K")
    name = "gguf_k_sweep"
    graph = True

    @staticmethod
    def random_blocks(rng, qt: int, N: int, K: int, scale: float = 1e-4):
        """Seeded K-quant super-blocks [N, K/256*bytes]: random quant, scale and
        min bytes with finite f16 super-block scales ~ N(0, scale)."""
        import numpy as np
        nb, bb = K // 256, (144 if qt == 12 else 210)
        raw = rng.integers(0, 256, (N, nb, bb), dtype=np.uint8)
        d = rng.normal(0.0, scale, (N, nb)).astype(np.float16)
        if qt == 12:  # Q4_K: f16 d, f16 dmin at bytes 0..3
            raw[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
            dmin = np.abs(rng.normal(0.0, scale, (N, nb))).astype(np.float16)
            raw[:, :, 2:4] = dmin.view(np.uint8).reshape(N, nb, 2)
        else:  # Q6_K: f16 d at bytes 208..209
            raw[:, :, 208:210] = d.view(np.uint8).reshape(N, nb, 2)
        return raw.reshape(N, nb * bb)

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        import numpy as np
        self.torch, self.D = torch, D
        rng = np.random.default_rng(SEED)
        layer, per_layer = [], 0
        for qt in [{"Q4_K": D.Q4_K, "Q6_K": D.Q6_K}[t] for t in self.types]:
            for name, N, K in LLAMA_SHAPES:
                b = torch.from_numpy(self.random_blocks(rng, qt, N, K).reshape(-1)).cuda()
                lin = D.GgufKLinear.from_blocks(b, qt, K, N, name)
                layer.append(lin)
                per_layer += lin.weight_bytes
        self.copies = max(2, -(-3 * L2_BYTES // per_layer))
        self.layers = [layer] + [[D.GgufKLinear(l.blocks.clone(), l.qtype, l.in_dim, l.out_dim, l.name)
                                  for l in layer] for _ in range(self.copies - 1)]
        g = torch.Generator(device="cuda").manual_seed(SEED)
        self.calls = []
        for li, lay in enumerate(self.layers):
            for m in self.ms:
                for lin in lay:
                    x = torch.randn((m, lin.in_dim), generator=g, device="cuda").half()
                    y = torch.empty((m, lin.out_dim), device="cuda", dtype=torch.float16)
                    self.calls.append((li, lin, x, y))
        self.i = 0
        self.work_per_step = self.bytes()
        self.kernel_work = None
        self.config = self.describe()

    @classmethod
    def describe(cls, world: int = 1):
        per_layer = sum(N * (K // 256) * K_BLOCK_BYTES[t] for t in cls.types for _, N, K in LLAMA_SHAPES)
        copies = max(2, -(-3 * L2_BYTES // per_layer))
        return {"workload": cls.name, "M": list(cls.ms), "types": list(cls.types),
                "shapes": [f"{n}:{k}->{N}" for n, N, k in LLAMA_SHAPES], "activation": "f16",
                "weights": "seeded random super-blocks (finite f16 scales)",
                "l2": f"{copies} rotating layer copies ({copies * per_layer / 1e6:.0f} MB > 126 MB L2)",
                "launch": "CUDA graph per layer copy"}

    @classmethod
    def bytes(cls):
        b = 0
        for m in cls.ms:
            for t in cls.types:
                for _, N, K in LLAMA_SHAPES:
                    b += N * (K // 256) * K_BLOCK_BYTES[t] + 2 * m * K + 2 * m * N
        return b

    def run_copy(self, li):
        for lj, lin, x, y in self.calls:
            if lj == li:
                lin.forward(x, out=y)

    def build_graphs(self):
        build_copy_graphs(self)

    def step(self):
        self.graphs[self.i % self.copies].replay()
        self.i += 1


class GgufKPrefill(GgufKSweep):
    """K-quant prefill: the 7 linears of a Llama-3-8B layer as the file's Q4_K
    and Q6_K super-blocks at M = 512 (a 512-token prompt), f16: the tcgen05
    GEMM dequantises each super-block once per token tile."""
    metric, unit, bound, dtype = "dequant-GEMM TFLOP/s", "TFLOP/s", "tensor", "q4_k/q6_k x f16 -> f16 MMA"
    kernel = "dequant_gemm_kernel<Q4_K, Q6_K> (whole sweep)"
    ms = (512,)
    types = ("Q4_K", "Q6_K")
    name = "gguf_k_prefill"

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        super().__init__(torch, D)
        self.work_per_step = self.flops()

    @classmethod
    def flops(cls):
        return sum(2 * m * N * K for m in cls.ms for _ in cls.types for _, N, K in LLAMA_SHAPES)


class GgufSweepM32(GgufSweep):
    """GGUF sweep at M = 32 (the batched-decode row count of the Llama GGUF
    decoder; Q4_0 at 32 rows is still HBM-bound: ~104 flop per byte)."""
    kernel = "dequant_gemm_kernel, 32-token tiles (whole sweep)"
    ms = (32,)
    name = "gguf_sweep_m32"


class GgufPrefill(GgufSweep):
    """GGUF prefill sweep: the same sweep at M = 512 (tensor-bound)."""
    metric, unit, bound, dtype = "dequant-GEMM TFLOP/s", "TFLOP/s", "tensor", "q4_0/q8_0 x f32 -> f16 MMA"
    kernel = "dequant_gemm_kernel (whole sweep)"
    ms = (512,)
    name = "gguf_prefill"

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        super().__init__(torch, D)
        self.work_per_step = self.flops()

    @classmethod
    def flops(cls):
        return sum(2 * m * N * K for m in cls.ms for _ in GGUF_BLOCK_BYTES for _, N, K in LAYER_SHAPES)


QWEN_LAYER_LINEARS = [  # (name, out N, in K): the fused linears of one Qwen3-8B layer
    ("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 24576, 4096), ("down", 4096, 12288),
]


class W8A16Prefill:
    """W8A16 prefill: the 4 fused linears of a Qwen3-8B layer at M = 512 (a
    512-token prompt), f16 activations, f32 row scales, through
    dial_w8a16_linear (the tcgen05 dequant GEMM).  Metric: TFLOP/s."""
    metric, unit, bound, dtype = "dequant-GEMM TFLOP/s", "TFLOP/s", "tensor", "int8 x f16 -> f16 MMA"
    kernel = "dequant_gemm_kernel (the layer's 4 linears)"
    M = 512
    graph = True

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        self.torch, self.D = torch, D
        g = torch.Generator(device="cuda").manual_seed(SEED)
        layer = []
        for name, N, K in QWEN_LAYER_LINEARS:
            w = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float32) * 0.02
            layer.append(D.W8A16Linear.from_linear(name, w))
            del w
        per_layer = sum(l.weight_bytes for l in layer)
        self.copies = max(2, -(-3 * L2_BYTES // per_layer))
        self.layers = [layer] + [[D.W8A16Linear(l.qweight.clone(), l.scales.clone(), l.in_dim, l.out_dim,
                                                l.name) for l in layer] for _ in range(self.copies - 1)]
        self.xs = {K: torch.randn((self.M, K), generator=g, device="cuda").half()
                   for _, _, K in QWEN_LAYER_LINEARS}
        self.ys = [torch.empty((self.M, N), device="cuda", dtype=torch.float16)
                   for _, N, _ in QWEN_LAYER_LINEARS]
        self.i = 0
        self.work_per_step = self.flops()
        self.config = self.describe()

    @classmethod
    def describe(cls, world: int = 1):
        per_layer = sum(N * K + 4 * N for _, N, K in QWEN_LAYER_LINEARS)
        copies = max(2, -(-3 * L2_BYTES // per_layer))
        return {"workload": "w8a16_prefill", "M": cls.M,
                "shapes": [f"{n}:{k}->{N}" for n, N, k in QWEN_LAYER_LINEARS], "activation": "f16",
                "weight": "int8 per-row, f32 scale",
                "l2": f"{copies} rotating layer copies ({copies * per_layer / 1e6:.0f} MB > 126 MB L2)",
                "launch": "CUDA graph per layer copy"}

    @classmethod
    def flops(cls):
        return sum(2 * cls.M * N * K for _, N, K in QWEN_LAYER_LINEARS)

    def run_copy(self, li):
        for lin, y in zip(self.layers[li], self.ys):
            lin.forward(self.xs[lin.in_dim], out=y)

    def build_graphs(self):
        build_copy_graphs(self)

    def step(self):
        self.graphs[self.i % self.copies].replay()
        self.i += 1


class AttentionDecode:
    """Batched decode attention of one layer: 32 sequences, each one query token
    over its 2049-row f16 KV cache (Llama-3-8B heads: 32 query / 8 KV, head_dim
    128), through dial_attention.  Metric: KV bytes read per second."""
    metric, unit, bound, dtype = "decode attention KV GB/s", "GB/s", "hbm", "f16"
    kernel = "attention_tc_kernel<f16, 4> + attention_combine_kernel"
    T, HQ, HKV, D, CTX = 32, 32, 8, 128, 2049
    graph = True
    traffic = None

    def __init__(self, torch, D_, rank: int = 0, world: int = 1):
        self.torch, self.Dl = torch, D_
        g = torch.Generator(device="cuda").manual_seed(SEED)
        self.S = self.CTX + 15  # cache rows per slot
        per = 2 * self.T * self.HKV * self.S * self.D * 2
        self.copies = max(2, -(-3 * L2_BYTES // per))  # layer caches rotated past the L2
        self.kc, self.vc = [], []
        for _ in range(self.copies):
            self.kc.append(torch.randn((self.T, self.HKV, self.S, self.D), generator=g, device="cuda",
                                       dtype=torch.float16))
            self.vc.append(torch.randn((self.T, self.HKV, self.S, self.D), generator=g, device="cuda",
                                       dtype=torch.float16))
        self.q = torch.randn((self.T, self.HQ, self.D), generator=g, device="cuda", dtype=torch.float16)
        self.out = torch.empty((self.T, self.HQ * self.D), device="cuda", dtype=torch.float16)
        self.pos = torch.full((self.T,), self.CTX - 1, dtype=torch.int32, device="cuda")
        self.slot = torch.arange(self.T, dtype=torch.int32, device="cuda")
        need = D_.lib().dial_attention_workspace_bytes(self.T, self.HQ, self.CTX)
        self.ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
        self.need = need
        self.i = 0
        self.work_per_step = self.bytes()
        self.config = self.describe()

    @classmethod
    def describe(cls, world: int = 1):
        per = 2 * cls.T * cls.HKV * (cls.CTX + 15) * cls.D * 2
        copies = max(2, -(-3 * L2_BYTES // per))
        return {"workload": "attention_batched", "sequences": cls.T, "context": cls.CTX,
                "heads": f"{cls.HQ}/{cls.HKV}", "head_dim": cls.D, "kv_cache": "f16",
                "l2": f"{copies} rotating layer caches ({copies * per / 1e6:.0f} MB > 126 MB L2)"}

    @classmethod
    def bytes(cls):
        return 2 * cls.T * cls.HKV * cls.CTX * cls.D * 2 + 2 * 2 * cls.T * cls.HQ * cls.D

    def run_copy(self, li):
        L = self.Dl.lib()
        self.Dl.check(L.dial_attention(self.q.data_ptr(), self.kc[li].data_ptr(), self.vc[li].data_ptr(),
                                       self.pos.data_ptr(), self.slot.data_ptr(), self.out.data_ptr(),
                                       self.ws.data_ptr() if self.need else None, self.need,
                                       self.Dl.F16, self.T, self.HQ, self.HKV, self.D, self.S, self.CTX,
                                       self.Dl.stream_ptr()), "dial_attention")

    def build_graphs(self):
        build_copy_graphs(self)

    def step(self):
        self.graphs[self.i % self.copies].replay()
        self.i += 1


class QwenDecode:
    """Qwen3-8B-shaped W8A16 decoder (36 layers, hidden 4096,
    MLP 12288, 32/8 heads, vocab 151936, random init N(0, 0.02)), 8 sequences,
    1024-token prompts (prefilled before timing), decoded as micro-batches of 1
    through a pipeline of one stage per rank (layers split by the stage
    planner, the output head counted as 3.2 layers).  A step advances every
    sequence by one greedy token.  Metric: decode tok/s of the whole job."""
    metric, unit, bound, dtype = "8B W8A16 decode tok/s", "tok/s", "hbm", "int8 x f16"
    kernel = "w8a16_gemv_kernel<NT=1> (the stage's linears from one graph, events)"
    graph = True
    scaling = "strong"
    # DRAM bytes per token of the stage's linears on one GPU: the DRAM read + write
    # bytes of one captured 12288 x 4096 w8a16_gemv_kernel launch (50,430,720 B
    # over its 24,576 weight units of 2 KB) times the token's 3,695,360 units
    traffic = 7_582_994_200
    n_seqs, mb_size, prompt_len, decode_cap = 8, 1, 1024, 448
    head_layers = 3.2  # the output head's cost in layers (weights read per token)
    copies_per_step = 8  # one graph per micro-batch
    act = "f16"
    split = "planner"  # layer split over the stages: "planner" or "even"
    head = "last"  # output head: on the last stage, or "vocab" (vocabulary-parallel)
    name = "qwen3_decode"

    @classmethod
    def model_config(cls):
        from dial_cuda.model import ModelConfig
        return ModelConfig(act_dtype=cls.act)

    @classmethod
    def micro_batch(cls, world):
        return cls.mb_size

    @classmethod
    def vocab_head(cls, world):
        return cls.head == "vocab" and world > 1

    @classmethod
    def ranges_for(cls, world):
        from dial_cuda.pipeline import stage_layers
        # a vocabulary-parallel head is spread over the stages after the split
        hl = 0.0 if cls.vocab_head(world) else cls.head_layers
        return stage_layers(cls.model_config().n_layers, world, head_layers=hl, method=cls.split)

    @classmethod
    def head_spans(cls, world):
        """Vocabulary rows per stage: shares that bring every stage's weight up
        to the mean (layers + the head's cost in layers) / stages."""
        from dial_cuda.model import vocab_shards
        n = [len(r) for r in cls.ranges_for(world)]
        target = (sum(n) + cls.head_layers) / world
        return vocab_shards(cls.model_config().vocab, [max(0.0, target - k) for k in n])

    @classmethod
    def model_desc(cls):
        return {"workload": "qwen3_8b_w8a16_decode", "model": "Qwen3-8B-shaped, random init",
                "layers": 36, "hidden": 4096, "intermediate": 12288, "heads": "32/8",
                "vocab": 151936, "weights": "int8 per row, f32 scale (layers and head)",
                "l2": "7.6 GB of weights per token >> 126 MB L2"}

    @classmethod
    def describe(cls, world: int = 1):
        return dict(cls.model_desc(), sequences=cls.n_seqs, micro_batch=cls.micro_batch(world),
                    prompt_len=cls.prompt_len, activation=cls.act, kv_cache=cls.act,
                    split=cls.split if world > 1 else "one stage",
                    stages=[[r.start, r.stop] for r in cls.ranges_for(world)],
                    head=("vocabulary-parallel rows " + str([list(v) for v in cls.head_spans(world)]))
                    if cls.vocab_head(world) else "last stage",
                    launch="one CUDA graph per micro-batch and stage; NCCL p2p hand-off")

    def __init__(self, torch, D, rank: int = 0, world: int = 1):
        from dial_cuda.model import Stage
        from dial_cuda.pipeline import ModelStageCompute, NcclChannel, Pipeline
        self.torch, self.D, self.rank, self.world = torch, D, rank, world
        self.cfg = self.model_config()
        self.mb_size = self.micro_batch(world)
        n_mb = self.n_seqs // self.mb_size
        self.ranges = self.ranges_for(world)
        rr = self.ranges[rank]
        self.max_seq = self.prompt_len + self.decode_cap + 16
        self.head_channel = None
        if self.vocab_head(world):
            from dial_cuda.pipeline import head_links
            spans = self.head_spans(world)
            rows = [v1 - v0 for v0, v1 in spans]
            self.stage = Stage(self.cfg, rr.start, rr.stop, n_slots=self.n_seqs, max_seq=self.max_seq,
                               with_head=False, head_rows=spans[rank])
            self.comp = ModelStageCompute(self.stage, n_mb, self.prompt_len, mb_size=self.mb_size,
                                          vocab_head_stages=world)
            self.channel = NcclChannel(rank, world)
            self.head_channel = NcclChannel(rank, world, links=head_links(world, rows))
            self.pipe = Pipeline(rank, world, self.comp, self.channel, n_mb,
                                 head_channel=self.head_channel, head_rows=rows)
        else:
            self.stage = Stage(self.cfg, rr.start, rr.stop, n_slots=self.n_seqs, max_seq=self.max_seq)
            self.comp = ModelStageCompute(self.stage, n_mb, self.prompt_len, mb_size=self.mb_size)
            self.channel = NcclChannel(rank, world) if world > 1 else None  # C-ABI stage communicators
            self.pipe = Pipeline(rank, world, self.comp, self.channel, n_mb)
        st = self.stage
        prompts = None
        if rank == 0:
            g = torch.Generator(device="cuda").manual_seed(SEED)
            prompts = [torch.randint(0, self.cfg.vocab, (self.prompt_len,), generator=g, device=st.device,
                                     dtype=torch.int32) for _ in range(self.n_seqs)]
        # prefill every sequence (untimed: the metric is decode throughput)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        ev0.record()
        self.pipe.prefill(prompts, prompt_len=self.prompt_len)
        ev1.record()
        torch.cuda.synchronize()
        self.prefill_ms = max_over_ranks(ev0.elapsed_time(ev1), world) / self.n_seqs
        self.work_per_step = self.n_seqs  # tokens (whole job)
        self.weight_bytes = st.weight_bytes
        self.steps_done = 0
        self.copies_per_step = n_mb
        self.config = self.describe(world)
        self.details = {"stage_weights_GB": round(self.weight_bytes / 1e9, 3),
                        "prefill_ms_per_seq": round(self.prefill_ms, 2)}

    def run_copy(self, _):
        """One eager micro-batch for the launch count (its state is restored)."""
        c = self.comp
        saved = [t.clone() for t in c.tokens]
        c._eager(0)
        for t, s in zip(c.tokens, saved):
            t.copy_(s)

    def build_graphs(self):
        c = self.comp
        saved = [t.clone() for t in c.tokens]  # the warm-up runs of the capture must not move tokens
        c.capture()
        for t, s in zip(c.tokens, saved):
            t.copy_(s)
        self.torch.cuda.synchronize()

    def _wrap(self):
        if self.steps_done >= self.decode_cap - 1:  # every rank wraps at the same step
            self.pipe.finish()
            self.comp.reset_positions(self.prompt_len)
            self.steps_done = 0

    def step(self):
        self._wrap()
        self.pipe.steps(1)
        self.steps_done += 1

    def step_e2e(self):
        """Serving loop: each token passes through pinned host memory."""
        self._wrap()
        self.pipe.steps(1, host_io=True)
        self.steps_done += 1
        return 4 * self.n_seqs, 4 * self.n_seqs

    def finish(self):
        self.pipe.finish()

    def close(self):
        if self.channel is not None:
            self.channel.close()
        if self.head_channel is not None:
            self.head_channel.close()

    def kernel_roofline(self, reps: int = 5):
        """HBM GB/s of the dominant kernel: this stage's linears (M = one
        micro-batch) launched back to back in model order from one CUDA graph,
        algorithmic bytes over the replay's event time."""
        torch, st = self.torch, self.stage
        lins = st.linears + [h for h in (st.head, st.head_shard) if h is not None]
        R = self.mb_size
        xs, ys = {}, []
        for lin in lins:
            wl = lin.lin
            if wl.in_dim not in xs:
                xs[wl.in_dim] = torch.randn((R, wl.in_dim), device="cuda").to(st.dt)
            ys.append(torch.empty((R, wl.out_dim), device="cuda", dtype=st.dt))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())

        def run():
            for lin, y in zip(lins, ys):
                lin.lin.forward(xs[lin.lin.in_dim], out=y)

        with torch.cuda.stream(side):
            run()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            run()
        gr.replay()
        torch.cuda.synchronize()
        total_b = sum(l.lin.weight_bytes + 2 * R * (l.lin.in_dim + l.lin.out_dim) for l in lins)
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gr.replay()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        del gr
        return total_b / (statistics.median(ts) / 1e3) / 1e9


class LlamaGgufDecode(QwenDecode):
    """Llama-3-8B-shaped GGUF decoder (32 layers, hidden 4096,
    MLP 14336, 32/8 heads, vocab 128256, theta 5e5, no QK-norm), layers Q4_0 and
    head Q8_0 from N(0, 0.02) weights, 32 sequences with 2048-token prompts
    (prefilled before timing), batched decode as P micro-batches of 32/P
    sequences through a pipeline of P stages (one micro-batch of 32 on one GPU).
    A step advances every sequence by one token."""
    metric, unit, bound, dtype = "8B GGUF Q4_0 batched decode tok/s", "tok/s", "hbm", "q4_0 x f16"
    kernel = "gguf_tma_kernel (M = one micro-batch; the stage's linears from one graph, events)"
    traffic = None
    n_seqs, mb_size, prompt_len, decode_cap = 32, None, 2048, 160
    head_layers = 1.4  # Q8_0 head 558 MB vs a Q4_0 layer's 123 MB + 268 MB of KV per step
    act = "f16"

    name = "llama_gguf_decode"

    @classmethod
    def model_config(cls):
        from dial_cuda.model import ModelConfig
        c = ModelConfig.llama3_8b_q4_0()
        c.act_dtype = cls.act
        return c

    @classmethod
    def micro_batch(cls, world):
        """As many micro-batches as stages (one on a single GPU): each stage reads
        its weights once per micro-batch, and with fewer micro-batches than
        stages some stage would idle."""
        assert cls.n_seqs % world == 0, "sequences must split evenly over the stages"
        return cls.n_seqs // world

    @classmethod
    def model_desc(cls):
        return {"workload": "llama3_8b_gguf_q4_0_batched_decode", "model": "Llama-3-8B-shaped, random init",
                "layers": 32, "hidden": 4096, "intermediate": 14336, "heads": "32/8", "vocab": 128256,
                "weights": "Q4_0 layers, Q8_0 head",
                "l2": "3.9 GB of weights + 9 GB of KV per step >> 126 MB L2"}


class QwenDecodeBf16(QwenDecode):
    """qwen3_decode with bf16 activations and KV cache."""
    dtype = "int8 x bf16"
    act = "bf16"
    name = "qwen3_decode_bf16"


class QwenGenerate(QwenDecode):
    """Qwen3-8B-shaped W8A16 decoder, batch 1: a 512-token prompt prefilled
    (untimed; its time is reported), then greedy decode steps of one token,
    f16 activations and KV cache, positions wrapping after 256 steps.  A step
    is one token.  Metric: decode tok/s."""
    metric = "8B W8A16 decode tok/s (batch 1)"
    n_seqs, mb_size, prompt_len, decode_cap = 1, 1, 512, 256
    copies_per_step = 1
    name = "qwen3_generate"

    @classmethod
    def model_desc(cls):
        return dict(super().model_desc(), workload="qwen3_8b_w8a16_generate")


WORKLOADS = {"w8a16_gemv": W8A16Gemv, "gguf_sweep": GgufSweep, "gguf_sweep_m32": GgufSweepM32,
             "gguf_prefill": GgufPrefill, "w8a16_prefill": W8A16Prefill,
             "gguf_k_sweep": GgufKSweep, "gguf_k_prefill": GgufKPrefill,
             "qwen3_decode": QwenDecode, "qwen3_decode_bf16": QwenDecodeBf16,
             "qwen3_generate": QwenGenerate, "llama_gguf_decode": LlamaGgufDecode,
             "attention_batched": AttentionDecode}


# ------------------------------------------------------------------ workloads (CPU oracle)
class CpuWorkload:
    """The same workload on the C oracle (the CPU restatement of the reference's path)."""

    def __init__(self, name):
        import numpy as np

        import oracle as O
        self.O, self.name = O, name
        rng = np.random.default_rng(SEED)
        wl = WORKLOADS[name]
        if name == "w8a16_gemv":
            w = rng.normal(0, 0.02, (wl.N, wl.K)).astype(np.float32)
            self.q, self.s32, _ = O.w8a16_quantize(w)
            self.x = rng.normal(0, 1, (1, wl.K)).astype(np.float16)
            self.work = wl.bytes()
        elif name in ("gguf_k_sweep", "gguf_k_prefill"):
            qts = [{"Q4_K": O.Q4_K, "Q6_K": O.Q6_K}[t] for t in wl.types]
            self.klins = [(O.gguf_k_random_blocks(rng, qt, N, K), qt, N, K)
                          for qt in qts for _, N, K in LLAMA_SHAPES]
            self.M = wl.ms[0]
            self.xk = {K: rng.normal(0, 1, (self.M, K)).astype(np.float16) for _, _, K in LLAMA_SHAPES}
            self.work = wl.flops() if name == "gguf_k_prefill" else wl.bytes()
        elif name == "w8a16_prefill":
            self.wlins = []
            for _, N, K in QWEN_LAYER_LINEARS:
                q, s32, _ = O.w8a16_quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32))
                self.wlins.append((q, s32, K))
            self.xw = {K: rng.normal(0, 1, (wl.M, K)).astype(np.float16) for _, _, K in QWEN_LAYER_LINEARS}
            self.work = wl.flops()
            self.M = wl.M
        else:
            self.lins = []
            for qt in (O.Q4_0, O.Q8_0):
                for _, N, K in LAYER_SHAPES:
                    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
                    self.lins.append((O.gguf_quantize(w, qt), qt, N, K))
            self.xs = {m: rng.normal(0, 1, (m, 12288)).astype(np.float32) for m in wl.ms}
            self.work = wl.flops() if name == "gguf_prefill" else wl.bytes()
            self.ms = wl.ms

    def step(self, frac=1.0):
        """One pass (or, for the big prefill sweep, `frac` of it: a bounded sample)."""
        O = self.O
        if self.name == "w8a16_gemv":
            O.w8a16_linear_f32(self.x, self.q, self.s32)
            return 1.0
        if self.name in ("gguf_k_sweep", "gguf_k_prefill"):  # the CPU QMatMul arithmetic (Q8_K activations)
            mm = max(1, int(round(self.M * frac)))
            for blocks, qt, N, K in self.klins:
                O.gguf_k_linear_candle(self.xk[K][:mm], blocks, qt, N)
            return mm / self.M
        if self.name == "w8a16_prefill":
            mm = max(1, int(round(self.M * frac)))
            for q, s32, K in self.wlins:
                O.w8a16_linear_f32(self.xw[K][:mm], q, s32)
            return mm / self.M
        done = 0.0
        for m in self.ms:
            mm = max(1, int(round(m * frac)))
            for blocks, qt, N, K in self.lins:
                O.gguf_linear_candle(self.xs[m][:mm, :K], blocks, qt, N)
            done = mm / m
        return done


_CPU_QWEN = {}


def _cpu_qwen_model(act):
    """A 36-layer Qwen3-8B-dim oracle model whose layers share one layer's int8
    weights (the CPU cost depends on the shapes only; 193 MB per layer already
    streams from DRAM), built once per process."""
    import numpy as np

    import oracle as O
    if act in _CPU_QWEN:
        return _CPU_QWEN[act]
    rng = np.random.default_rng(SEED)
    H, I, V, Dh, Hq, Hkv = 4096, 12288, 151936, 128, 32, 8
    QKV = (Hq + 2 * Hkv) * Dh

    def q8(shape):
        return (rng.integers(-127, 128, shape, dtype=np.int8),
                np.full(shape[0], 0.02 * 3.5 / 127, np.float32))

    one = np.float16(1.0).view(np.uint16) if act == O.F16 else np.uint16(0x3F80)
    L = {}
    for key, shape in (("qkv", (QKV, H)), ("o", (H, Hq * Dh)), ("gu", (2 * I, H)), ("down", (H, I))):
        L[f"{key}_q"], L[f"{key}_s"] = q8(shape)
    for n, dim in (("input_norm", H), ("post_norm", H), ("q_norm", Dh), ("k_norm", Dh)):
        L[n] = np.full(dim, one, np.uint16)
    block = (rng.standard_normal((4096, H), dtype=np.float32) * 0.02)
    block = block.astype(np.float16).view(np.uint16) if act == O.F16 else O.f32_to_bf16(block)
    embed = np.tile(block, (-(-V // 4096), 1))[:V]
    hq = np.tile(rng.integers(-127, 128, (4096, H), dtype=np.int8), (-(-V // 4096), 1))[:V]
    hs = np.full(V, 0.02 * 3.5 / 127, np.float32)
    cfg = dict(n_layers=36, hidden=H, inter=I, n_heads=Hq, n_kv=Hkv, head_dim=Dh, vocab=V,
               qk_norm=True, eps=1e-6, theta=1e6)
    _CPU_QWEN[act] = (cfg, [L] * 36, embed, np.full(H, one, np.uint16), hq, hs)
    return _CPU_QWEN[act]


def cpu_decode_measure(budget_s, act_name="f16"):
    """Qwen3-8B decode on the C oracle (the CPU restatement of the reference's
    layer + head path): the whole 36-layer model generating 2 greedy tokens
    from a 1-token prompt per pass (each token: 36 layers + final norm + head)."""
    import numpy as np

    import oracle as O
    act = O.F16 if act_name == "f16" else O.BF16
    cfg, layers, embed, norm, hq, hs = _cpu_qwen_model(act)
    prompt = np.array([1], np.int32)
    n_new = 2

    def per_token():
        t0 = time.perf_counter()
        O.decoder_generate(cfg, layers, embed, norm, hq, hs, prompt, n_new, act_dtype=act)
        return (time.perf_counter() - t0) / n_new

    ts = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or not ts:
        ts.append(per_token())
    t_tok = statistics.median(ts)
    sample = (f"{len(ts)} passes of 2 greedy tokens from a 1-token prompt on the 36-layer "
              f"Qwen3-8B-dim oracle model ({act_name}; the layers share one layer's int8 weights); "
              f"attention at context <= 2, so the GPU's 1024-token attention (about 4% of a token's "
              f"multiply-adds) is not in the CPU time")
    return 1.0 / t_tok, t_tok, O.num_threads(), sample


def cpu_gguf_decode_measure(budget_s):
    """Llama-3-8B GGUF batched decode on the C oracle: the candle-style GGUF
    linears (Q8_0-quantised activations, integer block dots) of one Q4_0 layer
    and of the Q8_0 head at M = 4 rows (one micro-batch); a token costs
    32 layers + head over 4.  Attention, norms and RoPE are left out, so the
    CPU rate is an upper bound."""
    import numpy as np

    import oracle as O
    rng = np.random.default_rng(SEED)
    H, I, V, Hq, Hkv, Dh, R = 4096, 14336, 128256, 32, 8, 128, 4

    # the cost depends on the shapes only: random quants with a finite block scale
    def blocks(qt, N, K):
        bb = O.BLOCK_BYTES[qt]
        b = rng.integers(0, 256, (N, K // 32, bb), dtype=np.uint8)
        b[:, :, 0:2] = np.frombuffer(np.float16(0.001).tobytes(), np.uint8)
        return b.reshape(N, -1)

    layer = [(blocks(O.Q4_0, N, K), O.Q4_0, N, K) for N, K in
             (((Hq + 2 * Hkv) * Dh, H), (H, Hq * Dh), (2 * I, H), (H, I))]
    head = (blocks(O.Q8_0, V, H), O.Q8_0, V, H)
    xs = {k: rng.normal(0, 1, (R, k)).astype(np.float32) for k in (H, I)}

    def run(lins):
        t0 = time.perf_counter()
        for b, qt, N, K in lins:
            O.gguf_linear_candle(xs[K], b, qt, N)
        return time.perf_counter() - t0

    run(layer)  # warm-up
    tl, th = [], []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or not tl:
        tl.append(run(layer))
        th.append(run([head]))
    a, b = statistics.median(tl), statistics.median(th)
    t_tok = (32 * a + b) / R
    sample = (f"{len(tl)} x (one Q4_0 layer's 4 linears + the Q8_0 head at 4 rows on the oracle); "
              f"token = (32 x {1e3 * a:.1f} ms + {1e3 * b:.1f} ms) / 4; attention not included")
    return 1.0 / t_tok, t_tok, O.num_threads(), sample


def cpu_attention_measure(budget_s):
    """The same attention in numpy (f32 math on f16 caches, all host threads
    numpy uses) over 4 of the 32 sequences per pass, scaled to KV bytes/s."""
    import numpy as np
    wl = AttentionDecode
    rng = np.random.default_rng(SEED)
    n = 4
    k = rng.standard_normal((n, wl.HKV, wl.CTX, wl.D)).astype(np.float16)
    v = rng.standard_normal((n, wl.HKV, wl.CTX, wl.D)).astype(np.float16)
    q = rng.standard_normal((n, wl.HQ, wl.D)).astype(np.float16)
    rep = wl.HQ // wl.HKV

    def one():
        for s in range(n):
            kf, vf = k[s].astype(np.float32), v[s].astype(np.float32)
            qs = q[s].astype(np.float32).reshape(wl.HKV, rep, wl.D)
            sc = np.einsum("grd,gkd->grk", qs, kf) / np.sqrt(wl.D)
            p = np.exp(sc - sc.max(axis=-1, keepdims=True))
            np.einsum("grk,gkd->grd", p / p.sum(axis=-1, keepdims=True), vf)

    one()
    t0, passes = time.perf_counter(), 0
    while time.perf_counter() - t0 < budget_s or passes == 0:
        one()
        passes += 1
    dt = time.perf_counter() - t0
    per_pass = 2 * n * wl.HKV * wl.CTX * wl.D * 2
    return per_pass * passes / dt, dt / passes, os.cpu_count() or 1, \
        f"{passes} passes over {n} of the {wl.T} sequences (numpy) in {dt:.1f}s"


_CPU_WORKLOADS = {}


def cpu_measure(name, budget_s):
    if name == "attention_batched":
        return cpu_attention_measure(budget_s)
    if name in ("qwen3_decode", "qwen3_generate"):
        return cpu_decode_measure(budget_s, "f16")
    if name == "qwen3_decode_bf16":
        return cpu_decode_measure(budget_s, "bf16")
    if name == "llama_gguf_decode":
        return cpu_gguf_decode_measure(budget_s)
    cw = _CPU_WORKLOADS.get(name) or _CPU_WORKLOADS.setdefault(name, CpuWorkload(name))
    frac = 1.0 if name not in ("gguf_prefill", "w8a16_prefill", "gguf_k_prefill") else 16 / 512  # 16 of 512 rows
    cw.step(frac)  # warm-up
    t0 = time.perf_counter()
    n, work = 0, 0.0
    while True:
        work += cw.step(frac) * cw.work
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    sample = (f"{n} passes of the C oracle in {dt:.1f}s" if frac == 1.0 else
              f"{n} passes over 16 of the 512 rows ({frac:.3f} of a step) in {dt:.1f}s, scaled")
    return work / dt, dt / n, cw.O.num_threads(), sample


def unit_scale(unit):
    return {"GB/s": 1e9, "TFLOP/s": 1e12}.get(unit, 1.0)


def parallelism(wl, world):
    pipelined = getattr(wl, "scaling", "weak") == "strong"
    return f"pipeline x{world}" if pipelined else f"replicas x{world}"


def run_reference(args, rank, world):
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    for _ in range(args.warmup):
        cpu_measure(args.workload, 0.0)
    per_step = max(1.0, min(20.0, 60.0 / max(args.steps, 1)))
    rates, threads, sample = [], 1, ""
    for _ in range(args.steps):
        rate, _, threads, sample = cpu_measure(args.workload, per_step)
        rates.append(rate)
    value = statistics.median(rates) / unit_scale(wl.unit)
    if wl.unit == "tok/s":
        work = wl.n_seqs  # tokens per step
    else:
        work = wl.bytes() if wl.unit == "GB/s" else wl.flops()
    line = {
        "impl": "reference", "metric": wl.metric, "value": round(value, 4), "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(work / (value * unit_scale(wl.unit)) * 1e3, 4),
        "higher_is_better": True, "scaling": getattr(wl, "scaling", "weak"), "vs_baseline": None,
        "dtype": wl.dtype, "data": getattr(wl, "data", DATA),
        "config": dict(wl.describe(world), parallelism=parallelism(wl, world)),
        "cpu_baseline": {"value": round(value, 4), "unit": wl.unit, "cores": threads, "kind": "port",
                         "sample": f"per step: {sample}"},
        "e2e": {"value": round(value, 4), "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU leg
def run_ours(args, rank, local, world):
    import torch

    import dial_cuda as D
    torch.cuda.set_device(local)
    wl = WORKLOADS[args.workload](torch, D, rank=rank, world=world)
    stream = torch.cuda.current_stream()
    pipelined = getattr(wl, "scaling", "weak") == "strong"  # one stage per rank
    # whole-job work per step: replicas each do a step's work, a pipeline does it once
    job_work = wl.work_per_step * (1 if pipelined else world)

    # launches per step, counted on an eager pass
    c0 = D.launch_count()
    if wl.graph:
        wl.run_copy(0)
    else:
        wl.step()
    torch.cuda.synchronize()
    launches_per_step = (D.launch_count() - c0) * getattr(wl, "copies_per_step", 1)
    launches_per_step = int(sum_over_ranks(launches_per_step, world))  # every rank's kernels
    if wl.graph:
        wl.build_graphs()
    for _ in range(max(args.warmup, 3)):
        wl.step()
    if hasattr(wl, "chain_graph"):
        wl.chain_graph.replay()  # the chained graph's first replay uploads it
    torch.cuda.synchronize()
    assert D.lib().dial_device_error(1) == 0

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch, local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed steps
        t_begin.record(stream)
        if hasattr(wl, "run_steps"):  # chained launches: no per-step events
            wl.run_steps(args.steps)
        else:
            for i in range(args.steps):
                starts[i].record(stream)
                wl.step()
                ends[i].record(stream)
        t_end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        w1 = time.perf_counter()
        barrier(world)
    if hasattr(wl, "finish"):
        wl.finish()
    total_ms = max_over_ranks(t_begin.elapsed_time(t_end), world)
    if hasattr(wl, "run_steps"):
        step_ms = [t_begin.elapsed_time(t_end) / args.steps] * args.steps
    else:
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    assert D.lib().dial_device_error(1) == 0

    e2e = None
    if hasattr(wl, "step_e2e"):
        for _ in range(3):
            wl.step_e2e()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d = d2h = 0
        for _ in range(args.steps):
            h2d, d2h = wl.step_e2e()
        e1.record(stream)
        torch.cuda.synchronize()
        if hasattr(wl, "finish"):
            wl.finish()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
        e2e = {"value": round(job_work * args.steps / (e2e_ms / 1e3) / unit_scale(wl.unit), 3),
               "unit": wl.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(e2e_ms / args.steps, 5)}

    pk, peak_src = peaks()
    value = job_work * args.steps / (total_ms / 1e3) / unit_scale(wl.unit)
    # roofline of the dominant kernel: algorithmic work per step / mean step time
    # (for the whole-model decode: the linears' bytes over their per-launch times)
    if hasattr(wl, "kernel_roofline"):
        achieved = wl.kernel_roofline()
        wl.details["step_weight_GBps"] = round(
            wl.weight_bytes * wl.copies_per_step / (statistics.mean(step_ms) / 1e3) / 1e9, 1)
    else:
        achieved = wl.work_per_step / (statistics.mean(step_ms) / 1e3) / unit_scale(wl.unit)
    if wl.bound == "hbm":
        peak = pk["hbm_gbs"]
    else:
        peak = pk["bf16_tflops"]
    line = {
        "metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong" if pipelined else "weak", "vs_baseline": None,
        "dtype": wl.dtype, "data": getattr(wl, "data", DATA),
        "config": dict(wl.config, parallelism=parallelism(wl, world)),
        "roofline": {"bound": wl.bound, "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s" if wl.bound == "hbm" else "TFLOP/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": getattr(wl, "traffic", None) if world == 1 else None,
                     "peak_source": f"{peak_src} ({'hbm_gbs' if wl.bound == 'hbm' else 'bf16_tflops'} burst)",
                     "kernel": wl.kernel},
        "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(w0, w1),
    }
    if getattr(wl, "details", None):
        line["details"] = wl.details
    if hasattr(wl, "close"):
        wl.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, _, threads, sample = cpu_measure(args.workload, args.cpu_budget)
        line["cpu_baseline"] = {"value": round(rate / unit_scale(wl.unit), 4), "unit": wl.unit,
                                "cores": threads, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="qwen3_decode")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--split", choices=["planner", "even"], default=None,
                    help="layer split of the pipeline workloads (default: the workload's)")
    ap.add_argument("--head", choices=["last", "vocab"], default=None,
                    help="output head of the pipeline workloads: on the last stage, or "
                         "vocabulary-parallel over the stages (default: the workload's)")
    args = ap.parse_args()
    if args.split is not None and hasattr(WORKLOADS[args.workload], "split"):
        WORKLOADS[args.workload].split = args.split
    if args.head is not None and hasattr(WORKLOADS[args.workload], "head"):
        WORKLOADS[args.workload].head = args.head
    rank, local, world = dist_setup()
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

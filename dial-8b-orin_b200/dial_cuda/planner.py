"""Stage planner front-end (dial_plan_stages in libdial_cuda.so, host only).

Mirrors the reference's AutoPlanner interface (dial-core/src/spm/planner.rs):

  reference                                   here
  PlannerAlgorithm {Dial, EdgeShard*}         DIAL, EDGESHARD_LATENCY, EDGESHARD_THROUGHPUT
  PlannerDevice / PlannerObjective            PlannerDevice / PlannerObjective (dataclasses)
  LayerMetric::{Uniform, PerLayer}            float or list of floats
  AutoPlanner::plan_with_algorithm            plan_stages(model, objective, devices, algorithm)
  PlanReport / PlannedSegment                 the returned dict

plus local_gpu_plan(), which builds the profile of the GPUs of one node for
the pipeline (each GPU a device, NVLink hand-off) and returns the stages.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Union

from . import DialError, lib

DIAL, EDGESHARD_LATENCY, EDGESHARD_THROUGHPUT = 0, 1, 2
LINKS_STAR, LINKS_CHAIN = 0, 1  # dial_plan_model.link_topology
MASTER, WORKER = 0, 1
MAX_DEVICES = 12
SCORE_DEFINITION = {
    DIAL: "risk_weighted_mean_and_tail_ttft_tpot_energy_and_remote_workers",
    EDGESHARD_LATENCY: "estimated_end_to_end_request_latency_ms",
    EDGESHARD_THROUGHPUT: "estimated_pipeline_bottleneck_ms_per_request",
}

Metric = Union[float, Sequence[float]]


class _Metric(ctypes.Structure):
    _fields_ = [("per_layer", ctypes.POINTER(ctypes.c_double)), ("uniform", ctypes.c_double)]


class _Device(ctypes.Structure):
    _fields_ = [("role", ctypes.c_int), ("enabled", ctypes.c_int),
                ("usable_memory_mb", ctypes.c_double), ("fixed_memory_mb", ctypes.c_double),
                ("layer_memory_mb", _Metric), ("prefill_ms", _Metric), ("decode_ms", _Metric),
                ("has_prefill_p95", ctypes.c_int), ("has_decode_p95", ctypes.c_int),
                ("prefill_p95_ms", _Metric), ("decode_p95_ms", _Metric),
                ("prefill_energy_mj", _Metric), ("decode_energy_mj", _Metric),
                ("rtt_ms", ctypes.c_double), ("protocol_ms", ctypes.c_double),
                ("bandwidth_mbps", ctypes.c_double), ("rtt_p95_ms", ctypes.c_double),
                ("protocol_p95_ms", ctypes.c_double), ("bandwidth_p05_mbps", ctypes.c_double)]


class _Objective(ctypes.Structure):
    _fields_ = [("prompt_tokens", ctypes.c_int), ("output_tokens", ctypes.c_int),
                ("dtype_bytes", ctypes.c_int), ("kv_context_tokens", ctypes.c_int),
                ("ttft_weight", ctypes.c_double), ("tpot_weight", ctypes.c_double),
                ("risk_weight", ctypes.c_double), ("energy_weight", ctypes.c_double),
                ("remote_device_penalty", ctypes.c_double),
                ("min_devices", ctypes.c_int), ("max_devices", ctypes.c_int)]


class _Model(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int), ("hidden_size", ctypes.c_int),
                ("num_attention_heads", ctypes.c_int), ("num_key_value_heads", ctypes.c_int),
                ("max_seq_len", ctypes.c_int),
                ("head_memory_mb", ctypes.c_double), ("head_prefill_ms", ctypes.c_double),
                ("head_decode_ms", ctypes.c_double), ("embed_memory_mb", ctypes.c_double),
                ("embed_prefill_ms", ctypes.c_double), ("embed_decode_ms", ctypes.c_double),
                ("link_topology", ctypes.c_int)]


class _Segment(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("start_layer", ctypes.c_int), ("end_layer", ctypes.c_int),
                ("memory_mb", ctypes.c_double), ("ttft_ms", ctypes.c_double),
                ("tpot_ms", ctypes.c_double), ("tail_ttft_ms", ctypes.c_double),
                ("tail_tpot_ms", ctypes.c_double)]


class _Result(ctypes.Structure):
    _fields_ = [("n_segments", ctypes.c_int), ("segments", _Segment * MAX_DEVICES),
                ("ttft_ms", ctypes.c_double), ("tpot_ms", ctypes.c_double),
                ("tail_ttft_ms", ctypes.c_double), ("tail_tpot_ms", ctypes.c_double),
                ("request_energy_mj", ctypes.c_double), ("score", ctypes.c_double),
                ("states_considered", ctypes.c_int64), ("feasible_transitions", ctypes.c_int64),
                ("rejected_for_memory", ctypes.c_int64)]


_SIGS = {
    "dial_plan_stages": ([ctypes.POINTER(_Model), ctypes.POINTER(_Objective), ctypes.POINTER(_Device),
                          ctypes.c_int, ctypes.c_int, ctypes.POINTER(_Result)], ctypes.c_int),
}


@dataclass
class PlannerDevice:
    name: str
    role: int
    usable_memory_mb: float
    layer_memory_mb: Metric
    prefill_ms: Metric
    decode_ms: Metric
    fixed_memory_mb: float = 0.0
    enabled: bool = True
    prefill_p95_ms: Optional[Metric] = None
    decode_p95_ms: Optional[Metric] = None
    prefill_energy_mj: Metric = 0.0
    decode_energy_mj: Metric = 0.0
    rtt_ms: float = 0.0
    protocol_ms: float = 0.0
    bandwidth_mbps: Optional[float] = None
    rtt_p95_ms: Optional[float] = None
    protocol_p95_ms: Optional[float] = None
    bandwidth_p05_mbps: Optional[float] = None


@dataclass
class PlannerObjective:
    prompt_tokens: int = 512
    output_tokens: int = 128
    dtype_bytes: int = 2
    kv_context_tokens: int = 0
    ttft_weight: float = 0.6
    tpot_weight: float = 0.4
    risk_weight: float = 0.0
    energy_weight: float = 0.0
    remote_device_penalty: float = 0.0
    min_devices: int = 1
    max_devices: Optional[int] = None


@dataclass
class PlannerModel:
    num_layers: int
    hidden_size: int
    num_attention_heads: int
    num_key_value_heads: int
    max_seq_len: int
    head_memory_mb: float = 0.0
    head_prefill_ms: float = 0.0
    head_decode_ms: float = 0.0
    embed_memory_mb: float = 0.0
    embed_prefill_ms: float = 0.0
    embed_decode_ms: float = 0.0
    link_topology: int = 0  # LINKS_STAR (the reference's) or LINKS_CHAIN (stage to stage)


def _metric(v: Metric, keep: list) -> _Metric:
    if isinstance(v, (int, float)):
        return _Metric(None, float(v))
    arr = (ctypes.c_double * len(v))(*[float(x) for x in v])
    keep.append(arr)
    return _Metric(ctypes.cast(arr, ctypes.POINTER(ctypes.c_double)), 0.0)


def plan_stages(model: PlannerModel, objective: PlannerObjective, devices: List[PlannerDevice],
                algorithm: int = DIAL) -> dict:
    """Runs dial_plan_stages; raises DialError with the planner's message on failure."""
    L = lib()
    fn = L.dial_plan_stages
    fn.argtypes, fn.restype = _SIGS["dial_plan_stages"]
    keep: list = []
    arr = (_Device * len(devices))()
    for i, d in enumerate(devices):
        a = arr[i]
        a.role, a.enabled = d.role, int(d.enabled)
        a.usable_memory_mb, a.fixed_memory_mb = d.usable_memory_mb, d.fixed_memory_mb
        a.layer_memory_mb = _metric(d.layer_memory_mb, keep)
        a.prefill_ms, a.decode_ms = _metric(d.prefill_ms, keep), _metric(d.decode_ms, keep)
        a.has_prefill_p95 = int(d.prefill_p95_ms is not None)
        a.has_decode_p95 = int(d.decode_p95_ms is not None)
        a.prefill_p95_ms = _metric(d.prefill_p95_ms if d.prefill_p95_ms is not None else 0.0, keep)
        a.decode_p95_ms = _metric(d.decode_p95_ms if d.decode_p95_ms is not None else 0.0, keep)
        a.prefill_energy_mj = _metric(d.prefill_energy_mj, keep)
        a.decode_energy_mj = _metric(d.decode_energy_mj, keep)
        a.rtt_ms, a.protocol_ms = d.rtt_ms, d.protocol_ms
        a.bandwidth_mbps = d.bandwidth_mbps if d.bandwidth_mbps is not None else -1.0
        a.rtt_p95_ms = d.rtt_p95_ms if d.rtt_p95_ms is not None else -1.0
        a.protocol_p95_ms = d.protocol_p95_ms if d.protocol_p95_ms is not None else -1.0
        a.bandwidth_p05_mbps = d.bandwidth_p05_mbps if d.bandwidth_p05_mbps is not None else -1.0
    o = objective
    obj = _Objective(o.prompt_tokens, o.output_tokens, o.dtype_bytes, o.kv_context_tokens,
                     o.ttft_weight, o.tpot_weight, o.risk_weight, o.energy_weight,
                     o.remote_device_penalty, o.min_devices,
                     o.max_devices if o.max_devices is not None else 0)
    m = model
    mod = _Model(m.num_layers, m.hidden_size, m.num_attention_heads, m.num_key_value_heads,
                 m.max_seq_len, m.head_memory_mb, m.head_prefill_ms, m.head_decode_ms,
                 m.embed_memory_mb, m.embed_prefill_ms, m.embed_decode_ms, m.link_topology)
    res = _Result()
    st = fn(ctypes.byref(mod), ctypes.byref(obj), arr, len(devices), algorithm, ctypes.byref(res))
    if st != 0:
        raise DialError(st, "dial_plan_stages", L.dial_last_error().decode(errors="replace"))
    segs = []
    for i in range(res.n_segments):
        s = res.segments[i]
        d = devices[s.device]
        segs.append({"device": d.name, "device_index": s.device,
                     "role": "master" if d.role == MASTER else "worker",
                     "start_layer": s.start_layer, "end_layer": s.end_layer,
                     "num_layers": s.end_layer - s.start_layer + 1,
                     "estimated_memory_mb": s.memory_mb, "estimated_ttft_ms": s.ttft_ms,
                     "estimated_tpot_ms": s.tpot_ms, "estimated_tail_ttft_ms": s.tail_ttft_ms,
                     "estimated_tail_tpot_ms": s.tail_tpot_ms})
    return {"algorithm": algorithm, "score_definition": SCORE_DEFINITION[algorithm],
            "model_layers": m.num_layers, "hidden_size": m.hidden_size,
            "prompt_tokens": o.prompt_tokens, "output_tokens": o.output_tokens,
            "risk_weight": o.risk_weight, "selected_device_count": res.n_segments,
            "cost": {"ttft_ms": res.ttft_ms, "tpot_ms": res.tpot_ms,
                     "tail_ttft_ms": res.tail_ttft_ms, "tail_tpot_ms": res.tail_tpot_ms,
                     "request_energy_mj": res.request_energy_mj, "score": res.score},
            "segments": segs, "states_considered": res.states_considered,
            "feasible_transitions": res.feasible_transitions,
            "rejected_for_memory": res.rejected_for_memory}


def local_gpu_plan(n_layers: int, n_gpus: int, *, layer_decode_ms: float = 0.071,
                   head_layers: float = 0.0, embed_layers: float = 0.0,
                   layer_memory_mb: float = 193.0, usable_memory_mb: float = 170_000.0,
                   hidden_size: int = 4096, heads: int = 32, kv_heads: int = 8,
                   max_seq_len: int = 4096, link_latency_ms: float = 0.015,
                   link_mbps: float = 770e3 * 8, stages: Optional[int] = None,
                   algorithm: int = EDGESHARD_THROUGHPUT) -> List[range]:
    """Layer ranges of a pipeline over `n_gpus` local GPUs (stage s on GPU s).

    Every GPU is a device with the same per-layer cost (default: a Qwen3-8B
    W8A16 layer's decode time on a B200); the output head and the embedding
    are charged as `head_layers` / `embed_layers` layer-equivalents to the last
    / first stage.  Hand-offs follow the stage-to-stage chain (LINKS_CHAIN):
    each stage after the first receives one hidden state per token over NVLink
    (`link_latency_ms`, `link_mbps`: 770 GB/s per direction, the measured peer
    copy rate).  `stages` forces the stage count (min = max devices); the
    default objective is the pipeline bottleneck (EdgeShardThroughput)."""
    devs = [PlannerDevice(name=f"cuda:{i}", role=MASTER if i == 0 else WORKER,
                          usable_memory_mb=usable_memory_mb, layer_memory_mb=layer_memory_mb,
                          prefill_ms=layer_decode_ms, decode_ms=layer_decode_ms,
                          rtt_ms=link_latency_ms if i else 0.0,
                          bandwidth_mbps=link_mbps if i else None)
            for i in range(n_gpus)]
    k = stages if stages is not None else n_gpus
    obj = PlannerObjective(prompt_tokens=1, output_tokens=1, min_devices=k, max_devices=k)
    model = PlannerModel(n_layers, hidden_size, heads, kv_heads, max_seq_len,
                         link_topology=LINKS_CHAIN,
                         head_memory_mb=head_layers * layer_memory_mb,
                         head_prefill_ms=head_layers * layer_decode_ms,
                         head_decode_ms=head_layers * layer_decode_ms,
                         embed_memory_mb=embed_layers * layer_memory_mb,
                         embed_prefill_ms=embed_layers * layer_decode_ms,
                         embed_decode_ms=embed_layers * layer_decode_ms)
    rep = plan_stages(model, obj, devs, algorithm)
    segs = sorted(rep["segments"], key=lambda s: s["start_layer"])
    return [range(s["start_layer"], s["end_layer"] + 1) for s in segs]

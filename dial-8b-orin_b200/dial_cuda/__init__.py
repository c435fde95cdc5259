"""Python front-end of libdial_cuda.so (the C ABI in include/dial_cuda.h).

This mirrors the reference's linear-module interface so a caller that used
DIAL's `TextLinear` finds the same shape of API:

  reference (lisa301/DIAL-8B-orin)                          here
  configure_worker_w8a16_from_args  worker_w8a16.rs:15-44  configure_worker_w8a16_from_args
  worker_w8a16_enabled / _summary   worker_w8a16.rs:46-63  worker_w8a16_enabled / _summary
  TextLinear::from_dense        worker_w8a16.rs:78-101      TextLinear.from_dense
  TextLinear::forward           worker_w8a16.rs:103-121     TextLinear.forward
  CudaW8A16Linear::from_linear  worker_w8a16.rs:301-366     W8A16Linear.from_linear
  CudaW8A16Linear::forward      worker_w8a16.rs:368-386     W8A16Linear.forward
  load_worker_gguf_linear       worker_gguf.rs:462-522      GgufLinear.from_blocks
  forward_worker_gguf           worker_gguf.rs:574-611      GgufLinear.forward
  QTensor::dequantize(_f16)     worker_gguf.rs:56-63        GgufLinear.dequantize

torch is used only for device memory and the current CUDA stream; all
arithmetic runs in the library's sm_100a kernels.  There is no CPU fallback:
if the library or a GPU is missing, calls raise.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(_HERE)
# DIAL_CUDA_LIB names another build of the library (e.g. one with other tile constants)
LIB_PATH = os.environ.get("DIAL_CUDA_LIB") or os.path.join(PKG_ROOT, "_build", "libdial_cuda.so")

F32, F16, BF16 = 0, 1, 2
Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14

STATUS = {
    0: "ok", 1: "invalid argument", 2: "unsupported dtype", 3: "misaligned", 4: "shape",
    5: "CUDA error", 6: "NCCL error", 7: "timeout", 8: "no device",
}


class DialError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        super().__init__(f"{where}: {STATUS.get(status, status)} ({status}): {message}")
        self.status = status


_lib: Optional[ctypes.CDLL] = None

# name -> (argtypes, restype); kept in the order of include/dial_cuda.h
_vp, _i64, _i32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
ID_BYTES = 128  # DIAL_STAGE_COMM_ID_BYTES

SIGNATURES = {
    "dial_status_string": ([_i32], ctypes.c_char_p),
    "dial_last_error": ([], ctypes.c_char_p),
    "dial_abi_version": ([], _i32),
    "dial_launch_count": ([], ctypes.c_uint64),
    "dial_device_error": ([_i32], _i32),
    "dial_w8a16_quantize": ([_vp, _i32, _i64, _i64, _vp, _vp, _i32, _vp], _i32),
    "dial_w8a16_dequantize": ([_vp, _vp, _i32, _i64, _i64, _vp, _i32, _vp], _i32),
    "dial_w8a16_linear_workspace_bytes": ([_i64], _sz),
    "dial_w8a16_linear": ([_vp, _i32, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _vp, _sz, _vp], _i32),
    "dial_gguf_qs_bytes": ([_i32, _i64, _i64], _sz),
    "dial_gguf_d_bytes": ([_i64, _i64], _sz),
    "dial_gguf_repack": ([_vp, _i32, _i64, _i64, _vp, _vp, _vp], _i32),
    "dial_gguf_unpack": ([_vp, _vp, _i32, _i64, _i64, _vp, _vp], _i32),
    "dial_gguf_quantize": ([_vp, _i32, _i64, _i64, _vp, _vp, _vp], _i32),
    "dial_gguf_dequantize": ([_vp, _vp, _i32, _i64, _i64, _vp, _i32, _vp], _i32),
    "dial_gguf_linear_workspace_bytes": ([_i64, _i64, _i64], _sz),
    "dial_gguf_linear": ([_vp, _i32, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _vp, _sz, _vp], _i32),
    "dial_gguf_linear_noalloc": ([_vp, _i32, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _vp], _i32),
    "dial_gguf_k_row_bytes": ([_i32, _i64], _sz),
    "dial_gguf_k_dequantize": ([_vp, _i32, _i64, _i64, _vp, _i32, _vp], _i32),
    "dial_gguf_k_linear": ([_vp, _i32, _vp, _i32, _vp, _i64, _i64, _i64, _vp], _i32),
    "dial_rmsnorm": ([_vp, _vp, _vp, _vp, _vp, _i32, _i64, _i64, ctypes.c_float, _vp], _i32),
    "dial_rope_tables": ([_vp, _vp, _i32, _i64, _i32, ctypes.c_float, _vp], _i32),
    "dial_qk_norm_rope_kv_append": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i64,
                                     _i32, _i32, _i32, _i64, ctypes.c_float, _i32, _vp], _i32),
    "dial_attention_workspace_bytes": ([_i64, _i32, _i64], _sz),
    "dial_attention": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i32, _i64, _i32, _i32, _i32, _i64,
                        _i64, _vp], _i32),
    "dial_decode_attention_workspace_bytes": ([_i32, _i64], _sz),
    "dial_decode_attention": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i32, _i32,
                               _i32, _i32, _i64, _i64, ctypes.c_float, _i32, _vp], _i32),
    "dial_head_merge": ([_vp, _i32, _i64, _vp, _vp], _i32),
    "dial_check_bounded_wait": ([_vp, _vp, _vp], _i32),
    "dial_swiglu": ([_vp, _vp, _i32, _i64, _i64, _vp], _i32),
    "dial_embedding": ([_vp, _vp, _vp, _i32, _i64, _i64, _i64, _vp], _i32),
    "dial_argmax": ([_vp, _vp, _i32, _i64, _i64, _vp], _i32),
    "dial_stage_comm_unique_id": ([_vp], _i32),
    "dial_stage_comm_init": ([_vp, _i32, _i32, _i32, ctypes.c_double, ctypes.POINTER(_vp)], _i32),
    "dial_stage_comm_send": ([_vp, _vp, _sz, _i32, _vp], _i32),
    "dial_stage_comm_recv": ([_vp, _vp, _sz, _i32, _vp], _i32),
    "dial_stage_comm_wait": ([_vp, _vp], _i32),
    "dial_stage_comm_destroy": ([_vp], _i32),
}


def lib() -> ctypes.CDLL:
    """Load libdial_cuda.so; raises (never falls back) if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}` "
                               "(or __graft_entry__.build()); there is no fallback path")
        L = ctypes.CDLL(LIB_PATH)
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != 0:
        raise DialError(status, where, lib().dial_last_error().decode(errors="replace"))


def launch_count() -> int:
    return int(lib().dial_launch_count())


# ------------------------------------------------------------------ torch plumbing
def _torch():
    import torch  # noqa: PLC0415  (torch is plumbing: device memory and streams)
    return torch


def _require_cuda(t) -> None:
    if not t.is_cuda:
        raise RuntimeError("dial_cuda ops take CUDA tensors; there is no CPU path")
    if not t.is_contiguous():
        raise RuntimeError("dial_cuda ops take contiguous tensors")


def dtype_code(dt) -> int:
    torch = _torch()
    if dt == torch.float32:
        return F32
    if dt == torch.float16:
        return F16
    if dt == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {dt}")


def stream_ptr(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


_stream_ws: dict = {}


def stream_workspace(device, need: int):
    """Zero-filled linear workspace shared by the calls issued on one stream.

    Calls on one stream run one after another, and every call leaves the
    workspace's counters zero, so they can share it; another stream gets its own.
    A stream that is being captured into a CUDA graph must have its workspace
    already (one eager call on that stream first): an allocation inside the
    capture would come from the graph's private pool.
    """
    torch = _torch()
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr())
    ws = _stream_ws.get(key)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("dial_cuda: no linear workspace for the capturing stream; make one "
                               "eager call on that stream before capturing")
        ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
        _stream_ws[key] = ws
    return ws, need


# ------------------------------------------------------------------ W8A16
class W8A16Linear:
    """Per-output-row int8 weight + scale, f16/bf16 activations (CudaW8A16Linear)."""

    def __init__(self, qweight, scales, in_dim: int, out_dim: int, name: str = ""):
        self.qweight, self.scales = qweight, scales
        self.in_dim, self.out_dim, self.name = in_dim, out_dim, name

    @classmethod
    def from_linear(cls, name: str, weight, scale_dtype=None) -> "W8A16Linear":
        """Quantise a dense [out, in] f32/f16 CUDA weight on the GPU (bit-exact with
        worker_w8a16.rs:322-341).  The reference stores f32 scales; f16 is allowed."""
        torch = _torch()
        _require_cuda(weight)
        if weight.dim() != 2:
            raise ValueError("weight must be [out_dim, in_dim]")
        if weight.dtype not in (torch.float32, torch.float16):
            raise TypeError(f"expected f32/f16 weight, got {weight.dtype}")
        scale_dtype = scale_dtype or torch.float32
        N, K = weight.shape
        q = torch.empty((N, K), dtype=torch.int8, device=weight.device)
        s = torch.empty((N,), dtype=scale_dtype, device=weight.device)
        check(lib().dial_w8a16_quantize(weight.data_ptr(), dtype_code(weight.dtype), N, K,
                                        q.data_ptr(), s.data_ptr(), dtype_code(scale_dtype),
                                        stream_ptr()), "dial_w8a16_quantize")
        return cls(q, s, K, N, name)

    def forward(self, x, out=None):
        """x [..., in_dim] f16/bf16 -> [..., out_dim] same dtype (worker_w8a16.rs:368-386)."""
        torch = _torch()
        _require_cuda(x)
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"W8A16 expects F16/BF16 activation, got {x.dtype}")
        if x.shape[-1] != self.in_dim:
            raise ValueError(f"W8A16 input mismatch: expected last dim {self.in_dim}, got {tuple(x.shape)}")
        rows = x.numel() // self.in_dim
        if out is None:
            out = torch.empty((*x.shape[:-1], self.out_dim), dtype=x.dtype, device=x.device)
        ws, need = stream_workspace(x.device, lib().dial_w8a16_linear_workspace_bytes(self.out_dim))
        check(lib().dial_w8a16_linear(x.data_ptr(), dtype_code(x.dtype), self.qweight.data_ptr(),
                                      self.scales.data_ptr(), dtype_code(self.scales.dtype),
                                      out.data_ptr(), rows, self.in_dim, self.out_dim,
                                      ws.data_ptr(), need, stream_ptr()), "dial_w8a16_linear")
        return out

    __call__ = forward

    def dequantize(self, dtype=None):
        torch = _torch()
        dtype = dtype or torch.float32
        w = torch.empty((self.out_dim, self.in_dim), dtype=dtype, device=self.qweight.device)
        check(lib().dial_w8a16_dequantize(self.qweight.data_ptr(), self.scales.data_ptr(),
                                          dtype_code(self.scales.dtype), self.out_dim, self.in_dim,
                                          w.data_ptr(), dtype_code(dtype), stream_ptr()),
              "dial_w8a16_dequantize")
        return w

    @property
    def weight_bytes(self) -> int:
        return self.qweight.numel() + self.scales.numel() * self.scales.element_size()


# ------------------------------------------------------------------ GGUF
class GgufLinear:
    """Q4_0 / Q8_0 weight in the split device layout (candle QMatMul equivalent)."""

    def __init__(self, qs, d, qtype: int, in_dim: int, out_dim: int, name: str = ""):
        self.qs, self.d, self.qtype = qs, d, qtype
        self.in_dim, self.out_dim, self.name = in_dim, out_dim, name
        self._ws = None

    @staticmethod
    def _alloc(qtype: int, N: int, K: int, device):
        torch = _torch()
        qs = torch.empty(lib().dial_gguf_qs_bytes(qtype, N, K), dtype=torch.uint8, device=device)
        d = torch.zeros(lib().dial_gguf_d_bytes(N, K) // 2, dtype=torch.int16, device=device)
        return qs, d

    @classmethod
    def from_blocks(cls, blocks, qtype: int, in_dim: int, out_dim: int, name: str = "") -> "GgufLinear":
        """blocks: CUDA uint8 tensor holding the native GGUF blocks of an [out_dim, in_dim]
        tensor (what load_worker_gguf_linear reads from the file)."""
        _require_cuda(blocks)
        qs, d = cls._alloc(qtype, out_dim, in_dim, blocks.device)
        check(lib().dial_gguf_repack(blocks.data_ptr(), qtype, out_dim, in_dim, qs.data_ptr(),
                                     d.data_ptr(), stream_ptr()), "dial_gguf_repack")
        return cls(qs, d, qtype, in_dim, out_dim, name)

    @classmethod
    def quantize(cls, weight, qtype: int, name: str = "") -> "GgufLinear":
        """GGML reference quantiser on the GPU from a dense f32 [out, in] weight."""
        torch = _torch()
        _require_cuda(weight)
        if weight.dtype != torch.float32:
            raise TypeError("GGUF quantiser takes f32 weights")
        N, K = weight.shape
        qs, d = cls._alloc(qtype, N, K, weight.device)
        check(lib().dial_gguf_quantize(weight.data_ptr(), qtype, N, K, qs.data_ptr(), d.data_ptr(),
                                       stream_ptr()), "dial_gguf_quantize")
        return cls(qs, d, qtype, K, N, name)

    def to_blocks(self):
        torch = _torch()
        bb = 18 if self.qtype == Q4_0 else 34
        out = torch.empty(self.out_dim * (self.in_dim // 32) * bb, dtype=torch.uint8, device=self.qs.device)
        check(lib().dial_gguf_unpack(self.qs.data_ptr(), self.d.data_ptr(), self.qtype, self.out_dim,
                                     self.in_dim, out.data_ptr(), stream_ptr()), "dial_gguf_unpack")
        return out

    def dequantize(self, dtype=None):
        torch = _torch()
        dtype = dtype or torch.float32
        w = torch.empty((self.out_dim, self.in_dim), dtype=dtype, device=self.qs.device)
        check(lib().dial_gguf_dequantize(self.qs.data_ptr(), self.d.data_ptr(), self.qtype,
                                         self.out_dim, self.in_dim, w.data_ptr(), dtype_code(dtype),
                                         stream_ptr()), "dial_gguf_dequantize")
        return w

    def workspace(self, rows: int):
        """Zero-filled workspace shared by the linears issued on the current stream."""
        need = lib().dial_gguf_linear_workspace_bytes(rows, self.in_dim, self.out_dim)
        return stream_workspace(self.qs.device, need)

    def forward(self, x, out=None):
        """x [..., in_dim] f32/f16/bf16 -> [..., out_dim] in x's dtype (worker_gguf.rs:574-611)."""
        torch = _torch()
        _require_cuda(x)
        if x.shape[-1] != self.in_dim:
            raise ValueError(f"GGUF input mismatch: expected last dim {self.in_dim}, got {tuple(x.shape)}")
        rows = x.numel() // self.in_dim
        if out is None:
            out = torch.empty((*x.shape[:-1], self.out_dim), dtype=x.dtype, device=x.device)
        ws, need = self.workspace(rows)
        check(lib().dial_gguf_linear(x.data_ptr(), dtype_code(x.dtype), self.qs.data_ptr(),
                                     self.d.data_ptr(), self.qtype, out.data_ptr(), rows, self.in_dim,
                                     self.out_dim, ws.data_ptr() if need else None, need,
                                     stream_ptr()), "dial_gguf_linear")
        return out

    __call__ = forward

    @property
    def weight_bytes(self) -> int:
        return self.qs.numel() + self.d.numel() * 2


class GgufKLinear:
    """Q4_K / Q6_K weight kept in the file's native super-block layout (the
    reference's Q4_K_M files through candle's QMatMul, worker_gguf.rs:462-611)."""

    def __init__(self, blocks, qtype: int, in_dim: int, out_dim: int, name: str = ""):
        self.blocks, self.qtype = blocks, qtype
        self.in_dim, self.out_dim, self.name = in_dim, out_dim, name

    @classmethod
    def from_blocks(cls, blocks, qtype: int, in_dim: int, out_dim: int, name: str = "") -> "GgufKLinear":
        """blocks: CUDA uint8 tensor with the [out_dim, in_dim] tensor's blocks as
        the file holds them (kept as they are; no device repack)."""
        _require_cuda(blocks)
        row = lib().dial_gguf_k_row_bytes(qtype, in_dim)
        if row == 0:
            raise ValueError(f"GGUF K-quant: bad type {qtype} or in_dim {in_dim} (needs a multiple of 256)")
        if blocks.numel() != row * out_dim:
            raise ValueError(f"GGUF K-quant: expected {row * out_dim} block bytes, got {blocks.numel()}")
        return cls(blocks.contiguous(), qtype, in_dim, out_dim, name)

    def dequantize(self, dtype=None):
        torch = _torch()
        dtype = dtype or torch.float32
        w = torch.empty((self.out_dim, self.in_dim), dtype=dtype, device=self.blocks.device)
        check(lib().dial_gguf_k_dequantize(self.blocks.data_ptr(), self.qtype, self.out_dim, self.in_dim,
                                           w.data_ptr(), dtype_code(dtype), stream_ptr()),
              "dial_gguf_k_dequantize")
        return w

    def forward(self, x, out=None):
        """x [..., in_dim] f32/f16/bf16 -> [..., out_dim] in x's dtype."""
        torch = _torch()
        _require_cuda(x)
        if x.shape[-1] != self.in_dim:
            raise ValueError(f"GGUF input mismatch: expected last dim {self.in_dim}, got {tuple(x.shape)}")
        x = x.contiguous()
        rows = x.numel() // self.in_dim
        if out is None:
            out = torch.empty((*x.shape[:-1], self.out_dim), dtype=x.dtype, device=x.device)
        check(lib().dial_gguf_k_linear(x.data_ptr(), dtype_code(x.dtype), self.blocks.data_ptr(), self.qtype,
                                       out.data_ptr(), rows, self.in_dim, self.out_dim, stream_ptr()),
              "dial_gguf_k_linear")
        return out

    __call__ = forward

    @property
    def weight_bytes(self) -> int:
        return self.blocks.numel()


# ------------------------------------------------------------------ worker selection
# worker_w8a16.rs:9-13: process-wide switch and the converted linears' totals
_WORKER_W8A16 = {"enabled": False, "linears": 0, "weight_bytes": 0}


def _is_f16(dtype) -> bool:
    return dtype in ("f16", "float16", F16) or str(dtype) == "torch.float16"


def configure_worker_w8a16_from_args(requested: bool, worker_mode: bool, device, dtype,
                                     gguf_enabled: bool = False) -> str:
    """worker_w8a16.rs:15-44.  W8A16 linears are enabled iff they were requested,
    no GGUF source is loaded (GGUF takes precedence), the process is a worker,
    the device is CUDA and the model dtype is f16 (the reference op accepts F16
    activations only).  Sets the switch that TextLinear.from_dense reads and
    returns the message the reference logs for the same case ("" when silent)."""
    cuda = str(device).startswith("cuda")
    enabled = bool(requested and not gguf_enabled and worker_mode and cuda and _is_f16(dtype))
    _WORKER_W8A16["enabled"] = enabled
    if requested and gguf_enabled:
        return ("both worker W8A16 and GGUF were requested; GGUF takes precedence and W8A16 is "
                "disabled")
    if requested and not worker_mode:
        return "worker W8A16 ignored in master mode; master weights remain unchanged"
    if requested and not cuda:
        return "worker W8A16 requested on a non-CUDA device; falling back to dense weights"
    if requested and not _is_f16(dtype):
        return f"worker W8A16 requires --dtype f16 (got {dtype}); falling back to dense weights"
    if enabled:
        return ("worker W8A16 enabled: CUDA linear weights use row-wise int8, activations/outputs "
                "remain F16")
    return ""


def worker_w8a16_enabled() -> bool:
    return _WORKER_W8A16["enabled"]


def worker_w8a16_summary():
    """(linears converted, their int8 weight + f32 scale bytes) while enabled, else None."""
    if not _WORKER_W8A16["enabled"]:
        return None
    return _WORKER_W8A16["linears"], _WORKER_W8A16["weight_bytes"]


class TextLinear:
    """Dispatch wrapper with the reference's constructor names (worker_w8a16.rs:65-121)."""

    def __init__(self, inner):
        self.inner = inner

    @classmethod
    def from_dense(cls, name: str, weight, scale_dtype=None, dense=None) -> "TextLinear":
        """worker_w8a16.rs:78-101: a W8A16 linear when the worker switch is on;
        otherwise the caller's own dense module `dense` is wrapped unchanged (the
        reference's TextLinear::Dense -- that path is the caller's, not this
        library's).  With the switch off and no `dense` given this raises."""
        if not worker_w8a16_enabled():
            if dense is None:
                raise RuntimeError(f"{name}: worker W8A16 is not enabled (configure_worker_w8a16_from_args)"
                                   " and no dense module was given")
            return cls(dense)
        lin = W8A16Linear.from_linear(name, weight, scale_dtype)
        _WORKER_W8A16["linears"] += 1
        _WORKER_W8A16["weight_bytes"] += lin.out_dim * lin.in_dim + lin.out_dim * 4  # :351
        return cls(lin)

    @classmethod
    def from_gguf(cls, name: str, blocks, qtype: int, in_dim: int, out_dim: int) -> "TextLinear":
        if qtype in (Q4_K, Q6_K):
            return cls(GgufKLinear.from_blocks(blocks, qtype, in_dim, out_dim, name))
        return cls(GgufLinear.from_blocks(blocks, qtype, in_dim, out_dim, name))

    def forward(self, x, out=None):
        return self.inner.forward(x, out)

    __call__ = forward

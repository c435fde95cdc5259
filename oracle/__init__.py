"""ctypes front-end for the CPU oracle (oracle/dial_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product library in
dial-8b-orin_b200/ never imports this module and never falls back to it.

Every function here follows the reference file:line cited in dial_oracle.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libdial_oracle.so")

F32, F16, BF16 = 0, 1, 2
Q4_0, Q8_0 = 2, 8
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}

_lib = None


def build() -> str:
    """Compile the oracle with oracle/Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "dial_oracle.c")
        ):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    sig = {
        "orc_f32_to_f16": ([vp, vp, i64], None),
        "orc_f16_to_f32": ([vp, vp, i64], None),
        "orc_f32_to_bf16": ([vp, vp, i64], None),
        "orc_bf16_to_f32": ([vp, vp, i64], None),
        "orc_num_threads": ([], i32),
        "orc_w8a16_quantize": ([vp, i32, i64, i64, vp, vp, vp], None),
        "orc_w8a16_dequantize": ([vp, vp, i32, i64, i64, vp], None),
        "orc_w8a16_linear": ([vp, i32, vp, vp, i32, i64, i64, i64, vp, vp], None),
        "orc_w8a16_linear_f32": ([vp, vp, vp, i64, i64, i64, vp], None),
        "orc_gguf_block_bytes": ([i32], i64),
        "orc_gguf_quantize": ([vp, i32, i64, i64, vp], i32),
        "orc_gguf_dequantize": ([vp, i32, i64, i64, vp], i32),
        "orc_gguf_linear_exact": ([vp, i32, vp, i32, i64, i64, i64, vp], i32),
        "orc_gguf_linear_candle": ([vp, i32, vp, i32, i64, i64, i64, vp], i32),
        "orc_q8_0_quantize_rows": ([vp, i32, i64, i64, vp, vp], i32),
        "orc_gguf_k_block_bytes": ([i32], i64),
        "orc_gguf_k_dequantize": ([vp, i32, i64, i64, vp], i32),
        "orc_gguf_k_linear_exact": ([vp, i32, vp, i32, i64, i64, i64, vp], i32),
        "orc_gguf_k_linear_candle": ([vp, i32, vp, i32, i64, i64, i64, vp], i32),
    }
    f32 = ctypes.c_float
    sig.update({
        "orc_rmsnorm": ([vp, vp, vp, vp, vp, i64, i64, f32], None),
        "orc_rope_tables": ([vp, vp, i64, i32, f32], None),
        "orc_decoder_generate": ([ctypes.POINTER(OrcDecoder), ctypes.POINTER(ctypes.c_void_p), vp, vp,
                                  vp, vp, vp, i32, i32, vp, vp], i32),
        "orc_decoder_run": ([ctypes.POINTER(OrcDecoder), ctypes.POINTER(ctypes.c_void_p), vp, vp,
                             vp, vp, vp, i32, i32, vp, vp, vp, vp, vp], i32),
    })
    for name, (argtypes, restype) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = argtypes
        fn.restype = restype


class OrcDecoder(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("qk_norm", ctypes.c_int32), ("eps", ctypes.c_float),
                ("theta", ctypes.c_float), ("act_dtype", ctypes.c_int32),
                ("weight_format", ctypes.c_int32), ("head_format", ctypes.c_int32)]


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, res: np.ndarray | None = None):
    """f16 in/out: (h, y) with h = f16(x + res) (or x), y = f16(h*rsqrt(mean(h^2)+eps)*w)."""
    x = np.ascontiguousarray(x, np.float16)
    rows, dim = x.shape
    y = np.empty_like(x)
    h = np.empty_like(x)
    r = None if res is None else np.ascontiguousarray(res, np.float16)
    lib().orc_rmsnorm(_p(x), _p(r), _p(h), _p(np.ascontiguousarray(w, np.float16)), _p(y), rows, dim,
                      eps)
    return h, y


def rope_tables(max_pos: int, head_dim: int, theta: float):
    c = np.empty((max_pos, head_dim // 2), np.float16)
    s = np.empty_like(c)
    lib().orc_rope_tables(_p(c), _p(s), max_pos, head_dim, theta)
    return c, s


def decoder_generate(cfg: dict, layers: list, embed: np.ndarray, final_norm: np.ndarray,
                     head_q: np.ndarray, head_s, prompt, n_new: int, act_dtype: int = F16,
                     weight_format: int = 0, head_format: int = 0, forced=None,
                     return_logits: bool = False, return_hidden: bool = False):
    """Greedy generation on the oracle decoder.

    act_dtype F16 or BF16: `embed`, the norms and every activation are 16-bit
    patterns of that type (numpy float16, or uint16 holding bf16 bits).
    weight_format / head_format: 0 W8A16 with f32 scales, 1 W8A16 with f16
    scales, Q4_0 or Q8_0 (native GGML blocks [N, K/32 * block bytes], `*_s`
    None).  layers: list of dicts with `qkv_q, o_q, gu_q, down_q` (int8 or
    blocks), `*_s` (scales or None) and `input_norm, post_norm, q_norm, k_norm`
    (the QK norms may be None when cfg["qk_norm"] is false).
    forced: optional [n_new] tokens fed back instead of the argmax (teacher forcing).
    Returns (tokens, top1-top2 margins of the rounded logits), plus the
    [n_new, vocab] f32 logits with return_logits and the [n_new, hidden] bits of
    the last position's residual stream before the final norm with
    return_hidden."""
    keys = ["qkv_q", "qkv_s", "o_q", "o_s", "gu_q", "gu_s", "down_q", "down_s", "input_norm",
            "post_norm", "q_norm", "k_norm"]
    keep = []
    ptrs = (ctypes.c_void_p * (len(layers) * len(keys)))()
    for i, L in enumerate(layers):
        for j, k in enumerate(keys):
            if L.get(k) is None:
                ptrs[i * len(keys) + j] = None
                continue
            a = np.ascontiguousarray(L[k])
            keep.append(a)
            ptrs[i * len(keys) + j] = a.ctypes.data
    d = OrcDecoder(cfg["n_layers"], cfg["hidden"], cfg["inter"], cfg["n_heads"], cfg["n_kv"],
                   cfg["head_dim"], cfg["vocab"], int(cfg["qk_norm"]), cfg["eps"], cfg["theta"],
                   act_dtype, weight_format, head_format)
    prompt = np.ascontiguousarray(prompt, np.int32)
    toks = np.empty(n_new, np.int32)
    margins = np.empty(n_new, np.float32)
    bits = lambda a: np.ascontiguousarray(a).view(np.uint16)
    head_q = np.ascontiguousarray(head_q)
    head_s = None if head_s is None else np.ascontiguousarray(head_s)
    fz = None if forced is None else np.ascontiguousarray(forced, np.int32)
    logits = np.empty((n_new, cfg["vocab"]), np.float32) if return_logits else None
    hidden = np.empty((n_new, cfg["hidden"]), np.uint16) if return_hidden else None
    rc = lib().orc_decoder_run(ctypes.byref(d), ptrs, _p(bits(embed)), _p(bits(final_norm)),
                               _p(head_q), _p(head_s), _p(prompt), len(prompt), n_new, _p(fz),
                               _p(toks), _p(margins), _p(logits), _p(hidden))
    assert rc == 0, "orc_decoder_run rejected its configuration"
    out = (toks, margins)
    if return_logits:
        out += (logits,)
    if return_hidden:
        out += (hidden,)
    return out


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _dt(a: np.ndarray, bf16: bool = False) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint16 and bf16:
        return BF16
    raise TypeError(f"unsupported activation dtype {a.dtype}")


# ---------------------------------------------------------------- conversions
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(x), _p(out), x.size)
    return out


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty(x.shape, np.float32)
    lib().orc_bf16_to_f32(_p(x), _p(out), x.size)
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16(_p(x), _p(out), x.size)
    return out


# ---------------------------------------------------------------- W8A16
def w8a16_quantize(w: np.ndarray):
    """w [N,K] f32 or f16 -> (q int8 [N,K], scale f32 [N], scale f16 [N])."""
    w = np.ascontiguousarray(w)
    N, K = w.shape
    q = np.empty((N, K), np.int8)
    s32 = np.empty(N, np.float32)
    s16 = np.empty(N, np.uint16)
    lib().orc_w8a16_quantize(_p(w), _dt(w), N, K, _p(q), _p(s32), _p(s16))
    return q, s32, s16.view(np.float16)


def w8a16_dequantize(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale)
    N, K = q.shape
    out = np.empty((N, K), np.float32)
    lib().orc_w8a16_dequantize(_p(q), _p(scale), _dt(scale), N, K, _p(out))
    return out


def w8a16_linear(x: np.ndarray, q: np.ndarray, scale: np.ndarray, x_is_bf16: bool = False):
    """x [M,K] (f16, or uint16 bf16 bits) -> (y_f32 [M,N] pre-rounding, y_half [M,N] bits)."""
    x = np.ascontiguousarray(x)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale)
    M, K = x.shape
    N = q.shape[0]
    y = np.empty((M, N), np.float32)
    yh = np.empty((M, N), np.uint16)
    lib().orc_w8a16_linear(_p(x), _dt(x, x_is_bf16), _p(q), _p(scale), _dt(scale), M, K, N,
                           _p(y), _p(yh))
    return y, yh


def w8a16_linear_f32(x_f16: np.ndarray, q: np.ndarray, scale_f32: np.ndarray) -> np.ndarray:
    x_f16 = np.ascontiguousarray(x_f16, dtype=np.float16)
    M, K = x_f16.shape
    N = q.shape[0]
    y = np.empty((M, N), np.float16)
    lib().orc_w8a16_linear_f32(_p(x_f16), _p(q), _p(np.ascontiguousarray(scale_f32, np.float32)),
                               M, K, N, _p(y))
    return y


# ---------------------------------------------------------------- GGUF
def gguf_quantize(w: np.ndarray, qtype: int) -> np.ndarray:
    """w [N,K] f32 -> native GGML blocks, uint8 [N, K/32*block_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.empty((N, K // 32 * BLOCK_BYTES[qtype]), np.uint8)
    rc = lib().orc_gguf_quantize(_p(w), qtype, N, K, _p(out))
    assert rc == 0
    return out


def gguf_dequantize(blocks: np.ndarray, qtype: int, N: int, K: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((N, K), np.float32)
    rc = lib().orc_gguf_dequantize(_p(blocks), qtype, N, K, _p(out))
    assert rc == 0
    return out


def gguf_linear_exact(x: np.ndarray, blocks: np.ndarray, qtype: int, N: int,
                      x_is_bf16: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x)
    M, K = x.shape
    y = np.empty((M, N), np.float64)
    rc = lib().orc_gguf_linear_exact(_p(x), _dt(x, x_is_bf16), _p(np.ascontiguousarray(blocks)),
                                     qtype, M, K, N, _p(y))
    assert rc == 0
    return y


def gguf_linear_candle(x: np.ndarray, blocks: np.ndarray, qtype: int, N: int,
                       x_is_bf16: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x)
    M, K = x.shape
    y = np.empty((M, N), np.float32)
    rc = lib().orc_gguf_linear_candle(_p(x), _dt(x, x_is_bf16), _p(np.ascontiguousarray(blocks)),
                                      qtype, M, K, N, _p(y))
    assert rc == 0
    return y


# ---------------------------------------------------------------- GGUF K-quants
Q4_K, Q6_K = 12, 14
K_BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}


def gguf_k_random_blocks(rng, qtype: int, N: int, K: int, scale: float = 1e-4) -> np.ndarray:
    """Seeded K-quant blocks [N, K/256*bytes]: random quant, scale and min bytes
    with finite f16 super-block scales ~ N(0, scale) (GGUF weights as a file
    holds them; a quantiser is not needed to exercise the arithmetic)."""
    nb = K // 256
    bb = K_BLOCK_BYTES[qtype]
    raw = rng.integers(0, 256, (N, nb, bb), dtype=np.uint8)
    d = rng.normal(0.0, scale, (N, nb)).astype(np.float16)
    if qtype == Q4_K:
        raw[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
        dmin = np.abs(rng.normal(0.0, scale, (N, nb))).astype(np.float16)
        raw[:, :, 2:4] = dmin.view(np.uint8).reshape(N, nb, 2)
    else:
        raw[:, :, 208:210] = d.view(np.uint8).reshape(N, nb, 2)
    return raw.reshape(N, nb * bb)


def gguf_k_dequantize(blocks: np.ndarray, qtype: int, N: int, K: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((N, K), np.float32)
    rc = lib().orc_gguf_k_dequantize(_p(blocks), qtype, N, K, _p(out))
    assert rc == 0
    return out


def gguf_k_linear_exact(x: np.ndarray, blocks: np.ndarray, qtype: int, N: int,
                        x_is_bf16: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x)
    M, K = x.shape
    y = np.empty((M, N), np.float64)
    rc = lib().orc_gguf_k_linear_exact(_p(x), _dt(x, x_is_bf16), _p(np.ascontiguousarray(blocks)),
                                       qtype, M, K, N, _p(y))
    assert rc == 0
    return y


def gguf_k_linear_candle(x: np.ndarray, blocks: np.ndarray, qtype: int, N: int,
                         x_is_bf16: bool = False) -> np.ndarray:
    """GGML / candle CPU arithmetic for Q4_K / Q6_K (Q8_K activations, integer dots)."""
    x = np.ascontiguousarray(x)
    M, K = x.shape
    y = np.empty((M, N), np.float32)
    rc = lib().orc_gguf_k_linear_candle(_p(x), _dt(x, x_is_bf16), _p(np.ascontiguousarray(blocks)),
                                        qtype, M, K, N, _p(y))
    assert rc == 0
    return y


def q8_0_quantize_rows(x: np.ndarray, x_is_bf16: bool = False):
    x = np.ascontiguousarray(x)
    M, K = x.shape
    qs = np.empty((M, K), np.int8)
    d = np.empty((M, K // 32), np.uint16)
    rc = lib().orc_q8_0_quantize_rows(_p(x), _dt(x, x_is_bf16), M, K, _p(qs), _p(d))
    assert rc == 0
    return qs, d.view(np.float16)


def num_threads() -> int:
    return int(lib().orc_num_threads())

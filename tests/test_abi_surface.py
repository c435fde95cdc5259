"""CPU-side checks of libdial_cuda.so: it loads, it exports every symbol that
include/dial_cuda.h declares, and argument validation returns the documented
status codes without touching a GPU (the reference returns
candle_core::Error::Msg for the same cases, worker_w8a16.rs:369-378, :410-416).
"""
import ctypes
import os
import re

import pytest

import dial_cuda as D

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_symbols():
    names = []
    for h in HEADERS:
        text = open(h).read()
        names += re.findall(r"^DIAL_API\s+[\w\s\*]+?\b(dial_\w+)\s*\(", text, flags=re.M)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "dial_w8a16_linear" in names and "dial_gguf_linear" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    L = D.lib()
    missing = [n for n in declared_symbols() if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"


def test_python_signatures_cover_header():
    from dial_cuda import model, planner
    bound = set(D.SIGNATURES) | set(model._SIGS) | set(planner._SIGS)
    assert set(declared_symbols()) <= bound, set(declared_symbols()) - bound


def test_abi_version_and_status_strings():
    L = D.lib()
    assert L.dial_abi_version() == 1
    assert L.dial_status_string(0) == b"ok"
    assert L.dial_status_string(3).startswith(b"misaligned")


def test_validation_without_gpu():
    L = D.lib()
    # null pointers
    assert L.dial_w8a16_linear(None, D.F16, None, None, D.F32, None, 1, 64, 64, None, 0, None) == 1
    assert b"null" in L.dial_last_error()
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: checks fail first
    # f32 activations are rejected by W8A16 (the reference requires F16)
    assert L.dial_w8a16_linear(fake, D.F32, fake, fake, D.F32, fake, 1, 64, 64, None, 0, None) == 2
    # K not a multiple of 16
    assert L.dial_w8a16_linear(fake, D.F16, fake, fake, D.F32, fake, 1, 60, 64, None, 0, None) == 4
    # misaligned activation pointer
    odd = ctypes.c_void_p(0x1002)
    assert L.dial_w8a16_linear(odd, D.F16, fake, fake, D.F32, fake, 1, 64, 64, None, 0, None) == 3
    # non-positive sizes
    assert L.dial_w8a16_linear(fake, D.F16, fake, fake, D.F32, fake, 0, 64, 64, None, 0, None) == 1
    # GGUF: bad type, K % 32, missing workspace
    assert L.dial_gguf_linear(fake, D.F32, fake, fake, 3, fake, 1, 64, 64, None, 0, None) == 2
    assert L.dial_gguf_linear(fake, D.F32, fake, fake, D.Q4_0, fake, 1, 48, 64, None, 0, None) == 4
    assert L.dial_gguf_linear(fake, D.F32, fake, fake, D.Q4_0, fake, 1, 64, 64, None, 0, None) == 1
    assert b"workspace" in L.dial_last_error()


def test_gguf_k_validation_without_gpu():
    L = D.lib()
    fake = ctypes.c_void_p(0x1000)
    # Q4_K / Q6_K only take K % 256 == 0, and only the K-quant entry points take them
    assert L.dial_gguf_k_linear(fake, D.F32, fake, D.Q4_K, fake, 1, 4000, 64, None) == 4
    assert L.dial_gguf_k_linear(fake, D.F32, fake, D.Q4_0, fake, 1, 4096, 64, None) == 2
    assert L.dial_gguf_k_linear(None, D.F32, fake, D.Q6_K, fake, 1, 4096, 64, None) == 1
    assert L.dial_gguf_k_linear(fake, D.F32, fake, D.Q6_K, fake, 0, 4096, 64, None) == 1
    # Q4_K blocks are read as 16-byte words, Q6_K blocks as 2-byte words
    assert L.dial_gguf_k_linear(fake, D.F32, ctypes.c_void_p(0x1002), D.Q4_K, fake, 1, 4096, 64, None) == 3
    assert L.dial_gguf_k_linear(fake, D.F32, ctypes.c_void_p(0x1001), D.Q6_K, fake, 1, 4096, 64, None) == 3
    assert L.dial_gguf_k_linear(ctypes.c_void_p(0x1008), D.F32, fake, D.Q6_K, fake, 1, 4096, 64, None) == 3
    assert L.dial_gguf_k_dequantize(fake, D.Q4_K, 4, 4096, fake, 7, None) == 2
    assert L.dial_gguf_linear(fake, D.F32, fake, fake, D.Q4_K, fake, 1, 4096, 64, None, 0, None) == 2
    assert L.dial_gguf_k_row_bytes(D.Q4_K, 4096) == 16 * 144
    assert L.dial_gguf_k_row_bytes(D.Q6_K, 14336) == 56 * 210
    assert L.dial_gguf_k_row_bytes(D.Q6_K, 4000) == 0
    assert L.dial_gguf_k_row_bytes(D.Q8_0, 4096) == 0


def test_gguf_size_helpers():
    L = D.lib()
    # K=4096 -> 32 groups of 4 blocks; Q4_0 64 B / group, Q8_0 128 B / group
    assert L.dial_gguf_qs_bytes(D.Q4_0, 10, 4096) == 10 * 32 * 64
    assert L.dial_gguf_qs_bytes(D.Q8_0, 10, 4096) == 10 * 32 * 128
    assert L.dial_gguf_d_bytes(10, 4096) == 16 * 128 * 2  # rows padded to 16
    # K=96 -> 3 blocks padded to one group of 4
    assert L.dial_gguf_qs_bytes(D.Q4_0, 1, 96) == 64
    assert L.dial_gguf_linear_workspace_bytes(1, 4096, 64) > 0


def test_no_cpu_fallback_when_library_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(D, "_lib", None)
    monkeypatch.setattr(D, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(RuntimeError, match="no fallback"):
        D.lib()

"""Generate the GGUF Q4_0 / Q8_0 golden fixtures in tests/golden/.

The reference (DIAL) does its GGUF arithmetic in candle-core 0.11.0, which is
not vendored and cannot be built here (no Rust toolchain).  The GGML block
format is public; the installed `gguf` Python package (gguf-py 0.19.0, the
llama.cpp project's own Python implementation, quants.py Q4_0/Q8_0
quantize_blocks / dequantize_blocks) is an independent implementation of the
same format.  This script runs it on seeded inputs (plus hand-made edge rows)
and stores inputs, block bytes and dequantised values.  The oracle and the
CUDA kernels are then checked against these bytes and values.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np

SEED = 299792458  # the reference's default --seed (dial-core/src/lib.rs:214-215)


def weights() -> np.ndarray:
    rng = np.random.default_rng(SEED)
    K = 256
    rows = [rng.normal(0.0, 0.02, K).astype(np.float32) for _ in range(6)]
    edge = []
    edge.append(np.zeros(K, np.float32))                                  # all-zero row (d = 0)
    r = rng.normal(0.0, 0.02, K).astype(np.float32)
    r[5], r[9] = 0.5, -0.5                                                # |max| tie: first wins
    edge.append(r)
    edge.append(np.linspace(-1.0, 1.0, K, dtype=np.float32))              # exact rounding ties
    edge.append(rng.normal(0.0, 1e-6, K).astype(np.float32))              # subnormal f16 scales
    edge.append(rng.normal(0.0, 300.0, K).astype(np.float32))             # large magnitudes
    r = np.full(K, -0.25, np.float32)
    r[::3] = 0.125                                                        # negative-dominant blocks
    edge.append(r)
    return np.stack(rows + edge)


def main() -> None:
    from gguf import GGMLQuantizationType, quants  # independent GGML implementation

    w = weights()
    out = {"w": w}
    for name, qt in (("q4_0", GGMLQuantizationType.Q4_0), ("q8_0", GGMLQuantizationType.Q8_0)):
        blocks = quants.quantize(w, qt)
        deq = quants.dequantize(blocks, qt).astype(np.float32)
        out[f"{name}_blocks"] = np.ascontiguousarray(blocks, dtype=np.uint8)
        out[f"{name}_dequant"] = deq
    rng = np.random.default_rng(SEED + 1)
    x = rng.normal(0.0, 1.0, (3, w.shape[1])).astype(np.float32)
    out["x"] = x
    # exact f64 linear on the gguf-dequantised weights: the value every linear
    # implementation is compared with (tolerance stated in the tests)
    for name in ("q4_0", "q8_0"):
        out[f"{name}_linear_f64"] = x.astype(np.float64) @ out[f"{name}_dequant"].astype(np.float64).T
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gguf_q4_0_q8_0.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: " + ", ".join(f"{k}{v.shape}" for k, v in out.items()))


if __name__ == "__main__":
    main()

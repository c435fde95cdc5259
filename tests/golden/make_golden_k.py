"""Generate the GGUF Q4_K / Q6_K golden fixtures in tests/golden/.

The reference's GGUF files are Q4_K_M (docs/worker_gguf.md:1-6), loaded through
candle-core 0.11.0's QMatMul (worker_gguf.rs:462-522), which is not vendored and
cannot be built here.  The installed `gguf` Python package (gguf-py 0.19.0, the
llama.cpp project's own implementation, quants.py Q4_K / Q6_K dequantize_blocks)
is an independent implementation of the same public block format.  This script
runs its dequantisers on seeded blocks plus hand-made edge blocks and stores the
block bytes and the dequantised f32 values; the oracle and the CUDA kernels are
checked against them.  (gguf-py has no K-quant quantiser, and neither path
needs one: the linear reads the file's blocks as they are.)

Run from the repository root:  python tests/golden/make_golden_k.py
"""
from __future__ import annotations

import os

import numpy as np

SEED = 299792458  # the reference's default --seed (dial-core/src/lib.rs:214-215)
N, K = 10, 512    # 2 super-blocks per row


def blocks(rng, bb: int, d_off: int | None, dmin_off: int | None) -> np.ndarray:
    """[N, K/256*bb] bytes; rows 0-5 random, rows 6-9 edge cases."""
    nb = K // 256
    raw = rng.integers(0, 256, (N, nb, bb), dtype=np.uint8)

    def put(row, off, vals):
        raw[row, :, off:off + 2] = np.asarray(vals, np.float16).view(np.uint8).reshape(nb, 2)

    for r in range(N):
        put(r, d_off, rng.normal(0.0, 1e-3, nb))
        if dmin_off is not None:
            put(r, dmin_off, np.abs(rng.normal(0.0, 1e-3, nb)))
    # row 6: every quant/scale byte 0xFF (largest 4/6-bit values, every high bit)
    raw[6] = 0xFF
    put(6, d_off, [0.5, -0.25])
    if dmin_off is not None:
        put(6, dmin_off, [0.125, 2.0])
    # row 7: zero super-block scales
    put(7, d_off, [0.0, -0.0])
    if dmin_off is not None:
        put(7, dmin_off, [0.0, 0.0])
    # row 8: subnormal f16 scales
    put(8, d_off, [6e-8, -3e-6])
    if dmin_off is not None:
        put(8, dmin_off, [5.96e-8, 1e-5])
    # row 9: large scales (products near the f16 range)
    put(9, d_off, [60000.0, -1000.0])
    if dmin_off is not None:
        put(9, dmin_off, [30000.0, 7.0])
    return raw.reshape(N, nb * bb)


def main() -> None:
    from gguf import GGMLQuantizationType, quants  # independent GGML implementation

    rng = np.random.default_rng(SEED)
    out = {}
    for name, qt, bb, d_off, dmin_off in (("q4_k", GGMLQuantizationType.Q4_K, 144, 0, 2),
                                          ("q6_k", GGMLQuantizationType.Q6_K, 210, 208, None)):
        b = blocks(rng, bb, d_off, dmin_off)
        out[f"{name}_blocks"] = b
        out[f"{name}_dequant"] = quants.dequantize(b, qt).astype(np.float32).reshape(N, K)
    x = rng.normal(0.0, 1.0, (3, K)).astype(np.float32)
    out["x"] = x
    for name in ("q4_k", "q6_k"):
        out[f"{name}_linear_f64"] = x.astype(np.float64) @ out[f"{name}_dequant"].astype(np.float64).T
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gguf_q4_k_q6_k.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: " + ", ".join(f"{k}{v.shape}" for k, v in out.items()))


if __name__ == "__main__":
    main()

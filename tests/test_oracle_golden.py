"""Pins the CPU oracle before anything is checked against it.

* GGUF Q4_0 / Q8_0: block bytes and dequantised values against the fixtures
  made by tests/golden/make_golden.py with the independent `gguf` package
  (gguf-py 0.19.0 quants.py) -- bit-exact, edge rows included.
* W8A16: the reference's own known-answer test
  `cuda_w8a16_matches_dense_for_decode_and_prefill`
  (dial-core/src/models/qwen3_vl/worker_w8a16.rs:483-516) restated: closed-form
  weights and inputs, K=64, N=37, rows {1, 9}, max_abs < 0.04 against the
  dense f16 linear.
* Quantiser rules of worker_w8a16.rs:334-341 (F5): half away from zero,
  multiply by the f32 reciprocal, clamp to +-127, scale 1.0 for zero rows.
"""
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gguf_q4_0_q8_0.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name,qt", [("q4_0", O.Q4_0), ("q8_0", O.Q8_0)])
def test_gguf_quantize_matches_gguf_package(golden, name, qt):
    w = golden["w"]
    blocks = O.gguf_quantize(w, qt)
    assert np.array_equal(blocks, golden[f"{name}_blocks"])


@pytest.mark.parametrize("name,qt", [("q4_0", O.Q4_0), ("q8_0", O.Q8_0)])
def test_gguf_dequantize_bit_exact(golden, name, qt):
    w = golden["w"]
    deq = O.gguf_dequantize(golden[f"{name}_blocks"], qt, *w.shape)
    assert np.array_equal(deq.view(np.uint32), golden[f"{name}_dequant"].view(np.uint32))


@pytest.mark.parametrize("name,qt", [("q4_0", O.Q4_0), ("q8_0", O.Q8_0)])
def test_gguf_linear_oracles(golden, name, qt):
    x = golden["x"]
    blocks = golden[f"{name}_blocks"]
    N = golden["w"].shape[0]
    exact = O.gguf_linear_exact(x, blocks, qt, N)
    ref = golden[f"{name}_linear_f64"]
    scale = np.abs(ref).max()
    assert np.abs(exact - ref).max() <= 1e-9 * scale
    # candle-style (Q8_0 activations, integer block dots) on the N(0, 0.02)
    # rows: within the north-star tolerance of the exact product (max error
    # relative to the largest output, 1e-2).  The hand-made edge rows are
    # left out: with K=256 their activation-quantisation error is of that size.
    cand = O.gguf_linear_candle(x, blocks, qt, N)
    r = slice(0, 6)
    assert np.abs(cand[:, r] - ref[:, r]).max() <= 1e-2 * np.abs(ref[:, r]).max()


def _reference_kat_weights():
    # worker_w8a16.rs:486-491: sin(idx*0.037)*0.25 + ((idx%11)-5)*0.002, as f32 then f16
    idx = np.arange(37 * 64, dtype=np.float32)
    w = (np.sin(idx * np.float32(0.037)) * np.float32(0.25)
         + ((np.arange(37 * 64) % 11).astype(np.float32) - np.float32(5.0)) * np.float32(0.002))
    return w.astype(np.float32).reshape(37, 64).astype(np.float16)


def test_reference_w8a16_kat():
    w16 = _reference_kat_weights()
    q, s32, _ = O.w8a16_quantize(w16)
    for rows in (1, 9):
        # worker_w8a16.rs:496-499: cos(idx*0.071)*0.5, f16
        x = (np.cos(np.arange(rows * 64, dtype=np.float32) * np.float32(0.071)) * np.float32(0.5))
        x = x.astype(np.float16).reshape(rows, 64)
        dense = (x.astype(np.float32) @ w16.astype(np.float32).T).astype(np.float16)
        _, yh = O.w8a16_linear(x, q, s32)
        actual = yh.view(np.float16).astype(np.float32)
        max_abs = np.abs(dense.astype(np.float32) - actual).max()
        assert max_abs < 0.04, f"rows={rows} max_abs={max_abs}"


def test_w8a16_quantizer_rules():
    # row 0: zero row -> scale 1, q 0; row 1: ties; row 2: exact extremes
    K = 16
    w = np.zeros((3, K), np.float32)
    w[1, :] = np.float32(127.0) * np.array([0.5, -0.5, 1.5, -1.5, 2.5, 0.0, 1.0, -1.0] * 2, np.float32) / 127.0
    w[1, 15] = 127.0
    w[2, :] = np.linspace(-3.0, 3.0, K, dtype=np.float32)
    q, s32, s16 = O.w8a16_quantize(w)
    assert s32[0] == np.float32(1.0) and not q[0].any()
    assert s32[1] == np.float32(127.0) / np.float32(127.0)
    # scale 1.0 -> q = round half away from zero of the value itself
    assert list(q[1, :8]) == [1, -1, 2, -2, 3, 0, 1, -1]
    assert q[2, 0] == -127 and q[2, -1] == 127
    assert s16[2] == np.float16(s32[2])
    # restated in numpy: q = clamp(round_half_away(w * (1/s)), +-127)
    inv = (np.float32(1.0) / s32).astype(np.float32)
    prod = (w * inv[:, None]).astype(np.float32)
    ref = np.clip(np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5)), -127, 127).astype(np.int8)
    assert np.array_equal(q, ref)


def test_w8a16_quantize_random_matches_numpy():
    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    q, s32, _ = O.w8a16_quantize(w)
    amax = np.abs(w).max(axis=1)
    s = (amax / np.float32(127.0)).astype(np.float32)
    assert np.array_equal(s, s32)
    inv = (np.float32(1.0) / s).astype(np.float32)
    prod = (w * inv[:, None]).astype(np.float32)
    ref = np.clip(np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5)), -127, 127).astype(np.int8)
    assert np.array_equal(q, ref)


def test_half_conversions_match_numpy():
    rng = np.random.default_rng(3)
    v = np.concatenate([rng.normal(0, 1, 4096), rng.normal(0, 1e-5, 1024), rng.normal(0, 3e4, 256),
                        [65504.0, 65519.9, 65520.0, -7e4, 6.1e-5, 5.96e-8, 2.98e-8, 0.0, -0.0]])
    v = v.astype(np.float32)
    assert np.array_equal(O.f32_to_f16_bits(v), v.astype(np.float16).view(np.uint16))
    bf = O.f32_to_bf16(v)
    back = O.bf16_to_f32(bf)
    # bf16 round-to-nearest-even: the error is at most half an ulp of bf16
    ulp = np.abs(back).view(np.uint32) & 0x7F800000
    assert np.all(np.abs(back - v) <= np.maximum(ulp.view(np.float32) * 2.0 ** -8, 1e-38))


# ---------------------------------------------------------------- GGUF K-quants
GOLDEN_K = os.path.join(os.path.dirname(__file__), "golden", "gguf_q4_k_q6_k.npz")


@pytest.mark.parametrize("name,qt", [("q4_k", O.Q4_K), ("q6_k", O.Q6_K)])
def test_gguf_k_dequantize_bit_exact(name, qt):
    """The oracle's Q4_K / Q6_K dequantisers equal gguf-py's bit for bit on seeded
    blocks and edge blocks (all-ones bytes, zero, subnormal and large scales)."""
    g = np.load(GOLDEN_K)
    blocks = g[f"{name}_blocks"]
    N, K = g[f"{name}_dequant"].shape
    w = O.gguf_k_dequantize(blocks, qt, N, K)
    assert np.array_equal(w.view(np.uint32), g[f"{name}_dequant"].view(np.uint32))


@pytest.mark.parametrize("name,qt", [("q4_k", O.Q4_K), ("q6_k", O.Q6_K)])
def test_gguf_k_linear_exact_matches_fixture(name, qt):
    g = np.load(GOLDEN_K)
    N = g[f"{name}_dequant"].shape[0]
    y = O.gguf_k_linear_exact(g["x"], g[f"{name}_blocks"], qt, N)
    ref = g[f"{name}_linear_f64"]
    assert np.abs(y - ref).max() <= 1e-12 * np.abs(ref).max()


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q6_K])
def test_gguf_k_random_blocks_are_finite(qt):
    rng = np.random.default_rng(3)
    b = O.gguf_k_random_blocks(rng, qt, 16, 1024)
    assert b.shape == (16, 4 * O.K_BLOCK_BYTES[qt])
    w = O.gguf_k_dequantize(b, qt, 16, 1024)
    assert np.isfinite(w).all() and np.abs(w).max() < 10.0


@pytest.mark.parametrize("name,qt", [("q4_k", O.Q4_K), ("q6_k", O.Q6_K)])
def test_gguf_k_candle_style_linear_near_exact(name, qt):
    """The CPU QMatMul arithmetic (activations quantised to Q8_K, integer
    sub-block dots) stays within its activation-rounding error of the exact
    product: 1e-2 on seeded blocks, 2.5e-2 on the golden edge rows."""
    g = np.load(GOLDEN_K)
    N = g[f"{name}_dequant"].shape[0]
    y = O.gguf_k_linear_candle(g["x"], g[f"{name}_blocks"], qt, N)
    ref = g[f"{name}_linear_f64"]
    assert np.abs(y - ref).max() <= 2.5e-2 * np.abs(ref).max()
    rng = np.random.default_rng(17)
    blocks = O.gguf_k_random_blocks(rng, qt, 300, 4096)
    x = rng.normal(0.0, 1.0, (3, 4096)).astype(np.float32)
    x[1] = 0.0  # an all-zero activation row quantises to d = 0
    yc = O.gguf_k_linear_candle(x, blocks, qt, 300)
    ye = O.gguf_k_linear_exact(x, blocks, qt, 300)
    assert np.abs(yc - ye).max() <= 1e-2 * np.abs(ye).max()
    assert np.all(yc[1] == 0.0)

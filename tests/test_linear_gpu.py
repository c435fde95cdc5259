"""GPU parity of the quantised linears against the CPU oracle, through the C ABI.

Bars (from the north star): dequantised weights and quantised bytes
bit-exact; linear outputs within max relative error 1e-2 (max |y - y_ref| /
max |y_ref|) with f32 accumulation.  The W8A16 kernels compute the same f32
sums as the reference kernel (worker_w8a16.rs:158-181) in another order, and
are checked far tighter (rel 2e-3, i.e. f16 output rounding); the GGUF
integer path reproduces candle's Q8_0-activation arithmetic and is checked
against the candle-style oracle at 1e-4 and against the exact product at 1e-2.
"""
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gguf_q4_0_q8_0.npz")


def rel_err(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(y, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.fixture(scope="module")
def D():
    import dial_cuda
    return dial_cuda


@pytest.fixture(scope="module")
def torch(cuda):
    import torch as _t
    return _t


def _to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------- W8A16
@pytest.mark.parametrize("N,K", [(37, 64), (300, 4096), (1024, 12288)])
@pytest.mark.parametrize("wdt", ["f32", "f16"])
def test_w8a16_quantize_bit_exact(D, torch, N, K, wdt):
    rng = np.random.default_rng(N * 7 + K)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    w[0, :] = 0.0  # all-zero row -> scale 1
    if wdt == "f16":
        w = w.astype(np.float16)
    q_ref, s32_ref, s16_ref = O.w8a16_quantize(w)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w))
    assert np.array_equal(lin.qweight.cpu().numpy(), q_ref)
    assert np.array_equal(lin.scales.cpu().numpy().view(np.uint32), s32_ref.view(np.uint32))
    lin16 = D.W8A16Linear.from_linear("t", _to_dev(torch, w), scale_dtype=torch.float16)
    assert np.array_equal(lin16.qweight.cpu().numpy(), q_ref)
    assert np.array_equal(lin16.scales.cpu().numpy().view(np.uint16), s16_ref.view(np.uint16))
    deq = lin.dequantize().cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), O.w8a16_dequantize(q_ref, s32_ref).view(np.uint32))


def test_w8a16_reference_kat(D, torch):
    """worker_w8a16.rs:483-516 on the GPU path: max_abs < 0.04 vs dense f16."""
    idx = np.arange(37 * 64, dtype=np.float32)
    w = (np.sin(idx * np.float32(0.037)) * np.float32(0.25)
         + ((np.arange(37 * 64) % 11).astype(np.float32) - np.float32(5.0)) * np.float32(0.002))
    w16 = w.reshape(37, 64).astype(np.float16)
    lin = D.W8A16Linear.from_linear("test.linear", _to_dev(torch, w16))
    for rows in (1, 9):
        x = (np.cos(np.arange(rows * 64, dtype=np.float32) * np.float32(0.071)) * np.float32(0.5))
        x = x.astype(np.float16).reshape(1, rows, 64)
        dense = (x.astype(np.float32) @ w16.astype(np.float32).T).astype(np.float16)
        y = lin.forward(_to_dev(torch, x)).cpu().numpy()
        assert y.shape == (1, rows, 37)
        assert np.abs(dense.astype(np.float32) - y.astype(np.float32)).max() < 0.04


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 16, 17, 32, 33, 64, 130])
@pytest.mark.parametrize("xdt", ["f16", "bf16"])
@pytest.mark.parametrize("sdt", ["f32", "f16"])
def test_w8a16_linear_parity(D, torch, M, xdt, sdt):
    N, K = 1000, 2048 + 16  # odd N tail; K tail past the last 128-wide group
    rng = np.random.default_rng(M * 131 + N)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w),
                                    scale_dtype=torch.float32 if sdt == "f32" else torch.float16)
    scale_np = lin.scales.cpu().numpy()
    if xdt == "f16":
        xh = x.astype(np.float16)
        y_ref, _ = O.w8a16_linear(xh, lin.qweight.cpu().numpy(), scale_np)
        xt = _to_dev(torch, xh)
    else:
        xb = O.f32_to_bf16(x)
        y_ref, _ = O.w8a16_linear(xb, lin.qweight.cpu().numpy(), scale_np, x_is_bf16=True)
        xt = _to_dev(torch, xb.view(np.int16)).view(torch.bfloat16)
    y = lin.forward(xt).float().cpu().numpy()
    tol = 2e-3 if xdt == "f16" else 8e-3  # output rounding of f16 / bf16
    assert rel_err(y, y_ref) <= tol


@pytest.mark.parametrize("M,N,K", [(1, 16, 16384), (4, 48, 8192), (3, 100, 64), (2, 1, 4096)])
def test_w8a16_linear_streamk_shapes(D, torch, M, N, K):
    """Few tiles over a long K: one tile's K range is split across up to 64 warps
    (the arrival counter / ordered slot sum), plus K < 128 (the in-CTA split) and
    a single output row.  Repeated calls must give bit-identical outputs."""
    rng = np.random.default_rng(M * 7 + N + K)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w))
    xt = _to_dev(torch, x)
    y1 = lin.forward(xt).float().cpu().numpy()
    y2 = lin.forward(xt).float().cpu().numpy()
    y_ref, _ = O.w8a16_linear(x, lin.qweight.cpu().numpy(), lin.scales.cpu().numpy())
    assert rel_err(y1, y_ref) <= 2e-3
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(8, 4096, 12288), (8, 24576, 4096), (7, 4096, 12288)])
def test_w8a16_linear_ring_reuse_is_race_free(D, torch, M, N, K):
    """Stream-K GEMV shapes where every warp refills its shared-memory ring many
    times: a refill must not overwrite a stage before every lane has read it.
    A missing ordering showed as about one wrong 16-row tile per call; twelve
    calls must all match the oracle and each other bit for bit."""
    rng = np.random.default_rng(M * 17 + N + K)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w))
    xt = _to_dev(torch, x)
    y_ref, _ = O.w8a16_linear(x, lin.qweight.cpu().numpy(), lin.scales.cpu().numpy())
    first = None
    for _ in range(12):
        y = lin.forward(xt).float().cpu().numpy()
        assert rel_err(y, y_ref) <= 2e-3
        if first is None:
            first = y
        assert np.array_equal(first.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("M,N,K,xdt", [(1, 12288, 1024, "f16"), (2, 40000, 1024, "bf16"),
                                        (9, 4096, 1536, "f16"), (16, 2400, 1024, "bf16")])
def test_w8a16_linear_tile_cta_shapes(D, torch, M, N, K, xdt):
    """Many 16-row tiles with staged activations: whole tiles per CTA, the K
    range split over its 8 warps and reduced in shared memory -- several tile
    rounds per CTA (up to 8 for N = 40000), one or two token groups (one or two
    shared-memory rounds).  Repeated calls must give bit-identical outputs."""
    rng = np.random.default_rng(M * 11 + N + K)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w))
    if xdt == "f16":
        xin = x.astype(np.float16)
        xt = _to_dev(torch, xin)
    else:
        xin = O.f32_to_bf16(x)
        xt = _to_dev(torch, xin.view(np.int16)).view(torch.bfloat16)
    y1 = lin.forward(xt).float().cpu().numpy()
    y2 = lin.forward(xt).float().cpu().numpy()
    assert D.lib().dial_device_error(1) == 0
    y_ref, _ = O.w8a16_linear(xin, lin.qweight.cpu().numpy(), lin.scales.cpu().numpy(),
                              x_is_bf16=(xdt == "bf16"))
    assert rel_err(y1, y_ref) <= (2e-3 if xdt == "f16" else 8e-3)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))


@pytest.mark.parametrize("amax", [3e4, 1e6, 2.0**-20])
def test_w8a16_bf16_activation_range(D, torch, amax):
    """bf16 activations far outside the f16 range (and tiny ones) on the decode
    path, which stages them as f16 under a per-token power-of-two scale."""
    rng = np.random.default_rng(int(amax) % 1000 + 5)
    N, K = 512, 4096
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (2, K)).astype(np.float32)
    x *= amax / np.abs(x).max(axis=1, keepdims=True)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w))
    xb = O.f32_to_bf16(x)
    y_ref, _ = O.w8a16_linear(xb, lin.qweight.cpu().numpy(), lin.scales.cpu().numpy(), x_is_bf16=True)
    y = lin.forward(_to_dev(torch, xb.view(np.int16)).view(torch.bfloat16)).float().cpu().numpy()
    assert np.isfinite(y).all()
    assert rel_err(y, y_ref) <= 8e-3


def test_w8a16_decode_config1_shape(D, torch):
    """The up-proj decode shape: x f16 [1,4096] ~N(0,1), W [12288,4096] ~N(0,0.02), f16 scale."""
    rng = np.random.default_rng(299792458)
    w = rng.normal(0, 0.02, (12288, 4096)).astype(np.float32)
    x = rng.normal(0, 1, (1, 4096)).astype(np.float16)
    lin = D.W8A16Linear.from_linear("up", _to_dev(torch, w), scale_dtype=torch.float16)
    y = lin.forward(_to_dev(torch, x)).float().cpu().numpy()
    y_ref, _ = O.w8a16_linear(x, lin.qweight.cpu().numpy(), lin.scales.cpu().numpy())
    assert rel_err(y, y_ref) <= 2e-3


# ---------------------------------------------------------------- GGUF
@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name,qt", [("q4_0", O.Q4_0), ("q8_0", O.Q8_0)])
def test_gguf_golden_roundtrip_and_dequant(D, torch, golden, name, qt):
    w = golden["w"]
    N, K = w.shape
    blocks = golden[f"{name}_blocks"]
    lin = D.GgufLinear.from_blocks(_to_dev(torch, blocks), qt, K, N)
    assert np.array_equal(lin.to_blocks().cpu().numpy(), blocks.reshape(-1))
    deq = lin.dequantize().cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), golden[f"{name}_dequant"].view(np.uint32))
    # GPU quantiser from the f32 weights gives the gguf package's bytes
    lq = D.GgufLinear.quantize(_to_dev(torch, w), qt)
    assert np.array_equal(lq.to_blocks().cpu().numpy(), blocks.reshape(-1))


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("K", [96, 4096, 12288])
def test_gguf_quantize_dequant_random(D, torch, qt, K):
    rng = np.random.default_rng(K + qt)
    w = rng.normal(0, 0.02, (70, K)).astype(np.float32)
    blocks = O.gguf_quantize(w, qt)
    lq = D.GgufLinear.quantize(_to_dev(torch, w), qt)
    assert np.array_equal(lq.to_blocks().cpu().numpy(), blocks.reshape(-1))
    deq = lq.dequantize().cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), O.gguf_dequantize(blocks, qt, 70, K).view(np.uint32))


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 32, 33, 512])
@pytest.mark.parametrize("xdt", ["f32", "f16", "bf16"])
def test_gguf_linear_parity(D, torch, qt, M, xdt):
    N, K = 1030, 4096 + 96  # row tail, and a K that ends in a partial group
    rng = np.random.default_rng(M * 17 + qt)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    blocks = O.gguf_quantize(w, qt)
    lin = D.GgufLinear.from_blocks(_to_dev(torch, blocks), qt, K, N)
    if xdt == "f32":
        xin, xt, bf = x, _to_dev(torch, x), False
    elif xdt == "f16":
        xin = x.astype(np.float16)
        xt, bf = _to_dev(torch, xin), False
    else:
        xin = O.f32_to_bf16(x)
        xt, bf = _to_dev(torch, xin.view(np.int16)).view(torch.bfloat16), True
    y = lin.forward(xt).float().cpu().numpy()
    exact = O.gguf_linear_exact(xin, blocks, qt, N, x_is_bf16=bf)
    out_tol = {"f32": 0.0, "f16": 1e-3, "bf16": 8e-3}[xdt]
    assert rel_err(y, exact) <= 1e-2 + out_tol
    if M <= 16 or K % 64:  # the integer (candle-arithmetic) path
        cand = O.gguf_linear_candle(xin, blocks, qt, N, x_is_bf16=bf)
        assert rel_err(y, cand) <= 1e-4 + out_tol


# BASELINE config 2's sweep: the 7 linears of an 8B decoder layer (q, k, v, o,
# gate, up: K = 4096; down: K = 12288), N(0, 0.02) weights, f32 N(0, 1)
# activations, M in {1, 8, 32, 512}.  Rows are independent, so at M = 512 the
# oracle checks 8 of them (first, last and seeded others) of the full launch.
CONFIG2_LINEARS = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
                   ("gate", 12288, 4096), ("up", 12288, 4096), ("down", 4096, 12288)]


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("M", [1, 8, 32, 512])
def test_gguf_config2_sweep_as_a_set(D, torch, qt, M):
    rng = np.random.default_rng(1000 + M + qt)
    rows = np.arange(M) if M <= 32 else np.unique(np.r_[0, M - 1, rng.choice(M, 6, replace=False)])
    for name, N, K in CONFIG2_LINEARS:
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        x = rng.normal(0, 1, (M, K)).astype(np.float32)
        blocks = O.gguf_quantize(w, qt)
        lin = D.GgufLinear.from_blocks(_to_dev(torch, blocks), qt, K, N)
        y = lin.forward(_to_dev(torch, x)).float().cpu().numpy()[rows]
        exact = O.gguf_linear_exact(x[rows], blocks, qt, N)
        assert rel_err(y, exact) <= 1e-2, (name, M)
        if M <= 16:  # the integer path reproduces candle's arithmetic
            cand = O.gguf_linear_candle(x[rows], blocks, qt, N)
            assert rel_err(y, cand) <= 1e-4, (name, M)
    assert D.lib().dial_device_error(1) == 0


def test_gguf_rejects_missing_workspace(D, torch):
    w = torch.zeros((64, 64), dtype=torch.float32, device="cuda")
    lin = D.GgufLinear.quantize(w, O.Q4_0)
    x = torch.zeros((1, 64), dtype=torch.float32, device="cuda")
    y = torch.empty((1, 64), dtype=torch.float32, device="cuda")
    st = D.lib().dial_gguf_linear(x.data_ptr(), D.F32, lin.qs.data_ptr(), lin.d.data_ptr(), D.Q4_0,
                                  y.data_ptr(), 1, 64, 64, None, 0, D.stream_ptr())
    assert st == 1


# ---------------------------------------------------------------- tcgen05 GEMM path (M > 32)
@pytest.mark.parametrize("M,N,K", [(33, 256, 64), (128, 512, 4096), (200, 1000, 1024),
                                   (512, 4096, 4096), (300, 12288, 192)])
@pytest.mark.parametrize("xdt", ["f16", "bf16"])
def test_w8a16_gemm_parity(D, torch, M, N, K, xdt):
    rng = np.random.default_rng(M + N + K)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    lin = D.W8A16Linear.from_linear("t", _to_dev(torch, w))
    if xdt == "f16":
        xin = x.astype(np.float16)
        xt = _to_dev(torch, xin)
    else:
        xin = O.f32_to_bf16(x)
        xt = _to_dev(torch, xin.view(np.int16)).view(torch.bfloat16)
    y = lin.forward(xt).float().cpu().numpy()
    assert D.lib().dial_device_error(1) == 0
    y_ref, _ = O.w8a16_linear(xin, lin.qweight.cpu().numpy(), lin.scales.cpu().numpy(),
                              x_is_bf16=(xdt == "bf16"))
    assert rel_err(y, y_ref) <= (2e-3 if xdt == "f16" else 8e-3)


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("M,N,K", [(64, 512, 4096), (512, 1024, 4096), (130, 300, 12288 + 64),
                                   (24, 1030, 4096), (32, 2048, 4160), (17, 28672, 4096)])
@pytest.mark.parametrize("xdt", ["f32", "f16", "bf16"])
def test_gguf_gemm_parity(D, torch, qt, M, N, K, xdt):
    rng = np.random.default_rng(M * 3 + N + qt)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    blocks = O.gguf_quantize(w, qt)
    lin = D.GgufLinear.from_blocks(_to_dev(torch, blocks), qt, K, N)
    if xdt == "f32":
        xin, xt, bf = x, _to_dev(torch, x), False
    elif xdt == "f16":
        xin = x.astype(np.float16)
        xt, bf = _to_dev(torch, xin), False
    else:
        xin = O.f32_to_bf16(x)
        xt, bf = _to_dev(torch, xin.view(np.int16)).view(torch.bfloat16), True
    y = lin.forward(xt).float().cpu().numpy()
    assert D.lib().dial_device_error(1) == 0
    exact = O.gguf_linear_exact(xin, blocks, qt, N, x_is_bf16=bf)
    # f16 operands (weights d*q and f32 activations rounded once) or bf16 operands
    tol = {"f32": 2e-3, "f16": 2e-3, "bf16": 1e-2}[xdt]
    assert rel_err(y, exact) <= tol

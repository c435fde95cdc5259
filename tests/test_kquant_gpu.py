"""GGUF Q4_K / Q6_K on the GPU through the C ABI, against the oracle.

Bars: dequantised weights bit-exact (f32, and the f16 / bf16 roundings of the
f32 values); linear outputs within max relative error (max |y - y_ref| /
max |y_ref|) 1e-4 in f32 and 1e-2 in f16 / bf16 of the exact f64 product on
the same dequantised weights (the kernel sums f32 products in another order
and rounds once to the activation dtype).
"""
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN_K = os.path.join(os.path.dirname(__file__), "golden", "gguf_q4_k_q6_k.npz")
TYPES = [("q4_k", O.Q4_K), ("q6_k", O.Q6_K)]


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


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _lin(D, torch, blocks, qt, N, K):
    return D.GgufKLinear.from_blocks(_dev(torch, blocks.reshape(-1)), qt, K, N)


@pytest.mark.parametrize("name,qt", TYPES)
def test_k_dequantize_golden_bit_exact(D, torch, name, qt):
    g = np.load(GOLDEN_K)
    ref = g[f"{name}_dequant"]
    N, K = ref.shape
    lin = _lin(D, torch, g[f"{name}_blocks"], qt, N, K)
    w = lin.dequantize(torch.float32).cpu().numpy()
    assert np.array_equal(w.view(np.uint32), ref.view(np.uint32))
    w16 = lin.dequantize(torch.float16).cpu().numpy()
    with np.errstate(over="ignore"):
        assert np.array_equal(w16.view(np.uint16), ref.astype(np.float16).view(np.uint16))
    wb = lin.dequantize(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(wb, O.f32_to_bf16(ref))


@pytest.mark.parametrize("name,qt", TYPES)
@pytest.mark.parametrize("N,K", [(300, 4096), (1030, 14336)])
def test_k_dequantize_random_bit_exact(D, torch, name, qt, N, K):
    rng = np.random.default_rng(N + K + qt)
    blocks = O.gguf_k_random_blocks(rng, qt, N, K)
    lin = _lin(D, torch, blocks, qt, N, K)
    w = lin.dequantize(torch.float32).cpu().numpy()
    assert np.array_equal(w.view(np.uint32), O.gguf_k_dequantize(blocks, qt, N, K).view(np.uint32))


@pytest.mark.parametrize("name,qt", TYPES)
def test_k_linear_golden(D, torch, name, qt):
    g = np.load(GOLDEN_K)
    N, K = g[f"{name}_dequant"].shape
    lin = _lin(D, torch, g[f"{name}_blocks"], qt, N, K)
    y = lin.forward(_dev(torch, g["x"])).cpu().numpy()
    assert rel_err(y, g[f"{name}_linear_f64"]) < 1e-4


@pytest.mark.parametrize("name,qt", TYPES)
@pytest.mark.parametrize("M", [1, 2, 3, 8, 9, 17, 32])
@pytest.mark.parametrize("xdt", ["f32", "f16", "bf16"])
def test_k_linear_parity(D, torch, name, qt, M, xdt):
    N, K = 1030, 4096
    rng = np.random.default_rng(M * 31 + qt)
    blocks = O.gguf_k_random_blocks(rng, qt, N, K)
    x = rng.normal(0.0, 1.0, (M, K)).astype(np.float32)
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[xdt]
    xt = _dev(torch, x).to(tdt)
    x_used = xt.float().cpu().numpy()  # the activations the kernel sees
    ref = O.gguf_k_linear_exact(x_used, blocks, qt, N)
    y = _lin(D, torch, blocks, qt, N, K).forward(xt).float().cpu().numpy()
    assert y.shape == (M, N)
    assert rel_err(y, ref) < (1e-4 if xdt == "f32" else 1e-2)


@pytest.mark.parametrize("name,qt", TYPES)
def test_k_linear_llama_shapes_and_repeat(D, torch, name, qt):
    """Llama-3-8B linear shapes (down projection K = 14336, an output head
    slice) at decode M = 1; two calls give identical bytes."""
    rng = np.random.default_rng(7 + qt)
    for N, K in ((4096, 14336), (8192, 4096)):
        blocks = O.gguf_k_random_blocks(rng, qt, N, K)
        x = rng.normal(0.0, 1.0, (1, K)).astype(np.float16)
        lin = _lin(D, torch, blocks, qt, N, K)
        xt = _dev(torch, x)
        y1 = lin.forward(xt)
        y2 = lin.forward(xt)
        assert torch.equal(y1, y2)
        ref = O.gguf_k_linear_exact(x.astype(np.float32), blocks, qt, N)
        assert rel_err(y1.float().cpu().numpy(), ref) < 1e-2


def test_text_linear_dispatches_k_quants(D, torch):
    rng = np.random.default_rng(11)
    blocks = O.gguf_k_random_blocks(rng, O.Q4_K, 64, 512)
    t = D.TextLinear.from_gguf("blk.0.ffn_down", _dev(torch, blocks.reshape(-1)), O.Q4_K, 512, 64)
    assert isinstance(t.inner, D.GgufKLinear)
    x = rng.normal(0.0, 1.0, (2, 512)).astype(np.float32)
    y = t(_dev(torch, x)).cpu().numpy()
    assert rel_err(y, O.gguf_k_linear_exact(x, blocks, O.Q4_K, 64)) < 1e-4


@pytest.mark.parametrize("qt,N,K,M", [(O.Q4_K, 1030, 2304, 5), (O.Q4_K, 4096, 4096, 8),
                                      (O.Q4_K, 100, 2048, 7), (O.Q4_K, 16, 14336, 1),
                                      (O.Q6_K, 1030, 6144, 5), (O.Q6_K, 4096, 4096, 8),
                                      (O.Q6_K, 100, 2048, 7), (O.Q6_K, 16, 14336, 1)])
@pytest.mark.parametrize("xdt", ["f16", "bf16"])
def test_k_quant_tensor_core_gemv_shapes(D, torch, qt, N, K, M, xdt):
    """The Q4_K / Q6_K tensor-core GEMVs (M <= 8, f16/bf16): uneven super-block
    counts per warp (Q4_K K = 2304: 9 super-blocks over 8 warps), every 2-byte
    offset of a Q6_K block inside its 16-byte-aligned box (K = 6144: 24 blocks
    per row), a 6-row tile tail, the smallest K each takes, one tile, and
    repeated calls give identical bytes."""
    rng = np.random.default_rng(N + K + M + qt)
    blocks = O.gguf_k_random_blocks(rng, qt, N, K)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[xdt]
    xt = _dev(torch, rng.normal(0.0, 1.0, (M, K)).astype(np.float32)).to(tdt)
    lin = _lin(D, torch, blocks, qt, N, K)
    y1 = lin.forward(xt)
    y2 = lin.forward(xt)
    assert torch.equal(y1, y2)
    ref = O.gguf_k_linear_exact(xt.float().cpu().numpy(), blocks, qt, N)
    assert rel_err(y1.float().cpu().numpy(), ref) < 1e-2
    assert D.lib().dial_device_error(1) == 0


@pytest.mark.parametrize("M,N,K", [(9, 1030, 4096), (32, 2048, 4096), (33, 1030, 4096),
                                   (128, 512, 2048), (512, 1030, 4096), (64, 4096, 14336)])
@pytest.mark.parametrize("xdt", ["f16", "bf16"])
@pytest.mark.parametrize("name,qt", TYPES)
def test_k_quant_prefill_gemm(D, torch, name, qt, M, N, K, xdt):
    """Prefill-sized Q4_K / Q6_K linears run on the tcgen05 GEMM, each
    super-block dequantised once per token tile (GGML's values rounded to the
    activation dtype; Q6_K blocks at every 2-byte offset of their boxes):
    against the exact oracle, and against the dequantised copy times x (the
    reference's f16 prefill route) in f32."""
    rng = np.random.default_rng(M + N + K + qt)
    blocks = O.gguf_k_random_blocks(rng, qt, N, K)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[xdt]
    xt = _dev(torch, rng.normal(0.0, 1.0, (M, K)).astype(np.float32)).to(tdt)
    lin = _lin(D, torch, blocks, qt, N, K)
    y = lin.forward(xt)
    assert D.lib().dial_device_error(1) == 0
    yf = y.float().cpu().numpy()
    ref = O.gguf_k_linear_exact(xt.float().cpu().numpy(), blocks, qt, N)
    assert rel_err(yf, ref) < 1e-2
    wcopy = lin.dequantize(tdt).float()  # the values the GEMM multiplies
    dense = (xt.float() @ wcopy.t()).cpu().numpy()
    assert rel_err(yf, dense) < (2e-3 if xdt == "f16" else 8e-3)
    assert torch.equal(y, lin.forward(xt))  # repeat: identical bytes

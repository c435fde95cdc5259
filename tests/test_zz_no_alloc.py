"""dial_gguf_linear_noalloc: the GGUF linear for callers that cannot allocate.

Some callers of this library cannot allocate device memory when they run a
linear (an allocator that is not re-entrant from their request loop, an FFI
host without a device allocator).  dial_gguf_linear_noalloc keeps its scratch
in a fixed array inside the library instead of a caller workspace.  This test
calls it through the C ABI and checks that two calls in a row give what the
workspace-taking dial_gguf_linear gives, within the tolerance the integer-path
parity tests use (1e-4 of the largest output), and what the oracle's candle
arithmetic gives; that the array is used up to its limit (K = 16384, rows in
more than one 32-row pass, f16 and bf16 outputs); and that K beyond its limit
is refused with a message.  It runs last (file name) and also passes alone.
"""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.abs(a.astype(np.float64) - b.astype(np.float64)).max()
                 / max(np.abs(b.astype(np.float64)).max(), 1e-30))


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_noalloc_matches_workspace_entry_point(cuda, qt):
    import torch

    import dial_cuda as D
    L = D.lib()
    rng = np.random.default_rng(4242 + qt)
    N, K = 1000, 4096
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    blocks = O.gguf_quantize(w, qt)
    lin = D.GgufLinear.from_blocks(torch.from_numpy(blocks).cuda(), qt, K, N)
    stream = D.stream_ptr()
    for call, M in enumerate((3, 40)):  # two calls in a row (the second spans two 32-row passes)
        x = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).cuda()
        ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
        out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        need = L.dial_gguf_linear_workspace_bytes(M, K, N)
        ws = torch.zeros(need, dtype=torch.uint8, device="cuda")  # zero-filled before first use
        # the workspace-taking entry point on the same integer path (at most 16 rows
        # per call: from 17 rows it takes the tensor-core GEMM)
        for m0 in range(0, M, 16):
            mc = min(16, M - m0)
            st = L.dial_gguf_linear(x[m0:].data_ptr(), D.F32, lin.qs.data_ptr(), lin.d.data_ptr(),
                                    qt, ref[m0:].data_ptr(), mc, K, N, ws.data_ptr(), need, stream)
            assert st == 0, L.dial_last_error()
        st = L.dial_gguf_linear_noalloc(x.data_ptr(), D.F32, lin.qs.data_ptr(), lin.d.data_ptr(),
                                        qt, out.data_ptr(), M, K, N, stream)
        assert st == 0, L.dial_last_error()
        torch.cuda.synchronize()
        got, want = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: unwritten outputs"
        assert _rel(got, want) <= 1e-4, f"call {call}"
        assert _rel(got, O.gguf_linear_candle(x.cpu().numpy(), blocks, qt, N)) <= 1e-4, f"call {call}"


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_noalloc_full_scratch_half_outputs(cuda, act):
    """K = 16384 fills the fixed array exactly (128 groups x 32 rows); 40 rows
    take two passes, whose f16/bf16 outputs land 32 rows apart."""
    import torch

    import dial_cuda as D
    L = D.lib()
    qt = O.Q4_0
    rng = np.random.default_rng(77 if act == "f16" else 78)
    N, K, M = 256, 16384, 40
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    blocks = O.gguf_quantize(w, qt)
    lin = D.GgufLinear.from_blocks(torch.from_numpy(blocks).cuda(), qt, K, N)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[act]
    code = {"f16": D.F16, "bf16": D.BF16}[act]
    x = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).cuda().to(tdt)
    xh = x.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = O.gguf_linear_candle(xh.view(np.float16) if act == "f16" else xh, blocks, qt, N,
                               x_is_bf16=act == "bf16")
    stream = D.stream_ptr()
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=tdt, device="cuda")
        st = L.dial_gguf_linear_noalloc(x.data_ptr(), code, lin.qs.data_ptr(), lin.d.data_ptr(), qt,
                                        out.data_ptr(), M, K, N, stream)
        assert st == 0, L.dial_last_error()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: unwritten outputs"
        # the oracle's f32 result against the output rounded to the activation type
        assert _rel(got, ref) <= {"f16": 2e-3, "bf16": 8e-3}[act], f"call {call}"


def test_noalloc_rejects_k_beyond_its_scratch(cuda):
    import dial_cuda as D
    L = D.lib()
    fake = ctypes.c_void_p(0x1000)  # rejected before any use
    st = L.dial_gguf_linear_noalloc(fake, D.F32, fake, fake, D.Q4_0, fake, 1, 16384 + 32, 64, None)
    assert st == 4
    assert b"K <= 16384" in L.dial_last_error()

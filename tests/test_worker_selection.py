"""The worker W8A16 switch (configure_worker_w8a16_from_args, worker_w8a16.rs:15-44)
and TextLinear.from_dense's use of it (worker_w8a16.rs:78-101).

Enabled iff requested && no GGUF source && worker mode && a CUDA device && f16;
the message for each disabled case follows the reference's order of checks.
"""
import pytest

import dial_cuda as D


@pytest.fixture(autouse=True)
def _reset():
    yield
    D.configure_worker_w8a16_from_args(False, False, "cpu", "f16")


@pytest.mark.parametrize("requested,gguf,worker,device,dtype,enabled,msg", [
    (True, False, True, "cuda:0", "f16", True, "worker W8A16 enabled"),
    (True, True, True, "cuda:0", "f16", False, "GGUF takes precedence"),
    (True, False, False, "cuda:0", "f16", False, "ignored in master mode"),
    (True, False, True, "cpu", "f16", False, "non-CUDA device"),
    (True, False, True, "cuda:0", "bf16", False, "requires --dtype f16"),
    (True, False, True, "cuda:0", "f32", False, "requires --dtype f16"),
    (False, False, True, "cuda:0", "f16", False, ""),
    (False, True, False, "cpu", "bf16", False, ""),
    # GGUF is reported first even when other conditions also fail (worker_w8a16.rs:27)
    (True, True, False, "cpu", "bf16", False, "GGUF takes precedence"),
    (True, False, False, "cpu", "f16", False, "ignored in master mode"),
])
def test_switch(requested, gguf, worker, device, dtype, enabled, msg):
    got = D.configure_worker_w8a16_from_args(requested, worker, device, dtype, gguf_enabled=gguf)
    assert D.worker_w8a16_enabled() is enabled
    assert (msg in got) if msg else got == ""
    if not enabled:
        assert D.worker_w8a16_summary() is None


def test_torch_dtype_and_device_objects():
    torch = pytest.importorskip("torch")
    assert D.configure_worker_w8a16_from_args(True, True, torch.device("cuda", 0), torch.float16)
    assert D.worker_w8a16_enabled()
    D.configure_worker_w8a16_from_args(True, True, torch.device("cuda", 0), torch.bfloat16)
    assert not D.worker_w8a16_enabled()


def test_from_dense_keeps_the_callers_dense_module_when_disabled():
    D.configure_worker_w8a16_from_args(True, True, "cpu", "f16")  # non-CUDA: disabled

    class Dense:
        def forward(self, x, out=None):
            return ("dense", x)

    t = D.TextLinear.from_dense("model.layers.0.mlp.up_proj", weight=None, dense=Dense())
    assert t(7) == ("dense", 7)
    with pytest.raises(RuntimeError, match="not enabled"):
        D.TextLinear.from_dense("model.layers.0.mlp.up_proj", weight=None)


@pytest.mark.gpu
def test_from_dense_converts_and_counts_when_enabled(cuda):
    import numpy as np
    import torch

    import oracle as O
    D.configure_worker_w8a16_from_args(True, True, cuda, torch.float16)
    assert D.worker_w8a16_summary() == (0, 0)
    w = np.random.default_rng(3).normal(0, 0.02, (96, 256)).astype(np.float32)
    t = D.TextLinear.from_dense("up_proj", torch.from_numpy(w).cuda())
    assert isinstance(t.inner, D.W8A16Linear)
    assert D.worker_w8a16_summary() == (1, 96 * 256 + 96 * 4)
    q, s, _ = O.w8a16_quantize(w)
    assert np.array_equal(t.inner.qweight.cpu().numpy(), q)
    assert np.array_equal(t.inner.scales.cpu().numpy(), s)

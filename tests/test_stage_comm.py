"""The stage hand-off's C ABI (dial_stage_comm_*).

CPU: clique ids, argument checks, and that a machine without a usable GPU gets
an error status.  GPU (one device): a one-rank communicator initialises and
tears down; a two-rank communicator whose peer never joins gives
DIAL_ERR_TIMEOUT within its host deadline (the failure is made on the host: a
rank that never arrives), after which the library still works.  The two-GPU
transfer path is covered by tests/test_pipeline_gpu.py (two-stage pipeline over
these communicators).
"""
import ctypes
import time

import pytest

DIAL_ERR_INVALID_ARG, DIAL_ERR_CUDA, DIAL_ERR_TIMEOUT = 1, 5, 7


@pytest.fixture(scope="module")
def D():
    # torch first: its NCCL is then the one in the process, and the library
    # reuses it (a later torch import next to another libnccl.so.2 would fail)
    import torch  # noqa: F401

    import dial_cuda
    return dial_cuda


def _uid(D):
    buf = (ctypes.c_uint8 * D.ID_BYTES)()
    assert D.lib().dial_stage_comm_unique_id(buf) == 0, D.lib().dial_last_error()
    return buf


def test_unique_ids_differ(D):
    a, b = bytes(_uid(D)), bytes(_uid(D))
    assert len(a) == 128 and a != b and any(a)


def test_argument_checks(D):
    L = D.lib()
    comm = ctypes.c_void_p()
    uid = _uid(D)
    assert L.dial_stage_comm_unique_id(None) == DIAL_ERR_INVALID_ARG
    assert L.dial_stage_comm_init(None, 0, 2, 0, 1.0, ctypes.byref(comm)) == DIAL_ERR_INVALID_ARG
    assert L.dial_stage_comm_init(uid, 2, 2, 0, 1.0, ctypes.byref(comm)) == DIAL_ERR_INVALID_ARG
    assert b"out of range" in L.dial_last_error()
    assert L.dial_stage_comm_init(uid, 0, 2, 0, 0.0, ctypes.byref(comm)) == DIAL_ERR_INVALID_ARG
    assert L.dial_stage_comm_send(None, None, 0, 0, None) == DIAL_ERR_INVALID_ARG
    assert L.dial_stage_comm_recv(None, None, 0, 0, None) == DIAL_ERR_INVALID_ARG
    assert L.dial_stage_comm_wait(None, None) == DIAL_ERR_INVALID_ARG
    assert L.dial_stage_comm_destroy(None) == 0


def test_init_without_a_gpu_fails_cleanly(D):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    comm = ctypes.c_void_p()
    assert D.lib().dial_stage_comm_init(_uid(D), 0, 1, 0, 1.0, ctypes.byref(comm)) == DIAL_ERR_CUDA
    assert not comm.value


@pytest.mark.gpu
def test_single_rank_communicator(D, cuda):
    L = D.lib()
    comm = ctypes.c_void_p()
    assert L.dial_stage_comm_init(_uid(D), 0, 1, 0, 30.0, ctypes.byref(comm)) == 0, L.dial_last_error()
    assert comm.value
    assert L.dial_stage_comm_wait(comm, None) == 0, L.dial_last_error()
    assert L.dial_stage_comm_destroy(comm) == 0, L.dial_last_error()


@pytest.mark.gpu
def test_missing_peer_times_out(D, cuda):
    """Rank 0 of a two-rank link whose rank 1 never joins: the bounded
    initialisation returns DIAL_ERR_TIMEOUT instead of hanging."""
    import torch
    L = D.lib()
    comm = ctypes.c_void_p()
    t0 = time.monotonic()
    st = L.dial_stage_comm_init(_uid(D), 0, 2, 0, 1.0, ctypes.byref(comm))
    assert st == DIAL_ERR_TIMEOUT, (st, L.dial_last_error())
    assert time.monotonic() - t0 < 30
    assert not comm.value
    # the process and the device are still usable
    ok = ctypes.c_void_p()
    assert L.dial_stage_comm_init(_uid(D), 0, 1, 0, 30.0, ctypes.byref(ok)) == 0, L.dial_last_error()
    assert L.dial_stage_comm_destroy(ok) == 0
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0


@pytest.mark.gpu
def test_device_wait_expires_with_a_status(cuda):
    """A device-side bounded wait that nothing signals (dial_check_bounded_wait):
    it gives up after its 1 s limit, the host reads DIAL_ERR_TIMEOUT from the
    device error flag, the copy the kernel started was drained, and the context
    still runs work afterwards."""
    import time

    import torch

    import dial_cuda as D
    D.lib().dial_device_error(1)  # start clean
    src = torch.arange(64, dtype=torch.int32, device="cuda")
    res = torch.full((3,), -7, dtype=torch.int32, device="cuda")
    t0 = time.time()
    D.check(D.lib().dial_check_bounded_wait(src.data_ptr(), res.data_ptr(), D.stream_ptr()),
            "dial_check_bounded_wait")
    torch.cuda.synchronize()
    took = time.time() - t0
    assert res.tolist() == [0, 1, 12]
    assert D.lib().dial_device_error(1) == 7  # DIAL_ERR_TIMEOUT
    assert D.lib().dial_device_error(0) == 0  # cleared
    assert 0.9 < took < 30
    assert int((src * 2).sum().item()) == 2 * sum(range(64))  # the context is usable

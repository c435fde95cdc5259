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

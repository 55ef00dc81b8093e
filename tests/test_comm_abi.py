"""The C-ABI collectives (oxc_comm_*) on the CPU: NCCL loads at run time and
makes a communicator id without a GPU; argument errors come back as the
reference's status codes before anything is launched.  The collectives
themselves run on real NCCL ranks in tests/test_gpu_sharded.py."""

import ctypes

import pytest


@pytest.fixture(scope="module")
def lib():
    from oxitorch_b200 import _native as N
    return N, N.load(require_device=False)


def test_unique_id_is_made_on_the_host(lib):
    N, L = lib
    a, b = (ctypes.c_uint8 * 128)(), (ctypes.c_uint8 * 128)()
    assert L.oxc_comm_unique_id(a) == N.OK
    assert L.oxc_comm_unique_id(b) == N.OK
    assert any(bytes(a)) and bytes(a) != bytes(b)


def test_argument_errors(lib):
    N, L = lib
    comm = ctypes.c_void_p()
    idbuf = (ctypes.c_uint8 * 128)()
    assert L.oxc_comm_init(ctypes.byref(comm), idbuf, 2, 2) == N.ERR_INVALID_ARGUMENT
    assert "rank 2 of world 2" in N.last_error()
    assert L.oxc_comm_init(ctypes.byref(comm), idbuf, 0, 0) == N.ERR_INVALID_ARGUMENT
    assert L.oxc_comm_init(None, idbuf, 1, 0) == N.ERR_INVALID_ARGUMENT
    assert L.oxc_comm_unique_id(None) == N.ERR_INVALID_ARGUMENT
    assert L.oxc_comm_allreduce_sum_f32(None, None, 4, None) == N.ERR_INVALID_ARGUMENT
    assert "null communicator" in N.last_error()
    assert L.oxc_comm_alltoallv(None, None, None, None, None, 4, None) == N.ERR_INVALID_ARGUMENT
    assert L.oxc_comm_destroy(None) == N.OK

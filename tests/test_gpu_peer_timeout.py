"""Failure detection of the peer-memory exchange on one GPU, without a fault:
every wait of the exchange kernels is bounded, and a wait that runs out writes
its kind to the group's host-mapped error word and lets its kernel finish, so
the context stays usable and the host raises (``PeerExchange.check``).

The test builds a two-rank group whose second "rank" is a plain allocation on
the same GPU that nothing ever writes: the receive waits for rows (and for
gradients) that no sender will store. The wait limit is shortened for the test
(``gsb_peer_set_wait_limit``) and restored afterwards."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture
def group():
    from gsplat_b200.cuda import _backend as B

    lib = B.lib()
    torch.cuda.set_device(DEV)
    err_host = ctypes.POINTER(ctypes.c_int)()
    err_dev = ctypes.c_void_p()
    B.call("gsb_peer_error_alloc", ctypes.byref(err_host), ctypes.byref(err_dev))
    mb = lib.gsb_peer_mailbox_bytes()
    size = mb + 3 * 65536
    arenas = []
    for _ in range(2):
        p = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        B.call("gsb_peer_alloc", ctypes.c_size_t(size), ctypes.byref(p), handle)
        arenas.append(p)
    g = B.GsbPeerGroup()
    for r, p in enumerate(arenas):
        g.arena[r] = p.value
    g.recv_offset, g.recv_stride, g.grad_offset = mb, 65536, mb + 2 * 65536
    g.rank, g.world = 0, 2
    g.error = err_dev.value
    prev = B.call("gsb_peer_set_wait_limit", 4096)  # polls: milliseconds, not seconds
    try:
        yield B, g, err_host
    finally:
        torch.cuda.synchronize(DEV)
        B.call("gsb_peer_set_wait_limit", prev)
        for p in arenas:
            B.call("gsb_peer_free", p)
        B.call("gsb_peer_error_free", err_host)


def _error_message(err_host):
    from gsplat_b200.distributed import PeerExchange

    pe = PeerExchange.__new__(PeerExchange)  # only the error-word decoding
    pe.err_host = err_host
    pe.rank = 0
    with pytest.raises(RuntimeError) as info:
        pe.check()
    return str(info.value)


def test_receive_wait_for_rows_runs_out(group):
    B, g, err_host = group
    stream = torch.cuda.current_stream(DEV).cuda_stream
    route = torch.full((2 * 2 + 1,), -1, dtype=torch.int64, device=DEV)
    nnz_recv = torch.full((1,), -1, dtype=torch.int64, device=DEV)
    n_world = torch.tensor([1, 1], dtype=torch.int64, device=DEV)
    dst = torch.zeros(4, dtype=torch.int32, device=DEV)
    dsts = (ctypes.c_void_p * 1)(dst.data_ptr())
    words = (ctypes.c_int * 1)(1)
    assert err_host[0] == 0
    rc = B.call("gsb_peer_recv_rows", ctypes.byref(g), 1, 1, route.data_ptr(), nnz_recv.data_ptr(),
                n_world.data_ptr(), 1, 2, 1, dsts, words, stream)
    assert rc == 0  # launched; the failure is reported by the kernel, not the launch
    torch.cuda.synchronize(DEV)  # returns: the wait is bounded
    assert err_host[0] == 2  # "a source's rows did not arrive"
    assert int(nnz_recv.item()) == 0 and bool((route[:3] == 0).all())
    assert "rows did not arrive" in _error_message(err_host)
    # the context is still usable
    assert float(torch.arange(4.0, device=DEV).sum()) == 6.0


def test_receive_wait_for_gradients_runs_out(group):
    B, g, err_host = group
    stream = torch.cuda.current_stream(DEV).cuda_stream
    nnz = torch.zeros(1, dtype=torch.int64, device=DEV)
    dst = torch.zeros(4, dtype=torch.float32, device=DEV)
    dsts = (ctypes.c_void_p * 1)(dst.data_ptr())
    words = (ctypes.c_int * 1)(1)
    rc = B.call("gsb_peer_recv_grads", ctypes.byref(g), 1, 1, nnz.data_ptr(), 1, dsts, words, stream)
    assert rc == 0
    torch.cuda.synchronize(DEV)
    assert err_host[0] == 3  # "gradients did not arrive"
    assert "gradients did not arrive" in _error_message(err_host)
    assert float(torch.ones(3, device=DEV).sum()) == 3.0

"""Device-side timeouts on ONE GPU, in the form this pool allows: a two-rank communicator whose "rank 1" region is a
second local allocation that no kernel ever writes into as rank 1. Every collective of rank 0 then waits for a peer
that never arrives; with the peer-wait bound set to 50 ms each kernel must give up, record ST_PEER_TIMEOUT (and the
waiting phase) in the communicator's status word, and return -- so the host sees the failure (vt_comm_status,
TPComm.check raising CommError) and the context stays usable. Nothing here faults, traps or spins unbounded: the
waits are the kernels' own bounded polls of flags nobody sets. The waits inside one CTA (bulk copies, MMA
completion) cannot be starved from the host this way and are not exercised here."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import rand_int8, rand_scales

pytestmark = pytest.mark.gpu

ST_PEER_TIMEOUT = 0x02000000


@pytest.fixture(scope="module")
def lonely_comm():
    """(library, communicator handle, regions) of rank 0 in a world of 2 whose rank 1 never runs."""
    from vllm_turing_b200 import _build, w8a8  # noqa: F401  (w8a8 registers the scaled_mm_ op)
    L = _build.load()
    torch.cuda.set_device(0)
    ll, big, scratch = 512 << 10, 8 << 20, 2 << 20
    size = L.vt_comm_region_bytes(2, ll, big, scratch)
    regions = []
    for _ in range(2):
        p, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        assert L.ce_alloc(size, ctypes.byref(p), h) == 0
        regions.append(p.value)
    bases = (ctypes.c_void_p * 2)(*regions)
    handle = L.vt_comm_create(0, 2, bases, ll, big, scratch)
    assert handle
    assert L.vt_set_wait_bounds(0.0, 50.0) == 0
    try:
        yield L, handle, regions
    finally:
        L.vt_set_wait_bounds(2000.0, 10000.0)
        torch.cuda.synchronize()
        L.vt_comm_destroy(handle)
        for p in regions:
            L.ce_free(p)


def _expect_timeout(L, handle, phase):
    torch.cuda.synchronize()
    st = L.vt_comm_status(handle, 1)
    assert st & 0xff000000 == ST_PEER_TIMEOUT, f"status {st:#010x}"
    assert st & 0xff == 1, f"status {st:#010x} should name rank 1"
    if phase is not None:
        assert st & 0xff00 == phase, f"status {st:#010x}: expected phase {phase:#x}"
    assert L.vt_comm_status(handle, 0) == 0, "the status word is cleared by reading with clear = 1"


@pytest.mark.parametrize("algo,phase", [(1, 0x000), (2, 0x100)])
def test_all_reduce_peer_never_arrives(lonely_comm, algo, phase):
    L, h, _ = lonely_comm
    x = torch.randn(5 * 5120, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(x)
    rc = L.vt_all_reduce(h, x.data_ptr(), out.data_ptr(), x.numel(), 1, algo, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    _expect_timeout(L, h, phase)


@pytest.mark.parametrize("M", [5, 256])
def test_fused_row_linear_peer_never_arrives(lonely_comm, M):
    """The decode tail (one kernel) and the prefill tail (GEMM + reduce kernel) of rank 0."""
    L, h, _ = lonely_comm
    N, K = 5120, 512
    a, w = rand_int8((M, K), 1).cuda(), rand_int8((N, K), 2).cuda()
    sa, sw = rand_scales(M, 3, 1e-2).cuda(), rand_scales(N, 4, 1e-3).cuda()
    res = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    nw = torch.ones(N, device="cuda", dtype=torch.bfloat16)
    q = torch.empty(M, N, dtype=torch.int8, device="cuda")
    s = torch.empty(M, dtype=torch.float32, device="cuda")
    rc = L.vt_tp_row_linear(h, a.data_ptr(), w.data_ptr(), sa.data_ptr(), sw.data_ptr(), res.data_ptr(),
                            nw.data_ptr(), 1e-6, q.data_ptr(), s.data_ptr(), None, M, N, K, 1,
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    _expect_timeout(L, h, 0x500 if M <= 32 else 0xb00)


def test_host_sees_the_failure_and_the_context_stays_usable(lonely_comm):
    from vllm_turing_b200 import w8a8
    from vllm_turing_b200.comm import CommError, TPComm
    L, h, _ = lonely_comm
    x = torch.randn(4096, device="cuda").to(torch.bfloat16)
    assert L.vt_all_reduce(h, x.data_ptr(), x.data_ptr(), x.numel(), 1, 1, torch.cuda.current_stream().cuda_stream) == 0
    view = TPComm.__new__(TPComm)   # the host-side object around this handle (no process group needed to check it)
    view.L, view.handle, view.rank = L, h, 0
    with pytest.raises(CommError):
        view.check()
    # the device still computes correctly after the timeouts
    M, N, K = 5, 2048, 512
    a, wt = rand_int8((M, K), 7), rand_int8((N, K), 8)
    sa, sw = rand_scales(M, 9, 1e-2), rand_scales(N, 10, 1e-3)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    w8a8.mma(out, a.cuda(), wt.cuda().t(), sa.cuda(), sw.cuda(), None)
    torch.cuda.synchronize()
    assert np.array_equal(O.to_bits(out.cpu()), O.scaled_mm(a.numpy(), wt.numpy(), sa.numpy(), sw.numpy(), None, 1))

"""The reference's two-rank transport entry points (har_all_reduce, ce_all_reduce, dag_all_gather; vllm_turing/csrc/
host_ar.cu:86-131, ce_ar.cu:101-146, dma_ag.cu:26-74) called through the C ABI on ONE GPU, with the peer emulated: its
side of the protocol (its LL words, its pushes and flags) is written into the buffers before the call, as the peer's
kernel would have done, so this rank's kernel finds everything it waits for and never spins on a second launch.
Checked: the result against the oracle's rank-ordered sum (bit-exact), what this rank hands the peer (its LL words /
pushed halves / staged payload and flags), and the per-block call counters over two calls (both parity slots). The
two-GPU versions, with real peers, are in test_tp_multigpu.py."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _lib():
    from vllm_turing_b200 import _build
    L = _build.load()
    assert L.har_preload() == 0
    return L


def _words(t):
    """16-bit tensor -> its 32-bit words (two elements each) as uint64 numpy."""
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32).astype(np.uint64)


@pytest.mark.parametrize("n,slot_words,dtype", [(5 * 5120, 32768, torch.bfloat16), (2 * 12345, 16385, torch.float16),
                                                (2, 64, torch.bfloat16)])
def test_har_all_reduce_emulated_peer(n, slot_words, dtype):
    L = _lib()
    dev = torch.device("cuda", 0)
    nwords = n // 2
    nb = L.har_blocks(slot_words)
    counters = torch.zeros(nb, dtype=torch.int32, device=dev)
    to_peer = torch.zeros(2 * slot_words, dtype=torch.int64, device=dev)   # this rank writes here (the peer's region)
    from_peer = torch.zeros(2 * slot_words, dtype=torch.int64, device=dev)  # the peer's words arrive here
    s = torch.cuda.current_stream().cuda_stream
    for seq in (1, 2):
        x0 = (torch.randn(n, generator=torch.Generator().manual_seed(10 * seq)) * 3).to(dtype)
        x1 = (torch.randn(n, generator=torch.Generator().manual_seed(10 * seq + 1)) * 3).to(dtype)
        slot = (seq & 1) * slot_words
        pre = (np.uint64(seq) << np.uint64(32)) | _words(x1)
        from_peer[slot:slot + nwords] = torch.from_numpy(pre.view(np.int64)).to(dev)
        out = torch.empty(n, dtype=dtype, device=dev)
        xd = x0.to(dev)
        rc = L.har_all_reduce(xd.data_ptr(), out.data_ptr(), nwords, 1 if dtype == torch.bfloat16 else 0,
                              to_peer.data_ptr(), from_peer.data_ptr(), counters.data_ptr(), slot_words, s)
        assert rc == 0
        torch.cuda.synchronize()
        assert L.vt_status(1) == 0, "a wait timed out"
        want = O.all_reduce([O.to_bits(x0), O.to_bits(x1)], 1 if dtype == torch.bfloat16 else 0)
        assert np.array_equal(O.to_bits(out.cpu()), want), f"call {seq}: sum differs from the oracle"
        sent = to_peer[slot:slot + nwords].cpu().numpy().view(np.uint64)
        assert np.array_equal(sent, (np.uint64(seq) << np.uint64(32)) | _words(x0)), "LL words handed to the peer"
        used = L.har_blocks(nwords)
        assert torch.all(counters[:used] == seq).item()
    assert L.har_all_reduce(0, 0, slot_words + 1, 1, 0, 0, 0, slot_words, s) == -1


@pytest.mark.parametrize("n", [5120 * 24, 16 * 1001])
def test_ce_all_reduce_emulated_peer(n):
    """Rank 0's call, the peer (rank 1) having pushed its copy of half 0 into R1 and its reduced half 1 into R2."""
    L = _lib()
    assert L.ce_driver_ok() == 0
    dev = torch.device("cuda", 0)
    cap = (n - n // 2) * 2 + 4096
    my = torch.zeros(256 + 2 * cap, dtype=torch.uint8, device=dev)
    peer = torch.zeros_like(my)
    h = n // 2
    for seq in (1, 2):
        x0 = (torch.randn(n, generator=torch.Generator().manual_seed(3 * seq)) * 2).half()
        x1 = (torch.randn(n, generator=torch.Generator().manual_seed(3 * seq + 1)) * 2).half()
        want = O.from_bits(O.all_reduce([O.to_bits(x0), O.to_bits(x1)], 0), torch.float16)
        my[256:256 + h * 2] = x1[:h].view(torch.uint8).to(dev)                         # the peer's push into R1
        my[256 + cap:256 + cap + (n - h) * 2] = want[h:].contiguous().view(torch.uint8).to(dev)   # its R2 push
        my[:256].view(torch.int32)[:64] = seq                                          # both flags of every slice
        out = torch.empty(n, dtype=torch.float16, device=dev)
        xd = x0.to(dev)
        rc = L.ce_all_reduce(xd.data_ptr(), out.data_ptr(), n, 0, my.data_ptr(), peer.data_ptr(), cap, seq, 8,
                             torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert L.vt_status(1) == 0, "a wait timed out"
        assert torch.equal(out.cpu().view(torch.int16), want.view(torch.int16)), f"call {seq}: sum"
        assert torch.equal(peer[256:256 + (n - h) * 2].cpu(), x0[h:].contiguous().view(torch.uint8)), "R1 push"
        assert torch.equal(peer[256 + cap:256 + cap + h * 2].cpu(), want[:h].contiguous().view(torch.uint8)), "R2 push"
        assert torch.all(peer[:256].view(torch.int32)[:64] == seq).item(), "flags"
    s = torch.cuda.current_stream().cuda_stream
    assert L.ce_all_reduce(xd.data_ptr(), out.data_ptr(), n + 8, 0, my.data_ptr(), peer.data_ptr(), cap, 3, 8, s) == 2
    assert L.ce_all_reduce(xd.data_ptr(), out.data_ptr(), n, 0, my.data_ptr(), peer.data_ptr(), 64, 3, 8, s) == 3


@pytest.mark.parametrize("m,P", [(3 << 20, 8), (4096 + 48, 3)])
def test_dag_all_gather_emulated_peer(m, P):
    """Rank 1's call through a registered host segment: [my stage | peer stage | my flags | peer flags]."""
    L = _lib()
    dev = torch.device("cuda", 0)
    size = 2 * m + 2 * 4096
    host = (ctypes.c_char * size)()
    base = ctypes.addressof(host)
    dbase = L.dag_register(base, size)
    assert dbase
    try:
        hv = np.frombuffer(host, dtype=np.uint8)
        my_stage, peer_stage = base, base + m
        my_flags, peer_flags = dbase + 2 * m, dbase + 2 * m + 4096
        for seq in (1, 2):
            mine = torch.randint(0, 256, (m,), generator=torch.Generator().manual_seed(seq), dtype=torch.uint8)
            theirs = torch.randint(0, 256, (m,), generator=torch.Generator().manual_seed(50 + seq), dtype=torch.uint8)
            hv[m:2 * m] = theirs.numpy()                                    # the peer's staged payload
            hv[2 * m + 4096:2 * m + 4096 + 4 * P].view(np.int32)[:] = seq   # and its piece flags
            g = torch.zeros(2 * m, dtype=torch.uint8, device=dev)
            g[m:] = mine.to(dev)                                            # rank 1: own payload in half 1
            s = torch.cuda.current_stream().cuda_stream
            assert L.dag_all_gather(g.data_ptr(), m, 1, my_stage, peer_stage, my_flags, peer_flags, seq, P, s,
                                    None, None, None, None, None) == 0
            torch.cuda.synchronize()
            assert L.vt_status(1) == 0, "a wait timed out"
            assert torch.equal(g[:m].cpu(), theirs), f"call {seq}: the peer's half"
            assert np.array_equal(hv[:m], mine.numpy()), f"call {seq}: staged payload"
            piece = ((m + P - 1) // P + 255) // 256 * 256
            np_ = (m + piece - 1) // piece
            assert np.all(hv[2 * m:2 * m + 4 * np_].view(np.int32) == seq), "piece flags"
    finally:
        assert L.har_unregister(base) == 0

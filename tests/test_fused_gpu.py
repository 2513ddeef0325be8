"""The fused row-linear + all-reduce + residual add + RMSNorm + int8 quant kernel (csrc/tp_fused.cu) and the
collectives of csrc/tp_comm.cu on ONE GPU (world size 1: the BASELINE config-1 "fused epilogue without collective"),
against the oracle chain. The multi-rank versions are in test_tp_multigpu.py."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist

from oracle import oracle as O
from tests.helpers import assert_bits_equal, q_off

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm1():
    from vllm_turing_b200.comm import TPComm
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29611")
        dist.init_process_group("gloo", rank=0, world_size=1)
    torch.cuda.set_device(0)
    c = TPComm(dist.group.WORLD, torch.device("cuda", 0))
    yield c
    c.close()


def _inputs(M, N, K, seed=0):
    from vllm_turing_b200.synthetic import make_layer_inputs
    return make_layer_inputs(M, N, K, seed=seed, rank=0)


@pytest.mark.parametrize("M,N,K", [(5, 5120, 17408), (1, 5120, 2176), (8, 5120, 4352), (3, 1024, 512),
                                   (16, 5120, 8704), (24, 5120, 17408), (32, 5120, 2176), (17, 1024, 5136)])
def test_fused_tp1_vs_oracle(comm1, M, N, K):
    li = _inputs(M, N, K, seed=M + K)
    res = li.residual.cuda()
    red = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    q, s = comm1.row_linear(li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), residual=res,
                            norm_w=li.norm_w.cuda(), eps=li.eps, reduced=red)
    torch.cuda.synchronize()
    comm1.check()
    ro, qo, so, redo = O.row_linear_tp([li.a.numpy()], [li.w.numpy()], [li.sa.numpy()], [li.sw.numpy()],
                                       O.to_bits(li.residual), O.to_bits(li.norm_w), li.eps, 1)
    assert_bits_equal(red, redo, "reduced")             # GEMM int32 exact + identical dequant rounding
    assert_bits_equal(res, ro, "residual")
    assert q_off(q.cpu().numpy(), qo) <= 1
    assert (q.cpu().numpy() != qo).mean() < 1e-2
    assert np.max(np.abs(s.cpu().numpy().reshape(-1) - so) / so) < 1e-2


def test_fused_plain_allreduce_mode(comm1):
    """residual = NULL: row-linear + all-reduce only."""
    M, N, K = 4, 5120, 4352
    li = _inputs(M, N, K, seed=7)
    red = comm1.row_linear(li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda())
    torch.cuda.synchronize()
    want = O.scaled_mm(li.a.numpy(), li.w.numpy(), li.sa.numpy(), li.sw.numpy(), None, 1)
    assert_bits_equal(red, want, "reduced")


def test_fused_back_to_back_and_graph(comm1):
    """30 calls without host syncs, then the same call captured in a CUDA graph and replayed: the device-side call
    counter keeps every launch on a fresh sequence number."""
    M, N, K = 5, 5120, 8704
    li = _inputs(M, N, K, seed=11)
    a, w, sa, sw, nw = li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), li.norm_w.cuda()
    res0 = li.residual.cuda()
    outs = []
    for _ in range(30):
        r = res0.clone()
        q, s = comm1.row_linear(a, w, sa, sw, residual=r, norm_w=nw, eps=1e-6)
        outs.append((r, q))
    torch.cuda.synchronize()
    comm1.check()
    for r, q in outs[1:]:
        assert torch.equal(r, outs[0][0]) and torch.equal(q, outs[0][1])
    seq0 = comm1.seq()
    r = res0.clone()
    q = torch.empty(M, N, dtype=torch.int8, device="cuda")
    s = torch.empty(M, 1, dtype=torch.float32, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        comm1.row_linear(a, w, sa, sw, residual=r, norm_w=nw, eps=1e-6, q=q, scales=s)
    for _ in range(4):
        r.copy_(res0)
        g.replay()
    torch.cuda.synchronize()
    comm1.check()
    assert comm1.seq() == seq0 + 4
    assert torch.equal(r, outs[0][0]) and torch.equal(q, outs[0][1])


@pytest.mark.parametrize("n,algo", [(5 * 5120, 1), (24 * 5120, 1), (5 * 5120, 2), (2048 * 5120, 2),
                                    (1 << 23, 0)])
def test_all_reduce_world1(comm1, n, algo):
    x = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 4).to(torch.bfloat16).cuda()
    y = comm1.all_reduce(x, algo=algo)
    torch.cuda.synchronize()
    comm1.check()
    assert torch.equal(y, x)


# ---- prefill shapes (M > 32): GEMM with the reduce-scatter in its epilogue, then reduce + row epilogue ----
@pytest.mark.parametrize("M,N,K", [(128, 5120, 4352), (256, 5120, 512), (384, 1024, 2176), (256, 2048, 1040)])
def test_prefill_fused_tp1_vs_oracle_and_chain(comm1, M, N, K):
    from vllm_turing_b200 import w8a8  # noqa: F401  (registers vllm_turing::scaled_mm_)
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant
    li = _inputs(M, N, K, seed=M + N + K)
    a, w, sa, sw, nw = li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), li.norm_w.cuda()
    res = li.residual.cuda()
    red = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    q, s = comm1.row_linear(a, w, sa, sw, residual=res, norm_w=nw, eps=li.eps, reduced=red)
    # the unfused chain on the same inputs: scaled_mm_ (prefill GEMM) -> vt_rms_norm_quant
    part = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    torch.ops.vllm_turing.scaled_mm_(part, a, w.t(), sa.view(-1, 1), sw.view(-1, 1), None)
    res_c = li.residual.cuda()
    q_c, s_c = rms_norm_dynamic_per_token_quant(part, nw, li.eps, res_c)
    torch.cuda.synchronize()
    comm1.check()
    ro, qo, so, redo = O.row_linear_tp_big([li.a.numpy()], [li.w.numpy()], [li.sa.numpy()], [li.sw.numpy()],
                                           O.to_bits(li.residual), O.to_bits(li.norm_w), li.eps, 1)
    assert_bits_equal(red, redo, "reduced")
    assert_bits_equal(res, ro, "residual")
    assert q_off(q.cpu().numpy(), qo) <= 1
    assert np.max(np.abs(s.cpu().numpy().reshape(-1) - so) / so) < 1e-2
    # the same bits as the chain (same GEMM epilogue order, same row arithmetic)
    assert torch.equal(red, part) and torch.equal(res, res_c)
    assert torch.equal(q, q_c) and torch.equal(s.view(-1), s_c.view(-1))


def test_prefill_fused_pieces_back_to_back_and_graph():
    """A communicator whose two-shot buffers hold 128 rows per piece: M = 512 runs as 4 pieces;
    20 calls without host syncs, then captured and replayed, all identical to the first."""
    from vllm_turing_b200.comm import TPComm
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29611")
        dist.init_process_group("gloo", rank=0, world_size=1)
    M, N, K = 512, 5120, 2176
    c = TPComm(dist.group.WORLD, torch.device("cuda", 0), big_bytes=128 * N * 2)
    try:
        li = _inputs(M, N, K, seed=5)
        a, w, sa, sw, nw = li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), li.norm_w.cuda()
        res0 = li.residual.cuda()
        seq0 = c.seq()
        outs = []
        for _ in range(20):
            r = res0.clone()
            q, s = c.row_linear(a, w, sa, sw, residual=r, norm_w=nw, eps=1e-6)
            outs.append((r, q, s))
        torch.cuda.synchronize()
        c.check()
        assert c.seq() == seq0   # one rank: the prefill tail exchanges nothing and takes no call numbers
        ro, qo, so, _ = O.row_linear_tp_big([li.a.numpy()], [li.w.numpy()], [li.sa.numpy()], [li.sw.numpy()],
                                            O.to_bits(li.residual), O.to_bits(li.norm_w), 1e-6, 1)
        assert_bits_equal(outs[0][0], ro, "residual")
        assert q_off(outs[0][1].cpu().numpy(), qo) <= 1
        for r, q, s in outs[1:]:
            assert torch.equal(r, outs[0][0]) and torch.equal(q, outs[0][1]) and torch.equal(s, outs[0][2])
        r = res0.clone()
        q = torch.empty(M, N, dtype=torch.int8, device="cuda")
        s = torch.empty(M, 1, dtype=torch.float32, device="cuda")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            c.row_linear(a, w, sa, sw, residual=r, norm_w=nw, eps=1e-6, q=q, scales=s)
        for _ in range(3):
            r.copy_(res0)
            g.replay()
        torch.cuda.synchronize()
        c.check()
        assert torch.equal(r, outs[0][0]) and torch.equal(q, outs[0][1])
        del g
    finally:
        c.close()


def test_prefill_fused_rejects_unsupported_rows(comm1):
    """M > 32 must be a multiple of 128 x world for the fused prefill tail; other M are refused (VT_EARG), so the
    caller falls back to the unfused chain."""
    M, N, K = 100, 5120, 512
    li = _inputs(M, N, K, seed=3)
    with pytest.raises(RuntimeError):
        comm1.row_linear(li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), residual=li.residual.cuda(),
                         norm_w=li.norm_w.cuda(), eps=1e-6)

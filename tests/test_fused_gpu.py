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

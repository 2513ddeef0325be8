"""AR8, the optional lossy all-reduce format (csrc/ar8.cu), against the CPU oracle (oracle/w8a8_oracle.c
orc_ar8_quant / orc_ar8_dequant_sum, the arithmetic of vllm_turing/csrc/host_ar.cu:133-201) and against the
reference's own AR8 kernels rebuilt for sm_100a (oracle/_ref/libref_host_ar.so): bit-exact. Plus the communicator glue
at one rank (TPComm.all_reduce_ar8, dmaag.all_gather_dim)."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libref_host_ar.so")


def _lib():
    from vllm_turing_b200 import _build
    return _build.load()


def _x(n, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, generator=g) * 3).half()
    x[:128] = 0                       # an all-zero group
    x[128:256] *= 1e-4                # a subnormal fp16 scale
    if n > 300:
        x[300] = 6e4
    return x


@pytest.mark.parametrize("n", [1024, 5 * 5120, 8192 * 5120 // 16 + 512 * 3])
def test_ar8_quant_bitexact(n):
    x = _x(n, n)
    packed = torch.empty(n + n // 64, dtype=torch.uint8, device="cuda")
    xd = x.cuda()
    assert _lib().ar8_quant(xd.data_ptr(), packed.data_ptr(), n, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy(), O.ar8_quant(O.to_bits(x)))


@pytest.mark.parametrize("world,n", [(1, 24 * 5120), (2, 24 * 5120), (3, 24 * 5120), (4, 24 * 5120),
                                     (8, 24 * 5120), (2, 128), (3, 128 * 7), (2, 5120 + 128)])
def test_ar8_dequant_sum_bitexact(world, n):
    """n % 512 == 0: the vectorised kernel; n % 128 == 0 only (odd blocks not 8-byte aligned, as the reference allows,
    host_ar.cu:190-201): the element-wise one. Same bits either way."""
    blocks = [O.ar8_quant(O.to_bits(_x(n, 100 + r))) for r in range(world)]
    g = torch.from_numpy(np.concatenate(blocks)).cuda()
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    assert _lib().vt_ar8_dequant_sum(g.data_ptr(), out.data_ptr(), n, world,
                                     torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert np.array_equal(O.to_bits(out.cpu()), O.ar8_dequant_sum(blocks))


def test_ar8_argument_checks():
    L = _lib()
    buf = torch.empty(4096, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.ar8_quant(buf.data_ptr(), buf.data_ptr(), 100, st) == -1           # n % 128
    assert L.vt_ar8_dequant_sum(buf.data_ptr(), buf.data_ptr(), 200, 2, st) == -1  # n % 128
    assert L.ar8_dequant_sum(buf.data_ptr(), buf.data_ptr(), 200, st) == -1         # n % 128
    assert L.vt_ar8_dequant_sum(buf.data_ptr(), buf.data_ptr(), 512, 9, st) == -1  # > 8 ranks


def test_against_reference_ar8_kernels():
    if not os.path.exists(REF):
        pytest.skip("oracle/_ref not built")
    R = ctypes.CDLL(REF)
    for f in (R.ar8_quant, R.ar8_dequant_sum):
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        f.restype = ctypes.c_int
    L = _lib()
    n = 16 * 5120
    st = torch.cuda.current_stream().cuda_stream
    xs = [_x(n, 7 + r).cuda() for r in range(2)]
    m = n + n // 64
    g_ref = torch.empty(2 * m, dtype=torch.uint8, device="cuda")
    g_us = torch.empty_like(g_ref)
    for r in range(2):
        assert R.ar8_quant(xs[r].data_ptr(), g_ref.data_ptr() + r * m, n, st) == 0
        assert L.ar8_quant(xs[r].data_ptr(), g_us.data_ptr() + r * m, n, st) == 0
    o_ref = torch.empty(n, dtype=torch.float16, device="cuda")
    o_us = torch.empty_like(o_ref)
    assert R.ar8_dequant_sum(g_ref.data_ptr(), o_ref.data_ptr(), n, st) == 0
    assert L.ar8_dequant_sum(g_us.data_ptr(), o_us.data_ptr(), n, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(g_ref.cpu(), g_us.cpu()), "packed blocks differ from the reference's"
    assert torch.equal(o_ref.cpu().view(torch.int16), o_us.cpu().view(torch.int16)), "sums differ"


@pytest.fixture(scope="module")
def comm1():
    import torch.distributed as dist
    from vllm_turing_b200.comm import TPComm
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29673")
        dist.init_process_group("gloo", rank=0, world_size=1)
    torch.cuda.set_device(0)
    c = TPComm(dist.group.WORLD, torch.device("cuda", 0))
    yield c
    c.close()


def test_comm_ar8_single_rank(comm1):
    """TPComm.all_reduce_ar8 at one rank: the packed block of the rank, gathered (nothing to fetch), summed: the
    oracle's dequantised quantisation of the input, bit for bit."""
    n = 8 * 5120
    x = _x(n, 5)
    y = comm1.all_reduce_ar8(x.cuda())
    torch.cuda.synchronize()
    assert np.array_equal(O.to_bits(y.cpu()), O.ar8_dequant_sum([O.ar8_quant(O.to_bits(x))]))
    assert comm1.status(clear=True) == 0


def test_all_gather_dim_single_rank(comm1):
    from vllm_turing_b200 import dmaag
    x = torch.randn(5, 24).to(torch.bfloat16).cuda()
    for dim in (-1, 0):
        got = dmaag.all_gather_dim(comm1, x, dim)
        torch.cuda.synchronize()
        assert got is not None and torch.equal(got.cpu(), x.cpu())

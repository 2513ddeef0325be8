"""Decode GEMV (csrc/w8a8_gemv.cu) against the CPU oracle: int32 accumulators bit-exact, dequantised outputs bit-exact
(same rounding points as vllm_turing/csrc/w8a8_gemv.cu:91), at the reference's test shapes and the BASELINE shapes."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden.make_golden import MM_CASES, mm_case_inputs
from tests.helpers import assert_bits_equal, rand_int8, rand_scales

pytestmark = pytest.mark.gpu


def _lib():
    from vllm_turing_b200 import _build
    return _build.load()


@pytest.mark.parametrize("case", [c for c in MM_CASES if c[0] <= 16])
def test_s32_golden_cases(golden, case):
    from vllm_turing_b200 import w8a8
    M, N, K = case
    a, w, sa, sw = mm_case_inputs(M, N, K)
    acc = w8a8.gemm_s32(a.cuda(), w.cuda()).cpu().numpy()
    assert np.array_equal(acc, golden[f"mm_{M}x{N}x{K}_acc"])


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 6, 7, 8, 10, 13, 16])
@pytest.mark.parametrize("NK", [(5120, 3072), (1000, 5136), (300, 5168), (40, 256)])
def test_s32_shapes(M, NK):
    """M sweep x the reference's odd shapes (tests/test_w8a8_mma.py:65-66: K % 128 = 16, N % 16 = 8)."""
    from vllm_turing_b200 import w8a8
    N, K = NK
    a, w = rand_int8((M, K), M * 7 + K), rand_int8((N, K), N * 11 + K)
    acc = w8a8.gemm_s32(a.cuda(), w.cuda()).cpu().numpy()
    assert np.array_equal(acc, O.gemm_s32(a.numpy(), w.numpy()))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(1, 5120, 8704), (5, 5120, 17408), (5, 34816, 5120), (8, 7168, 5120),
                                   (3, 136, 5136), (16, 5120, 3072)])
def test_scaled_mm_bit_exact(dtype, M, N, K):
    """w8a8_gemv through the plugin's scaled_mm_ op vs the oracle, incl. the BASELINE config 1 shapes."""
    from vllm_turing_b200 import w8a8
    code = 0 if dtype == torch.float16 else 1
    a, w = rand_int8((M, K), 1 + M), rand_int8((N, K), 2 + N)
    sa, sw = rand_scales(M, 3, 1e-2), rand_scales(N, 4, 1e-3)
    out = torch.empty(M, N, dtype=dtype, device="cuda")
    wc = w.cuda()
    if M <= w8a8.MAX_M:      # through the plugin op's dispatch
        assert w8a8.gemv_ok(out, a.cuda(), wc.t(), sa.cuda(), sw.cuda(), None)
        torch.ops.vllm_turing.scaled_mm_(out, a.cuda(), wc.t(), sa.cuda(), sw.cuda(), None)
    else:                    # the GEMV entry directly (it serves M <= 16 like the reference's)
        w8a8.gemv(out, a.cuda(), wc.t(), sa.cuda(), sw.cuda(), None)
    want = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), None, code)
    assert_bits_equal(out, want, f"scaled_mm M={M} N={N} K={K}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_bias_and_per_tensor_scale(dtype):
    """bias + per-tensor activation scale (tests/test_w8a8_mma.py:63-64) through the reference ABI entry."""
    L = _lib()
    code = 0 if dtype == torch.float16 else 1
    M, N, K = 5, 8192, 5120
    a, w = rand_int8((M, K), 21), rand_int8((N, K), 22)
    sa, sw = rand_scales(1, 23, 1e-2), rand_scales(N, 24, 1e-3)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(25)).to(dtype)
    out = torch.empty(M, N, dtype=dtype, device="cuda")
    ac, wc, sac, swc, bc = a.cuda(), w.cuda(), sa.cuda(), sw.cuda(), bias.cuda()
    rc = L.w8a8_gemv(ac.data_ptr(), wc.data_ptr(), sac.data_ptr(), swc.data_ptr(), bc.data_ptr(), out.data_ptr(),
                     M, N, K, 0, 1, code, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    want = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), O.to_bits(bias), code)
    assert_bits_equal(out, want, "bias / per-tensor")
    assert L.vt_status(1) == 0


def test_rejects_bad_arguments():
    L = _lib()
    z = torch.zeros(64, dtype=torch.int8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert L.w8a8_gemv(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), None, z.data_ptr(), 1, 2, 24, 1, 1,
                       1, s) == -1        # K % 16 != 0 (vllm_turing/csrc/w8a8_gemv.cu:349)
    assert L.w8a8_gemv(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), None, z.data_ptr(), 17, 2, 32, 1, 1,
                       1, s) == -1        # M > 16
    assert L.w8a8_gemv(z.data_ptr() + 1, z.data_ptr(), z.data_ptr(), z.data_ptr(), None, z.data_ptr(), 1, 2, 32, 1,
                       1, 1, s) == -1     # misaligned a


def test_back_to_back_calls_reuse_workspace():
    """64 launches without host syncs over alternating shapes: the self-cleaning split-K scratch stays exact."""
    from vllm_turing_b200 import w8a8
    shapes = [(5, 5120, 17408), (3, 34816, 5120), (8, 5120, 8704)]
    ins = [(rand_int8((M, K), 100 + i).cuda(), rand_int8((N, K), 200 + i).cuda()) for i, (M, N, K) in
           enumerate(shapes)]
    outs = [w8a8.gemm_s32(a, w) for _ in range(21) for a, w in ins]
    torch.cuda.synchronize()
    refs = [O.gemm_s32(a.cpu().numpy(), w.cpu().numpy()) for a, w in ins]
    for i, o in enumerate(outs):
        assert np.array_equal(o.cpu().numpy(), refs[i % 3]), f"call {i}"


def test_cuda_graph_replay():
    """The GEMV captured in a CUDA graph (decode runs in graphs) and replayed with fresh inputs."""
    from vllm_turing_b200 import w8a8
    M, N, K = 5, 5120, 8704
    a = rand_int8((M, K), 1).cuda()
    w = rand_int8((N, K), 2).cuda()
    sa, sw = rand_scales(M, 3, 1e-2).cuda(), rand_scales(N, 4, 1e-3).cuda()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    torch.ops.vllm_turing.scaled_mm_(out, a, w.t(), sa, sw, None)     # sizes the workspace outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        torch.ops.vllm_turing.scaled_mm_(out, a, w.t(), sa, sw, None)
    for it in range(5):
        a.copy_(rand_int8((M, K), 50 + it).cuda())
        g.replay()
        torch.cuda.synchronize()
        want = O.scaled_mm(a.cpu().numpy(), w.cpu().numpy(), sa.cpu().numpy(), sw.cpu().numpy(), None, 1)
        assert_bits_equal(out, want, f"replay {it}")
    assert w8a8 is not None

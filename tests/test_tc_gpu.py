"""The tcgen05 kind::i8 GEMMs (csrc/w8a8_tc.cu) against the oracle: int32 accumulators bit-exact, dequantised outputs
bit-exact in each path's epilogue order -- w8a8_big: sa * (sw * acc) (vllm_turing/csrc/w8a8_big.cu:26-35); w8a8_mma:
(acc * sa) * sw + bias (vllm_turing/csrc/w8a8_gemv.cu:288) -- at the reference's test shapes (tests/test_w8a8_mma.py:
109-116, tests/test_w8a8_big.py:45-54) and the BASELINE prefill / decode shapes."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bits_equal, rand_int8, rand_scales

pytestmark = pytest.mark.gpu


def _lib():
    from vllm_turing_b200 import _build
    return _build.load()


def _s():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("M,N,K", [(1, 128, 16), (5, 34816, 5120), (5, 5120, 17408), (9, 5120, 5136),
                                   (13, 1000, 5136), (16, 5120, 17408), (17, 300, 5168), (24, 5120, 2176),
                                   (32, 5120, 8704), (25, 7168, 5120), (32, 136, 128), (3, 40, 65536)])
def test_small_s32(M, N, K):
    """decode orientation (weights as the A operand, stream-K over the SMs): M 1..32; single-tile and single-K-block
    cases, tiles split across several CTAs, CTAs spanning several tiles, K not a multiple of the 128-byte block"""
    L = _lib()
    a, w = rand_int8((M, K), M + K), rand_int8((N, K), N + 3 * K)
    acc = torch.full((M, N), -7, dtype=torch.int32, device="cuda")
    ac, wc = a.cuda(), w.cuda()
    nz0 = L.vt_workspace_nonzero(8 << 20)
    assert L.vt_gemm_s32(ac.data_ptr(), wc.data_ptr(), acc.data_ptr(), M, N, K, _s()) == 0
    torch.cuda.synchronize()
    got, ref = acc.cpu().numpy(), O.gemm_s32(a.numpy(), w.numpy())
    if not np.array_equal(got, ref):
        bad = np.argwhere(got != ref)
        d = (got - ref)[got != ref]
        raise AssertionError(
            f"{len(bad)} mismatches; workspace non-zero before {nz0}, after {L.vt_workspace_nonzero(8 << 20)}; "
            f"first {bad[:6].tolist()}; rows {np.unique(bad[:, 0]).tolist()[:12]}; n in [{bad[:, 1].min()}, "
            f"{bad[:, 1].max()}]; unwritten (-7) {(got == -7).sum()}; diffs {d[:8].tolist()}; status {L.vt_status(0):#x}")
    assert L.vt_status(1) == 0


@pytest.mark.parametrize("M,N,K", [(33, 256, 128), (128, 5120, 3072), (200, 1000, 5136), (2048, 5120, 8704),
                                   (1680, 8704, 5120), (300, 136, 5168), (2600, 1000, 256)])
def test_big_s32(M, N, K):
    """prefill orientation (activations as the A operand, 128 x 256 tiles, grouped raster of 16 A tiles: 2600 rows
    make a full group and a 5-tile one)"""
    a, w = rand_int8((M, K), 5 * M + K), rand_int8((N, K), 7 * N + K)
    acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
    ac, wc = a.cuda(), w.cuda()
    assert _lib().vt_gemm_s32(ac.data_ptr(), wc.data_ptr(), acc.data_ptr(), M, N, K, _s()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), O.gemm_s32(a.numpy(), w.numpy()))
    assert _lib().vt_status(1) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(128, 5120, 3072), (2048, 5120, 8704), (1680, 8704, 5120), (8192, 5120, 2176)])
def test_big_dequant_bit_exact(dtype, M, N, K):
    code = 0 if dtype == torch.float16 else 1
    a, w = rand_int8((M, K), M + 11), rand_int8((N, K), N + 13)
    sa, sw = rand_scales(M, 1, 1e-2), rand_scales(N, 2, 1e-3)
    out = torch.empty(M, N, dtype=dtype, device="cuda")
    ac, wc, sac, swc = a.cuda(), w.cuda(), sa.cuda(), sw.cuda()
    assert _lib().w8a8_big(ac.data_ptr(), wc.data_ptr(), sac.data_ptr(), swc.data_ptr(), out.data_ptr(), M, N, K,
                           code, _s()) == 0
    want = O.dequant_big(O.gemm_s32(a.numpy(), w.numpy()), sa.numpy(), sw.numpy(), code)
    assert_bits_equal(out, want, f"w8a8_big M={M}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K,bias,per_row", [(13, 5120, 8704, False, True), (20, 17408, 5120, False, True),
                                                (31, 8192, 5120, True, True), (21, 5120, 3072, False, False),
                                                (27, 1000, 5136, False, True), (32, 300, 5168, True, True),
                                                (9, 7168, 5120, False, True)])
def test_mma_dequant_bit_exact(dtype, M, N, K, bias, per_row):
    """the reference's w8a8_mma cases (tests/test_w8a8_mma.py:61-68): bias, per-tensor scale, odd K / N"""
    code = 0 if dtype == torch.float16 else 1
    a, w = rand_int8((M, K), M + 17), rand_int8((N, K), N + 19)
    sa = rand_scales(M if per_row else 1, 3, 1e-2)
    sw = rand_scales(N, 4, 1e-3)
    b = torch.randn(N, generator=torch.Generator().manual_seed(5)).to(dtype) if bias else None
    out = torch.empty(M, N, dtype=dtype, device="cuda")
    ac, wc, sac, swc = a.cuda(), w.cuda(), sa.cuda(), sw.cuda()
    bc = b.cuda() if b is not None else None
    assert _lib().w8a8_mma(ac.data_ptr(), wc.data_ptr(), sac.data_ptr(), swc.data_ptr(),
                           bc.data_ptr() if bc is not None else None, out.data_ptr(), M, N, K, int(per_row), 1, code,
                           _s()) == 0
    want = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), O.to_bits(b) if b is not None else None, code)
    assert_bits_equal(out, want, f"w8a8_mma M={M}")


def test_dispatch_through_scaled_mm_op():
    """vllm_turing::scaled_mm_ picks the GEMV (M <= VLLM_TURING_GEMV_MAX_M, off by default), the small-M tensor-core
    kernel (M <= 32) and the prefill kernel (larger M), as vllm_turing/w8a8.py:108-117 does."""
    from vllm_turing_b200 import w8a8
    N, K = 5120, 8704
    w = rand_int8((N, K), 1)
    wc = w.cuda()
    sw = rand_scales(N, 2, 1e-3)
    for M, path in ((5, "gemv" if w8a8.MAX_M >= 5 else "mma"), (24, "mma"), (512, "big")):
        a = rand_int8((M, K), 3 + M)
        sa = rand_scales(M, 4, 1e-2)
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        args = (out, a.cuda(), wc.t(), sa.cuda().view(-1, 1), sw.cuda().view(-1, 1), None)
        got = "gemv" if w8a8.gemv_ok(*args) else ("mma" if w8a8.mma_ok(*args) else
                                                  ("big" if w8a8.big_ok(*args) else "vllm"))
        assert got == path
        torch.ops.vllm_turing.scaled_mm_(*args)
        acc = O.gemm_s32(a.numpy(), w.numpy())
        want = (O.dequant_big(acc, sa.numpy(), sw.numpy(), 1) if path == "big"
                else O.dequant(acc, sa.numpy(), sw.numpy(), None, 1))
        assert_bits_equal(out, want, f"dispatch M={M}")


def test_back_to_back_small_and_big():
    """Mixed launches without host syncs: the split-K scratch and tickets stay consistent."""
    L = _lib()
    cases = [(24, 5120, 8704), (2048, 5120, 2176), (16, 34816, 5120), (32, 5120, 17408)]
    ins = [(rand_int8((M, K), 40 + i).cuda(), rand_int8((N, K), 50 + i).cuda()) for i, (M, N, K) in enumerate(cases)]
    outs = []
    for rep in range(4):
        for (M, N, K), (a, w) in zip(cases, ins):
            acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
            assert L.vt_gemm_s32(a.data_ptr(), w.data_ptr(), acc.data_ptr(), M, N, K, _s()) == 0
            outs.append(acc)
    torch.cuda.synchronize()
    refs = [O.gemm_s32(a.cpu().numpy(), w.cpu().numpy()) for a, w in ins]
    for i, o in enumerate(outs):
        assert np.array_equal(o.cpu().numpy(), refs[i % len(cases)]), f"launch {i}"


@pytest.mark.parametrize("M,N,K", [(5, 34816, 5120), (16, 5120, 17408), (1, 128, 128), (32, 1024, 2176),
                                   (9, 4352, 5120)])
def test_mma_blocked_weight_layout(M, N, K):
    """the decode GEMM on the tile-blocked weight layout (w8a8.block_weight): the same bits as on the row-major
    weight, and as the oracle"""
    from vllm_turing_b200 import w8a8
    a, w = rand_int8((M, K), M + 31), rand_int8((N, K), N + 37)
    sa, sw = rand_scales(M, 5, 1e-2), rand_scales(N, 6, 1e-3)
    ac, wc, sac, swc = a.cuda(), w.cuda(), sa.cuda().view(-1, 1), sw.cuda().view(-1, 1)
    out_b = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    out_r = torch.empty_like(out_b)
    w8a8.mma_blocked(out_b, ac, w8a8.block_weight(wc), sac, swc)
    w8a8.mma(out_r, ac, wc.t(), sac, swc, None)
    torch.cuda.synchronize()
    assert torch.equal(out_b, out_r)
    assert_bits_equal(out_b, O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), None, 1), f"blocked M={M}")

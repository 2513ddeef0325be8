"""Parity against the reference itself: its own GEMV / int8-MMA kernels (vllm_turing/csrc/w8a8_gemv.cu), compiled from
the reference sources for sm_100a into oracle/_ref/ (make -C oracle ref; the reference's nvcc flags with the B200
arch), run on the same inputs as this package's kernels. Outputs must be bitwise equal (same int32 sums, same epilogue
rounding, vllm_turing/csrc/w8a8_gemv.cu:91 and :288). The timing of both is printed (-s) as a comparison point: the
reference's sm_75 design recompiled for B200 against the B200-native kernels. Skipped when oracle/_ref was not built
(the reference tree was absent where the repository was built)."""
import ctypes
import os

import pytest
import torch

from tests.helpers import rand_int8, rand_scales

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "libref_w8a8_gemv.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF):
        pytest.skip("oracle/_ref not built")
    L = ctypes.CDLL(REF)
    for f in (L.w8a8_gemv, L.w8a8_mma):
        f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_void_p]
        f.restype = ctypes.c_int
    return L


def _run(fn, a, w, sa, sw, out, M, N, K, code):
    return fn(a.data_ptr(), w.data_ptr(), sa.data_ptr(), sw.data_ptr(), None, out.data_ptr(), M, N, K, 1, 1, code,
              torch.cuda.current_stream().cuda_stream)


def _time(fn, reps=20):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3


@pytest.mark.parametrize("M,N,K,entry", [(1, 5120, 17408, "w8a8_gemv"), (5, 5120, 17408, "w8a8_gemv"),
                                         (5, 34816, 5120, "w8a8_gemv"), (8, 5120, 8704, "w8a8_gemv"),
                                         (16, 5120, 3072, "w8a8_gemv"), (24, 5120, 8704, "w8a8_mma"),
                                         (32, 17408, 5120, "w8a8_mma"), (13, 1000, 5136, "w8a8_mma")])
def test_bitwise_equal_to_reference_kernels(ref, M, N, K, entry):
    from vllm_turing_b200 import _build
    ours = _build.load()
    a, w = rand_int8((M, K), 31 + M).cuda(), rand_int8((N, K), 37 + N).cuda()
    sa, sw = rand_scales(M, 41, 1e-2).cuda(), rand_scales(N, 43, 1e-3).cuda()
    o_ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    o_us = torch.empty_like(o_ref)
    assert _run(getattr(ref, entry), a, w, sa, sw, o_ref, M, N, K, 1) == 0
    # this package's entry of the same name (its GEMV takes M <= 16, the tensor-core kernel M <= 32)
    assert _run(getattr(ours, entry), a, w, sa, sw, o_us, M, N, K, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(o_ref, o_us), f"{entry} M={M} N={N} K={K} differs from the reference kernel"
    t_ref = _time(lambda: _run(getattr(ref, entry), a, w, sa, sw, o_ref, M, N, K, 1))
    t_us = _time(lambda: _run(getattr(ours, entry), a, w, sa, sw, o_us, M, N, K, 1))
    gb = N * K / 1e9
    print(f"\n[ref-kernel] {entry} M={M} N={N} K={K}: reference sm_75 design on B200 {t_ref:.1f} us "
          f"({gb / t_ref * 1e6:.0f} GB/s), B200-native {t_us:.1f} us ({gb / t_us * 1e6:.0f} GB/s), "
          f"{t_ref / t_us:.2f}x")

"""w8a8_gemv_noalloc: the GEMV for callers that cannot allocate device memory when they call it (code running inside a
memory profiler or a custom allocator, or after all device memory went to a pool). Called through the C ABI, it must
give the same outputs as the regular entry w8a8_gemv (the GEMV tests compare bit-exactly, so this does too) on two
calls in a row with different inputs, allocate nothing itself, and reject shapes beyond its fixed scratch array.
This file is collected last so a failure here does not stop the other tests of a run; it also passes alone."""
import ctypes

import pytest
import torch

from tests.helpers import rand_int8, rand_scales

pytestmark = pytest.mark.gpu


def _lib():
    from vllm_turing_b200 import _build
    return _build.load()


def _call(fn, a, w, sa, sw, out, M, N, K):
    return fn(a.data_ptr(), w.data_ptr(), sa.data_ptr(), sw.data_ptr(), None, out.data_ptr(), M, N, K, 1, 1, 1,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,N,K", [(5, 34816, 5120), (5, 5120, 17408), (8, 7168, 5120), (3, 136, 5136)])
def test_noalloc_matches_regular_entry_twice(M, N, K):
    L = _lib()
    torch.cuda.set_device(0)
    outs = []
    for call in range(2):                  # two calls in a row, different inputs
        a = rand_int8((M, K), 100 * call + M).cuda()
        w = rand_int8((N, K), 100 * call + N).cuda()
        sa, sw = rand_scales(M, call + 1, 1e-2).cuda(), rand_scales(N, call + 2, 1e-3).cuda()
        ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        got = torch.empty_like(ref)
        assert _call(L.w8a8_gemv, a, w, sa, sw, ref, M, N, K) == 0
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        assert _call(L.w8a8_gemv_noalloc, a, w, sa, sw, got, M, N, K) == 0
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before
        assert torch.equal(got, ref), f"call {call}: differs from w8a8_gemv"
        outs.append(got)
    assert not torch.equal(outs[0], outs[1])


def test_noalloc_rejects_sizes_beyond_its_array():
    L = _lib()
    z = torch.zeros(64, dtype=torch.int8, device="cuda")
    p = z.data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    # M * N = 16 * 20480 = 327680 > 262144: rejected before any launch
    assert L.w8a8_gemv_noalloc(ctypes.c_void_p(p), p, p, p, None, p, 16, 20480, 32, 1, 1, 1, s) == -1
    assert L.w8a8_gemv_noalloc(p, p, p, p, None, p, 1, 4, 24, 1, 1, 1, s) == -1      # K % 16 != 0, as w8a8_gemv

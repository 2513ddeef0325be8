"""w8a8_gemv_noalloc: the GEMV for callers that cannot allocate device memory when they call it -- code running inside
vLLM's memory profiling (which attributes every allocation made during the profiled forward), inside a custom
allocator, or in a process that has already handed all free device memory to a pool.

Called through the C ABI, it must
  - give the same bits as the regular entry w8a8_gemv and as the CPU oracle, on two calls in a row with different
    inputs (the array keeps the previous call's contents);
  - allocate nothing: the driver's free-memory figure (torch.cuda.mem_get_info, which also sees a cudaMalloc made
    inside the library, unlike torch's own allocator statistics) is unchanged across the second call. The first call
    on a device may load the library's module together with its fixed array (lazy module loading), so it comes first,
    before the measured window; shapes the regular entry has not seen yet are used, so a fallback to the library's
    growing workspace would show;
  - report a device-side timeout through vt_noalloc_status (0 after clean calls);
  - reject shapes beyond its fixed array.
This file is collected last so a failure here does not stop the other tests of a run; it also passes alone."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import rand_int8, rand_scales

pytestmark = pytest.mark.gpu


def _lib():
    from vllm_turing_b200 import _build
    return _build.load()


def _call(fn, a, w, sa, sw, out, M, N, K):
    return fn(a.data_ptr(), w.data_ptr(), sa.data_ptr(), sw.data_ptr(), None, out.data_ptr(), M, N, K, 1, 1, 1,
              torch.cuda.current_stream().cuda_stream)


# shapes chosen so the regular entry's library workspace has not been sized for them by earlier tests
@pytest.mark.parametrize("M,N,K", [(7, 37376, 5120), (5, 5120, 17408), (8, 7168, 5120), (3, 136, 5136)])
def test_noalloc_matches_regular_entry_and_oracle_twice(M, N, K):
    L = _lib()
    torch.cuda.set_device(0)
    ins = []
    for call in range(2):                  # two calls in a row, different inputs; every tensor made up front
        a, w = rand_int8((M, K), 100 * call + M), rand_int8((N, K), 100 * call + N)
        sa, sw = rand_scales(M, call + 1, 1e-2), rand_scales(N, call + 2, 1e-3)
        ins.append(dict(h=(a, w, sa, sw), d=(a.cuda(), w.cuda(), sa.cuda(), sw.cuda()),
                        got=torch.empty(M, N, dtype=torch.bfloat16, device="cuda"),
                        ref=torch.empty(M, N, dtype=torch.bfloat16, device="cuda")))
    torch.cuda.synchronize()
    assert L.vt_noalloc_status(1) != 0xffffffff
    # call 1 (may load the module and its array), then the measured window around call 2
    assert _call(L.w8a8_gemv_noalloc, *ins[0]["d"], ins[0]["got"], M, N, K) == 0
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    assert _call(L.w8a8_gemv_noalloc, *ins[1]["d"], ins[1]["got"], M, N, K) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "w8a8_gemv_noalloc changed the device's free memory"
    assert L.vt_noalloc_status(1) == 0, "a kernel of w8a8_gemv_noalloc reported a timeout"
    for call, x in enumerate(ins):
        assert _call(L.w8a8_gemv, *x["d"], x["ref"], M, N, K) == 0
        torch.cuda.synchronize()
        assert torch.equal(x["got"], x["ref"]), f"call {call}: differs from w8a8_gemv"
        a, w, sa, sw = x["h"]
        want = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), None, 1)
        assert np.array_equal(O.to_bits(x["got"]), want), f"call {call}: differs from the oracle"
    assert not torch.equal(ins[0]["got"], ins[1]["got"])


def test_noalloc_rejects_sizes_beyond_its_array():
    L = _lib()
    z = torch.zeros(64, dtype=torch.int8, device="cuda")
    p = z.data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    # M * N = 16 * 20480 = 327680 > 262144: rejected before any launch
    assert L.w8a8_gemv_noalloc(ctypes.c_void_p(p), p, p, p, None, p, 16, 20480, 32, 1, 1, 1, s) == -1
    assert L.w8a8_gemv_noalloc(p, p, p, p, None, p, 1, 4, 24, 1, 1, 1, s) == -1      # K % 16 != 0, as w8a8_gemv

"""Every kernel that uses the library's split-K workspace (the GEMV and the tcgen05 decode GEMM) must leave it all
zero: the next call, of any kernel and shape, relies on it (partial sums are added into it, tickets count in it).
Checked after each call of a sequence that mixes entries, shapes, dtypes and per-tensor scales."""
import pytest
import torch

from tests.helpers import rand_int8, rand_scales

pytestmark = pytest.mark.gpu

CASES = [  # (entry, M, N, K, per_row_sa)
    ("w8a8_gemv", 5, 5120, 17408, 1), ("w8a8_gemv", 16, 5120, 3072, 1), ("w8a8_gemv", 8, 5120, 8704, 1),
    ("w8a8_gemv", 5, 8192, 5120, 0), ("w8a8_gemv", 3, 34816, 5120, 1), ("w8a8_gemv", 1, 5120, 2176, 1),
    ("w8a8_mma", 24, 5120, 8704, 1), ("w8a8_mma", 32, 17408, 5120, 1), ("w8a8_mma", 13, 1000, 5136, 1),
    ("w8a8_mma", 9, 5120, 5136, 0), ("w8a8_mma", 17, 300, 5168, 1), ("vt_gemv_s32", 7, 5120, 4352, 1),
    ("vt_gemm_s32", 20, 5120, 2176, 1),
]
# every GEMV shape of the M sweep in test_gemv_gpu, and the golden GEMM cases
CASES += [("vt_gemv_s32", M, N, K, 1) for M in (1, 2, 3, 4, 5, 6, 7, 8, 10, 13, 16)
          for N, K in ((5120, 3072), (1000, 5136), (300, 5168), (40, 256))]
CASES += [("vt_gemv_s32", 1, 64, 64, 1), ("vt_gemv_s32", 5, 136, 5136, 1), ("vt_gemv_s32", 16, 256, 1024, 1),
          ("vt_gemm_s32", 24, 40, 256, 1), ("vt_gemm_s32", 32, 300, 5168, 1), ("vt_gemm_s32", 9, 5120, 5136, 1)]


def test_workspace_left_zeroed_after_every_call():
    from vllm_turing_b200 import _build
    L = _build.load()
    s = torch.cuda.current_stream().cuda_stream
    assert L.vt_workspace_nonzero(8 << 20) == 0
    for i, (entry, M, N, K, per_row) in enumerate(CASES):
        a, w = rand_int8((M, K), 3 * i + 1).cuda(), rand_int8((N, K), 3 * i + 2).cuda()
        sa, sw = rand_scales(M if per_row else 1, i, 1e-2).cuda(), rand_scales(N, i + 1, 1e-3).cuda()
        if entry.startswith("vt_"):
            out = torch.empty(M, N, dtype=torch.int32, device="cuda")
            rc = getattr(L, entry)(a.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, K, s)
        else:
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            rc = getattr(L, entry)(a.data_ptr(), w.data_ptr(), sa.data_ptr(), sw.data_ptr(), None, out.data_ptr(),
                                   M, N, K, per_row, 1, 1, s)
        assert rc == 0, (entry, M, N, K, rc)
        nz = L.vt_workspace_nonzero(8 << 20)
        assert nz == 0, f"{entry} M={M} N={N} K={K} left {nz} non-zero scratch words"

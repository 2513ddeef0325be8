"""The int8 LM head (W8A16: int8 weight rows with fp32 row scales, 16-bit activations; csrc/w8a16_tc.cu) against the
CPU oracle (oracle/w8a8_oracle.c: orc_w8a16, the arithmetic of vllm_turing/csrc/w8a16_gemv.cu:64-106 with the sum in
float64), against the golden vectors made by the reference's own lmhead.quantize_rows, and against the reference's
own W8A16 kernels rebuilt for sm_100a (oracle/_ref).

Tolerance (floating point: the fp32 sums are taken in a different order than the reference's): |got - want| <= one
unit in the last place of the 16-bit type at |want| + 2^-16 * s[n] * sum_k |x w| (oracle.w8a16_close <= 1). The
bound's second term is K * 2^-24 * mag at K = 256, and for the sizes here far above any observed fp32 summation error
while still far below the size of a single wrong product."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def _lib():
    from vllm_turing_b200 import _build
    return _build.load()


def _inputs(M, N, K, seed, dtype=torch.bfloat16, bias=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 1e-3 + 1e-5
    b = (torch.randn(N, generator=g) * 0.1).to(dtype) if bias else None
    return x, w, s, b


def _check(out, x, w, s, b, code, what):
    want, _, mag = O.w8a16(O.to_bits(x), w.numpy(), s.numpy(), O.to_bits(b) if b is not None else None, code,
                           want_acc=True)
    err = O.w8a16_close(O.to_bits(out.cpu()), want, mag, s.numpy(), code)
    assert err <= 1.0, f"{what}: worst error {err:.2f} x the tolerance"


CASES = [(1, 136, 256), (5, 1000, 5120), (16, 300, 1040), (17, 2048, 512), (32, 640, 5120), (33, 129, 384),
         (64, 1024, 2048), (5, 18992, 5120), (3, 1, 64)]


@pytest.mark.parametrize("M,N,K", CASES)
@pytest.mark.parametrize("dtype,code", [(torch.bfloat16, 1), (torch.float16, 0)])
def test_w8a16_vs_oracle(M, N, K, dtype, code):
    from vllm_turing_b200 import lmhead
    x, w, s, b = _inputs(M, N, K, M * 7 + N + K, dtype, bias=(M % 2 == 1))
    dx, dw, ds = x.cuda(), w.cuda(), s.cuda()
    db = b.cuda() if b is not None else None
    out = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
    lmhead.mm_into(out, dx, dw, ds, db)
    torch.cuda.synchronize()
    _check(out, x, w, s, b, code, f"M={M} N={N} K={K} {dtype}")
    assert _lib().vt_status(1) == 0


@pytest.mark.parametrize("code", [0, 1])
@pytest.mark.parametrize("case", [(1, 64, 256), (5, 300, 1040), (17, 136, 512)])
def test_w8a16_golden(golden, code, case):
    """The reference's quantised head (lmhead.quantize_rows, golden) through the kernel, against the golden logits."""
    from vllm_turing_b200 import lmhead
    key = f"lm_{code}_{case[0]}x{case[1]}x{case[2]}"
    dt = torch.bfloat16 if code else torch.float16
    x = O.from_bits(golden[key + "_x"], dt).cuda()
    b = O.from_bits(golden[key + "_b"], dt).cuda()
    q, s = torch.from_numpy(golden[key + "_q"]).cuda(), torch.from_numpy(golden[key + "_s"]).cuda()
    out = torch.ops.vllm_turing.w8a16_mm(x, q, s, b)
    torch.cuda.synchronize()
    _, _, mag = O.w8a16(golden[key + "_x"], golden[key + "_q"], golden[key + "_s"], golden[key + "_b"], code,
                        want_acc=True)
    err = O.w8a16_close(O.to_bits(out.cpu()), golden[key + "_out"], mag, golden[key + "_s"], code)
    assert err <= 1.0, f"{key}: {err:.2f}"


def test_quantize_rows_on_gpu_matches_oracle(golden):
    """On the GPU (where the reference quantises its head, lmhead.py:125-128) torch divides by the scalar 127 as a
    multiplication by its float32 reciprocal; the oracle's device="cuda" form restates that, bit for bit."""
    from vllm_turing_b200 import lmhead
    for code in (0, 1):
        for case in ("1x64x256", "5x300x1040", "17x136x512"):
            key = f"lm_{code}_{case}"
            w = O.from_bits(golden[key + "_w"], torch.bfloat16 if code else torch.float16)
            q, s = lmhead.quantize_rows(w.cuda())
            qo, so = O.lmhead_quant(w.float().numpy(), device="cuda")
            assert np.array_equal(s.cpu().numpy(), so) and np.array_equal(q.cpu().numpy(), qo), key


def test_output_stride_leaves_other_columns():
    """ldo > N: the kernel writes columns [0, N) of each row of a wider buffer and nothing else."""
    from vllm_turing_b200 import lmhead
    M, N, K, ld = 5, 1000, 1024, 4000
    x, w, s, _ = _inputs(M, N, K, 11)
    buf = torch.full((M, ld), 7.0, dtype=torch.bfloat16, device="cuda")
    lmhead.mm_into(buf[:, 1000:], x.cuda(), w.cuda(), s.cuda(), None, ldo=ld)
    torch.cuda.synchronize()
    _check(buf[:, 1000:2000], x, w, s, None, 1, "strided")
    host = buf.cpu()
    assert (host[:, :1000] == 7.0).all() and (host[:, 2000:] == 7.0).all()


def test_rows_gather_variant():
    """w8a16_gemv_rows with an index list (the reference's pruned-vocabulary path): CUDA-core kernel."""
    M, N, K = 7, 2000, 1024
    x, w, s, b = _inputs(M, N, K, 21, torch.float16, bias=True)
    rows = torch.randperm(N, generator=torch.Generator().manual_seed(1))[:333].to(torch.int32)
    out = torch.empty(M, 333, dtype=torch.float16, device="cuda")
    dx, dw, ds, db, dr = x.cuda(), w.cuda(), s.cuda(), b.cuda(), rows.cuda()
    rc = _lib().w8a16_gemv_rows(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), db.data_ptr(), out.data_ptr(), M, 333, K,
                                0, dr.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    ri = rows.long()
    _check(out, x, w[ri].contiguous(), s[ri].contiguous(), b[ri].contiguous(), 0, "rows")


def test_op_passes_and_large_m_path():
    """M = 100: two kernel passes; M = 300 (> GEMV_MAX_M): the reference's dequantise-and-matmul path."""
    for M in (100, 300):
        x, w, s, _ = _inputs(M, 520, 512, M)
        out = torch.ops.vllm_turing.w8a16_mm(x.cuda(), w.cuda(), s.cuda(), None)
        torch.cuda.synchronize()
        if M <= 256:
            _check(out, x, w, s, None, 1, f"op M={M}")
        else:
            want = O.bits_to_float(O.w8a16(O.to_bits(x), w.numpy(), s.numpy(), None, 1), 1).astype(np.float64)
            got = O.bits_to_float(O.to_bits(out.cpu()), 1).astype(np.float64)
            assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-2


def test_argument_checks():
    L = _lib()
    x, w, s, _ = _inputs(5, 256, 64, 3)
    dx, dw, ds = x.cuda(), w.cuda(), s.cuda()
    out = torch.empty(5, 256, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    args = (dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), None, out.data_ptr())
    assert L.w8a16_gemv(*args, 17, 256, 64, 1, st) == -1          # GEMV entry: M <= 16 (w8a16_gemv.cu:127)
    assert L.w8a16_gemv(*args, 5, 256, 60, 1, st) == -1           # K % 16
    assert L.w8a16_mma(*args, 5, 255, 64, 2, st) == -1            # N even (w8a16_mma.cu:163)
    assert L.w8a16_mma(*args, 65, 256, 64, 2, st) == -1           # M <= 64
    ws = torch.zeros(int(L.vt_w8a16_ws_bytes(5, 64)), dtype=torch.uint8, device="cuda")
    assert L.vt_w8a16_mm(*args, 5, 256, 64, 255, 1, ws.data_ptr(), ws.numel(), st) == -1   # ldo < N
    assert L.vt_w8a16_mm(*args, 5, 256, 64, 256, 1, ws.data_ptr(), 64, st) == -1           # workspace too small
    assert L.w8a16_gemv(*args, 5, 256, 64, 1, st) == 0
    torch.cuda.synchronize()


def test_workspace_left_zeroed_and_graph_replay():
    """The caller's workspace's split-K slots are zero after the calls (cleared by the head CTAs; they follow the
    status word, the activation limbs [32, K] and their exponents), and the kernel replays in a CUDA graph with fresh
    activations."""
    from vllm_turing_b200 import lmhead
    M, N, K = 5, 18992, 5120
    slots = 256 + (32 * K + 255) // 256 * 256 + 256
    x, w, s, _ = _inputs(M, N, K, 5)
    dx, dw, ds = x.cuda(), w.cuda(), s.cuda()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    lmhead.mm_into(out, dx, dw, ds)
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(lmhead.workspace(dx.device, K)[slots:])) == 0
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lmhead.mm_into(out, dx, dw, ds)
    for it in range(2):
        x2 = torch.randn(M, K, generator=torch.Generator().manual_seed(50 + it)).to(torch.bfloat16)
        dx.copy_(x2.cuda())
        g.replay()
        torch.cuda.synchronize()
        _check(out, x2, w, s, None, 1, f"graph replay {it}")
    assert int(torch.count_nonzero(lmhead.workspace(dx.device, K)[slots:])) == 0
    del g


def test_logits_gathered_single_rank():
    from vllm_turing_b200 import lmhead
    x, w, s, _ = _inputs(5, 4096, 1024, 8)
    a = lmhead.logits_gathered(x.cuda(), w.cuda(), s.cuda())
    b = torch.ops.vllm_turing.w8a16_mm(x.cuda(), w.cuda(), s.cuda(), None)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


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


@pytest.mark.parametrize("M,N,entry", [(1, 18992, "w8a16_gemv"), (5, 18992, "w8a16_gemv"),
                                       (16, 37984, "w8a16_gemv"), (30, 18992, "w8a16_mma")])
def test_against_reference_kernels(M, N, entry):
    """The reference's own W8A16 kernels (vllm_turing/csrc/w8a16_gemv.cu, w8a16_mma.cu, rebuilt for sm_100a) on the same
    inputs: both within the tolerance of the oracle. Timings printed (-s)."""
    so = os.path.join(REF, "libref_" + ("w8a16_gemv" if entry == "w8a16_gemv" else "w8a16_mma") + ".so")
    if not os.path.exists(so):
        pytest.skip("oracle/_ref not built")
    R = ctypes.CDLL(so)
    fn = getattr(R, entry)
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    fn.restype = ctypes.c_int
    K = 5120
    dt, code = (torch.float16, 0) if entry == "w8a16_mma" else (torch.bfloat16, 1)
    x, w, s, _ = _inputs(M, N, K, 77 + M, dt)
    dx, dw, ds = x.cuda(), w.cuda(), s.cuda()
    o_ref = torch.empty(M, N, dtype=dt, device="cuda")
    o_us = torch.empty_like(o_ref)
    last = 2 if entry == "w8a16_mma" else code
    st = torch.cuda.current_stream().cuda_stream
    ref_call = lambda: fn(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), None, o_ref.data_ptr(), M, N, K, last, st)
    us_call = lambda: getattr(_lib(), entry)(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), None, o_us.data_ptr(), M, N,
                                             K, last, st)
    assert ref_call() == 0 and us_call() == 0
    torch.cuda.synchronize()
    _check(o_ref, x, w, s, None, code, "reference kernel")
    _check(o_us, x, w, s, None, code, "this kernel")
    t_ref, t_us = _time(ref_call), _time(us_call)
    gb = N * K / 1e9
    print(f"\n{entry} M={M} N={N}: reference {t_ref:.1f} us ({gb / t_ref * 1e6:.0f} GB/s), "
          f"tcgen05 {t_us:.1f} us ({gb / t_us * 1e6:.0f} GB/s)")

"""Python face of the CPU oracle (oracle/w8a8_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs as the checker.
The product package (vllm_turing_b200) never imports this module.

Arrays are numpy. 16-bit floats travel as uint16 bit patterns (numpy has no bfloat16); `to_bits` / `from_bits` convert
torch tensors. dtype codes are the reference's C-ABI codes (vllm_turing/csrc/w8a8_gemv.cu:346): 0 fp16, 1 bf16.
"""
import ctypes
import os
import subprocess

import numpy as np

_here = os.path.dirname(os.path.abspath(__file__))
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_long
_F = ctypes.c_float


def lib():
    """The oracle library; built from w8a8_oracle.c with the committed Makefile if it is missing or stale."""
    global _lib
    if _lib is None:
        so = os.path.join(_here, "libw8a8_oracle.so")
        src = os.path.join(_here, "w8a8_oracle.c")
        if not os.path.exists(so) or (os.path.exists(src) and os.path.getmtime(so) < os.path.getmtime(src)):
            subprocess.run(["make", "-C", _here, "libw8a8_oracle.so"], check=True, capture_output=True)
        L = ctypes.CDLL(so)
        sig = {
            "orc_gemm_s32": [_P, _P, _P, _I, _I, _I],
            "orc_dequant": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I],
            "orc_dequant_big": [_P, _P, _P, _P, _I, _I, _I],
            "orc_scaled_mm": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I],
            "orc_quant_rows": [_P, _P, _P, _I, _I, _I],
            "orc_weight_quant": [_P, _P, _P, _I, _I],
            "orc_all_reduce": [_P, _I, _P, _L, _I],
            "orc_add_rms_norm_quant": [_P, _P, _P, _F, _P, _P, _P, _I, _I, _I],
            "orc_row_linear_tp": [_I, _P, _P, _P, _P, _P, _P, _F, _P, _P, _P, _I, _I, _I, _I],
            "orc_silu_mul_quant": [_P, _P, _P, _I, _I, _I],
            "orc_all_gather": [_P, _I, _P, _L],
            "orc_lmhead_quant": [_P, _P, _P, _I, _I, _I],
            "orc_w8a16": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I],
            "orc_ar8_quant": [_P, _P, _L],
            "orc_ar8_dequant_sum": [_P, _P, _L, _I],
            "orc_set_threads": [_I],
            "orc_num_threads": [],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _I if name == "orc_num_threads" else None
        _lib = L
    return _lib


def _p(x):
    assert x.flags["C_CONTIGUOUS"], "oracle inputs must be contiguous"
    return x.ctypes.data_as(ctypes.c_void_p)


def set_threads(n):
    lib().orc_set_threads(int(n))


def num_threads():
    return lib().orc_num_threads()


# ---- torch <-> numpy bit patterns ------------------------------------------------------------------------------------
def to_bits(t):
    """torch fp16/bf16 tensor -> numpy uint16 bit patterns (CPU copy)."""
    import torch
    assert t.dtype in (torch.float16, torch.bfloat16)
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(b, dtype):
    """numpy uint16 bit patterns -> torch tensor of `dtype` (fp16/bf16) on the CPU."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(dtype)


def bits_to_float(b, dtype_code):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    if dtype_code == 1:
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


# ---- operations -----------------------------------------------------------------------------------------------------
def gemm_s32(a, w):
    """int32 [M, N] = a int8 [M, K] . w int8 [N, K]^T (exact)."""
    M, K = a.shape
    N = w.shape[0]
    acc = np.empty((M, N), np.int32)
    lib().orc_gemm_s32(_p(a), _p(w), _p(acc), M, N, K)
    return acc


def dequant(acc, sa, sw, bias=None, dtype=1):
    M, N = acc.shape
    out = np.empty((M, N), np.uint16)
    sa = np.ascontiguousarray(sa, np.float32).reshape(-1)
    sw = np.ascontiguousarray(sw, np.float32).reshape(-1)
    lib().orc_dequant(_p(acc), _p(sa), _p(sw), _p(bias) if bias is not None else None, _p(out), M, N,
                      int(sa.size > 1), int(sw.size > 1), dtype)
    return out


def dequant_big(acc, sa, sw, dtype=1):
    """The prefill epilogue order sa * (sw * acc) (vllm_turing/csrc/w8a8_big.cu:26-35)."""
    acc = np.ascontiguousarray(acc, np.int32)
    M, N = acc.shape
    out = np.empty((M, N), np.uint16)
    lib().orc_dequant_big(_p(acc), _p(np.ascontiguousarray(sa, np.float32).reshape(-1)),
                          _p(np.ascontiguousarray(sw, np.float32).reshape(-1)), _p(out), M, N, dtype)
    return out


def scaled_mm(a, w, sa, sw, bias=None, dtype=1):
    """bits [M, N] of the W8A8 linear (GEMM + per-token x per-channel dequant)."""
    M, K = a.shape
    N = w.shape[0]
    out = np.empty((M, N), np.uint16)
    sa = np.ascontiguousarray(sa, np.float32).reshape(-1)
    sw = np.ascontiguousarray(sw, np.float32).reshape(-1)
    lib().orc_scaled_mm(_p(a), _p(w), _p(sa), _p(sw), _p(bias) if bias is not None else None, _p(out), M, N, K,
                        int(sa.size > 1), int(sw.size > 1), dtype)
    return out


def quant_rows(x_bits, dtype=1):
    """(int8 [M, N], float32 [M]) per-token dynamic quantisation of 16-bit rows."""
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    M, N = x_bits.shape
    q = np.empty((M, N), np.int8)
    s = np.empty((M,), np.float32)
    lib().orc_quant_rows(_p(x_bits), _p(q), _p(s), M, N, dtype)
    return q, s


def weight_quant(w):
    """(int8 [N, K], float32 [N]) per-output-channel weight quantisation of a float32 [N, K] weight."""
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    q = np.empty((N, K), np.int8)
    s = np.empty((N,), np.float32)
    lib().orc_weight_quant(_p(w), _p(q), _p(s), N, K)
    return q, s


def all_reduce(parts, dtype=1):
    parts = [np.ascontiguousarray(p, np.uint16) for p in parts]
    out = np.empty_like(parts[0])
    arr = (ctypes.c_void_p * len(parts))(*[p.ctypes.data for p in parts])
    lib().orc_all_reduce(arr, len(parts), _p(out), parts[0].size, dtype)
    return out


def add_rms_norm_quant(x_bits, residual_bits, weight_bits, eps, dtype=1, want_normed=False):
    """-> (new residual bits, q int8, scales float32, normed bits or None); inputs are not modified."""
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    res = np.array(residual_bits, np.uint16, copy=True)
    wb = np.ascontiguousarray(weight_bits, np.uint16)
    M, N = x_bits.shape
    q = np.empty((M, N), np.int8)
    s = np.empty((M,), np.float32)
    normed = np.empty((M, N), np.uint16) if want_normed else None
    lib().orc_add_rms_norm_quant(_p(x_bits), _p(res), _p(wb), float(eps), _p(q), _p(s),
                                 _p(normed) if want_normed else None, M, N, dtype)
    return res, q, s, normed


def row_linear_tp_big(a_list, w_list, sa_list, sw_list, residual_bits, weight_bits, eps, dtype=1):
    """The TP layer tail with the prefill GEMM's dequant order (sa * (sw * acc), vllm_turing/csrc/w8a8_big.cu:26-35,
    the order the reference's scaled_mm takes for M > 32, vllm_turing/w8a8.py:108-117): per rank gemm_s32 then
    dequant_big, the rank-ordered all-reduce, then add_rms_norm_quant -> (new residual, q, scales, reduced)."""
    parts = [dequant_big(gemm_s32(a, w), sa, sw, dtype) for a, w, sa, sw in zip(a_list, w_list, sa_list, sw_list)]
    red = all_reduce(parts, dtype)
    res, q, s, _ = add_rms_norm_quant(red, residual_bits, weight_bits, eps, dtype)
    return res, q, s, red


def row_linear_tp(a_list, w_list, sa_list, sw_list, residual_bits, weight_bits, eps, dtype=1):
    """The whole TP layer tail -> (new residual, q, scales, reduced)."""
    n = len(a_list)
    M, K = a_list[0].shape
    N = w_list[0].shape[0]
    res = np.array(residual_bits, np.uint16, copy=True)
    q = np.empty((M, N), np.int8)
    s = np.empty((M,), np.float32)
    red = np.empty((M, N), np.uint16)
    keep = [[np.ascontiguousarray(x) for x in lst] for lst in (a_list, w_list, sa_list, sw_list)]  # alive
    arrs = [(ctypes.c_void_p * n)(*[x.ctypes.data for x in lst]) for lst in keep]
    wb = np.ascontiguousarray(weight_bits)
    lib().orc_row_linear_tp(n, arrs[0], arrs[1], arrs[2], arrs[3], _p(res), _p(wb),
                            float(eps), _p(q), _p(s), _p(red), M, N, K, dtype)
    return res, q, s, red


def silu_mul_quant(gu_bits, dtype=0):
    gu_bits = np.ascontiguousarray(gu_bits, np.uint16)
    M, I2 = gu_bits.shape
    q = np.empty((M, I2 // 2), np.int8)
    s = np.empty((M,), np.float32)
    lib().orc_silu_mul_quant(_p(gu_bits), _p(q), _p(s), M, I2 // 2, dtype)
    return q, s


def all_gather(payloads):
    payloads = [np.ascontiguousarray(p, np.uint8) for p in payloads]
    m = payloads[0].size
    out = np.empty(len(payloads) * m, np.uint8)
    arr = (ctypes.c_void_p * len(payloads))(*[p.ctypes.data for p in payloads])
    lib().orc_all_gather(arr, len(payloads), _p(out), m)
    return out


def lmhead_quant(w, device="cpu"):
    """(int8 [N, K], float32 [N]) per-row quantisation of the LM head (vllm_turing/lmhead.py:52-61) as torch computes
    it on `device`: "cuda" divides by 127 as a multiplication by its float32 reciprocal, "cpu" divides."""
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    q = np.empty((N, K), np.int8)
    s = np.empty((N,), np.float32)
    lib().orc_lmhead_quant(_p(w), _p(q), _p(s), N, K, int(device == "cuda"))
    return q, s


def w8a16(x_bits, w, s, bias_bits=None, dtype=1, want_acc=False):
    """bits [M, N] of the W8A16 LM head, plus (acc, mag) float64 [M, N] when want_acc: the exact sums and the sums of
    |products| (the scale of any fp32 summation error)."""
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    w = np.ascontiguousarray(w, np.int8)
    s = np.ascontiguousarray(s, np.float32).reshape(-1)
    M, K = x_bits.shape
    N = w.shape[0]
    out = np.empty((M, N), np.uint16)
    acc = np.empty((M, N), np.float64) if want_acc else None
    mag = np.empty((M, N), np.float64) if want_acc else None
    bias_bits = np.ascontiguousarray(bias_bits, np.uint16) if bias_bits is not None else None
    lib().orc_w8a16(_p(x_bits), _p(w), _p(s), _p(bias_bits) if bias_bits is not None else None, _p(out),
                    _p(acc) if want_acc else None, _p(mag) if want_acc else None, M, N, K, dtype)
    return (out, acc, mag) if want_acc else out


def w8a16_close(got_bits, want_bits, mag, s, dtype=1, rel_sum=2.0 ** -16):
    """The W8A16 parity test: |got - want| <= 1 unit in the last place of the 16-bit type at |want| plus
    rel_sum * s[n] * mag[m, n] (fp32 summation-order error, generously bounded). Returns the worst ratio of error to
    tolerance (<= 1 passes)."""
    g = bits_to_float(got_bits, dtype).astype(np.float64)
    w = bits_to_float(want_bits, dtype).astype(np.float64)
    mant = 8 if dtype == 1 else 11
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(w), 1e-30))) - (mant - 1))
    tol = ulp + rel_sum * np.abs(np.asarray(s, np.float64).reshape(1, -1)) * mag
    return float(np.max(np.abs(g - w) / np.maximum(tol, 1e-30))) if g.size else 0.0


def ar8_quant(x_bits):
    """uint8 packed block [n + n / 64] of fp16 bits x [n] (n % 128 == 0): int8 values, then fp16 scales per 128
    (vllm_turing/csrc/host_ar.cu:138-160)."""
    x_bits = np.ascontiguousarray(x_bits, np.uint16).reshape(-1)
    n = x_bits.size
    packed = np.empty(n + n // 64, np.uint8)
    lib().orc_ar8_quant(_p(x_bits), _p(packed), n)
    return packed


def ar8_dequant_sum(blocks):
    """fp16 bits [n] = rank-ordered float32 sum of the dequantised packed blocks (host_ar.cu:163-180)."""
    blocks = [np.ascontiguousarray(b, np.uint8) for b in blocks]
    blk = blocks[0].size
    n = blk * 64 // 65
    g = np.ascontiguousarray(np.concatenate(blocks))
    out = np.empty(n, np.uint16)
    lib().orc_ar8_dequant_sum(_p(g), _p(out), n, len(blocks))
    return out

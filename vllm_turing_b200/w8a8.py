"""INT8 W8A8 GEMM behind vLLM's cutlass_scaled_mm on B200 (sm_100a).

vLLM's W8A8 int8 linear layers call vllm._custom_ops.cutlass_scaled_mm(a, b, scale_a, scale_b, out_dtype, bias). As in
the reference (vllm_turing/w8a8.py:125-150), the wrapper is replaced by one that runs the custom op
vllm_turing::scaled_mm_ with the same arguments, dispatching by M at run time (also inside torch.compile / CUDA-graph
capture, where M is concrete):
  - M <= VLLM_TURING_GEMV_MAX_M (default 0, i.e. off): the streamed dp4a GEMV (csrc/gemv_core.cuh),
  - M <= VLLM_TURING_MMA_MAX_M (default 32): the small-M tcgen05 kernel (weights as the MMA's A operand, stream-K over
    the SMs); on B200 it streams decode weights at least as fast as the dp4a GEMV at every M from 1 to 32, so it is
    the default decode path (the reference's default, GEMV up to 12 rows, suits its sm_75 part),
  - larger M (prefill): the tcgen05 kind::i8 GEMM with TMEM accumulators (VLLM_TURING_BIG=0 keeps vLLM's),
  - anything else (non-16-aligned shapes, other dtypes): vLLM's own op.
The kernels live in libvllm_turing_b200.so, loaded with ctypes (no torch C++ ABI involved), as the reference does.
"""
import os

import torch

from . import _build

MAX_M = int(os.environ.get("VLLM_TURING_GEMV_MAX_M", "0"))
MMA_MAX_M = min(int(os.environ.get("VLLM_TURING_MMA_MAX_M", "32")), 32)
BIG = os.environ.get("VLLM_TURING_BIG", "1") != "0"
_ws = {}   # device -> persistent zeroed split-K workspace (graph capture keeps its address)


def lib():
    return _build.load()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(dt):
    return 0 if dt == torch.float16 else 1


def gemv_ok(out, a, b, sa, sb, bias, max_m=None):
    """The GEMV path's layout requirements (vllm_turing/w8a8.py:38-46, same checks)."""
    M, K = a.shape
    return (1 <= M <= (MAX_M if max_m is None else max_m) and K % 16 == 0 and a.dtype == torch.int8
            and a.is_contiguous() and b.dtype == torch.int8 and b.stride(0) == 1 and b.stride(1) == K
            and out.is_contiguous() and out.dtype in (torch.float16, torch.bfloat16)
            and sa.dtype == torch.float32 and sb.dtype == torch.float32
            and sa.numel() in (1, M) and sb.numel() in (1, b.shape[1])
            and a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0
            and (bias is None or (bias.dtype == out.dtype and bias.is_contiguous())))


def workspace(device, M, N):
    """Persistent zeroed split-K workspace for this device (GEMV and tensor-core decode), grown outside capture only."""
    need = max(lib().w8a8_gemv_ws_bytes(M, N), lib().w8a8_mma_ws_bytes(M, N))
    ws = _ws.get(device)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("vllm_turing_b200: split-K workspace must be sized before CUDA graph capture")
        ws = _ws[device] = torch.zeros(max(need, 8 << 20), dtype=torch.uint8, device=device)
    return ws


def interleave_gate_up(w, sw):
    """The gate/up weight [2I, K] (gate rows, then up rows) and its scales [2I] in the row order gate_up_silu_quant
    takes: 128-row tile t = gate rows 64t..64t+63, then up rows 64t..64t+63. Made once, when the weights are loaded."""
    n2, K = w.shape
    I = n2 // 2
    if n2 != 2 * I or I % 64:
        raise ValueError("interleave_gate_up: 2I rows with I % 64 == 0")
    wi = torch.stack((w[:I].reshape(I // 64, 64, K), w[I:].reshape(I // 64, 64, K)), dim=1).reshape(n2, K)
    s = sw.reshape(-1)
    si = torch.stack((s[:I].reshape(I // 64, 64), s[I:].reshape(I // 64, 64)), dim=1).reshape(n2)
    return wi.contiguous(), si.contiguous()


_silu_ws = {}   # device -> zeroed workspace of gate_up_silu_quant (graph capture keeps its address)


def gate_up_silu_quant(a, w_il, sa, sw_il, q=None, scales=None, dtype=torch.bfloat16):
    """(q int8 [M, I], scales float32 [M, 1]) = silu_mul_quant(scaled_mm(a, w.t(), sa, sw)) in one kernel, for the
    interleaved weight of interleave_gate_up. Bit-identical to the two-op chain."""
    M, K = a.shape
    I = w_il.shape[0] // 2
    L = lib()
    need = L.vt_gate_up_silu_quant_ws_bytes(M, I)
    ws = _silu_ws.get(a.device)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("vllm_turing_b200: gate_up_silu_quant workspace must be sized before CUDA graph capture")
        ws = _silu_ws[a.device] = torch.zeros(max(need, 4 << 20), dtype=torch.uint8, device=a.device)
    q = q if q is not None else torch.empty(M, I, dtype=torch.int8, device=a.device)
    scales = scales if scales is not None else torch.empty(M, 1, dtype=torch.float32, device=a.device)
    rc = L.vt_gate_up_silu_quant(a.data_ptr(), w_il.data_ptr(), sa.data_ptr(), sw_il.data_ptr(), q.data_ptr(),
                                 scales.data_ptr(), M, I, K, int(sa.numel() > 1), _dtype_code(dtype), ws.data_ptr(),
                                 ws.numel(), _stream())
    if rc != 0:
        raise RuntimeError(f"vt_gate_up_silu_quant failed: {rc}")
    return q, scales


def gemv(out, a, b, sa, sb, bias):
    """out[M, N] = (a . w^T) * sa * sb (+ bias), w = b.t() the row-major [N, K] weight."""
    M, K = a.shape
    N = b.shape[1]
    ws = workspace(a.device, M, N)
    rc = lib().w8a8_gemv_ws(a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(),
                            bias.data_ptr() if bias is not None else None, out.data_ptr(), M, N, K,
                            int(sa.numel() > 1), int(sb.numel() > 1), _dtype_code(out.dtype), ws.data_ptr(),
                            ws.numel(), _stream())
    if rc != 0:
        raise RuntimeError(f"w8a8_gemv launch failed: {rc}")


def gemm_s32(a, w):
    """int32 accumulators a [M, K] . w [N, K]^T (parity checks): the GEMV for small M, the tcgen05 GEMM above."""
    M, K = a.shape
    N = w.shape[0]
    acc = torch.empty(M, N, dtype=torch.int32, device=a.device)
    L = lib()
    if M <= 16:
        rc = L.vt_gemv_s32(a.data_ptr(), w.data_ptr(), acc.data_ptr(), M, N, K, _stream())
    else:
        if not hasattr(L, "vt_gemm_s32"):
            raise RuntimeError("vllm_turing_b200: tensor-core GEMM not built")
        rc = L.vt_gemm_s32(a.data_ptr(), w.data_ptr(), acc.data_ptr(), M, N, K, _stream())
    if rc != 0:
        raise RuntimeError(f"int32 GEMM failed: {rc}")
    return acc


def _has(name):
    return hasattr(lib(), name)


def mma_ok(out, a, b, sa, sb, bias):
    return a.shape[0] > MAX_M and _has("w8a8_mma_ws") and gemv_ok(out, a, b, sa, sb, bias, MMA_MAX_M)


def mma(out, a, b, sa, sb, bias):
    M, K = a.shape
    N = b.shape[1]
    ws = workspace(a.device, M, N)
    rc = lib().w8a8_mma_ws(a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(),
                           bias.data_ptr() if bias is not None else None, out.data_ptr(), M, N, K,
                           int(sa.numel() > 1), int(sb.numel() > 1), _dtype_code(out.dtype), ws.data_ptr(),
                           ws.numel(), _stream())
    if rc != 0:
        raise RuntimeError(f"w8a8_mma launch failed: {rc}")


def block_weight(w):
    """The row-major weight [N, K] int8 in the tile-blocked layout mma_blocked reads: [N/128, K/128, 128, 128], each
    128 x 128 block contiguous and a 128-row tile's blocks in K order (made once, at load time)."""
    N, K = w.shape
    if N % 128 or K % 128:
        raise ValueError("block_weight: N and K must be multiples of 128")
    return w.reshape(N // 128, 128, K // 128, 128).permute(0, 2, 1, 3).contiguous()


def mma_blocked(out, a, wb, sa, sb, bias=None):
    """out[M, N] = (a . w^T) * sa * sb (+ bias) for the weight of block_weight(w) (the decode GEMM, M <= 32)."""
    M, K = a.shape
    N = wb.shape[0] * 128
    ws = workspace(a.device, M, N)
    rc = lib().w8a8_mma_blocked_ws(a.data_ptr(), wb.data_ptr(), sa.data_ptr(), sb.data_ptr(),
                                   bias.data_ptr() if bias is not None else None, out.data_ptr(), M, N, K,
                                   int(sa.numel() > 1), int(sb.numel() > 1), _dtype_code(out.dtype), ws.data_ptr(),
                                   ws.numel(), _stream())
    if rc != 0:
        raise RuntimeError(f"w8a8_mma_blocked failed: {rc}")


def big_ok(out, a, b, sa, sb, bias):
    """The prefill kernel's requirements (vllm_turing/w8a8.py:58-66, same checks)."""
    M, K = a.shape
    N = b.shape[1]
    return (BIG and _has("w8a8_big") and M > MMA_MAX_M and bias is None and K % 16 == 0 and N % 16 == 0
            and a.dtype == torch.int8 and a.is_contiguous() and b.dtype == torch.int8 and b.stride(0) == 1
            and b.stride(1) == K and out.is_contiguous() and out.dtype in (torch.float16, torch.bfloat16)
            and sa.dtype == torch.float32 and sb.dtype == torch.float32 and sa.numel() == M and sb.numel() == N
            and sa.is_contiguous() and sb.is_contiguous() and a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0)


def big(out, a, b, sa, sb):
    M, K = a.shape
    N = b.shape[1]
    rc = lib().w8a8_big(a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(), out.data_ptr(), M, N, K,
                        _dtype_code(out.dtype), _stream())
    if rc != 0:
        raise RuntimeError(f"w8a8_big failed: {rc}")


_lib_def = torch.library.Library("vllm_turing", "DEF")
_lib_def.define("scaled_mm_(Tensor(a!) out, Tensor a, Tensor b, Tensor a_scales, Tensor b_scales, Tensor? bias) -> ()")


@torch.library.impl(_lib_def, "scaled_mm_", "CUDA")
def _scaled_mm_cuda(out, a, b, a_scales, b_scales, bias):
    if gemv_ok(out, a, b, a_scales, b_scales, bias):
        gemv(out, a, b, a_scales, b_scales, bias)
    elif mma_ok(out, a, b, a_scales, b_scales, bias):
        mma(out, a, b, a_scales, b_scales, bias)
    elif big_ok(out, a, b, a_scales, b_scales, bias):
        big(out, a, b, a_scales, b_scales)
    else:
        torch.ops._C.cutlass_scaled_mm(out, a, b, a_scales, b_scales, bias)


@torch.library.register_fake("vllm_turing::scaled_mm_")
def _scaled_mm_fake(out, a, b, a_scales, b_scales, bias):
    return None


def scaled_mm(a, b, scale_a, scale_b, out_dtype, bias=None):
    """vLLM's cutlass_scaled_mm contract (vllm_turing/w8a8.py:136-147): a [..., K] int8, b [K, N] view."""
    assert out_dtype is torch.bfloat16 or out_dtype is torch.float16
    assert bias is None or bias.numel() == b.shape[1] and bias.dtype == out_dtype
    target_shape = (*a.shape[:-1], b.shape[1])
    a = a.view(-1, a.shape[-1])
    out = torch.empty((a.shape[0], b.shape[1]), dtype=out_dtype, device=a.device)
    torch.ops.vllm_turing.scaled_mm_(out, a, b, scale_a, scale_b, bias)
    return out.view(*target_shape)


def install():
    """Replace vllm._custom_ops.cutlass_scaled_mm on B200 (compute capability 10.0)."""
    from vllm import _custom_ops as ops
    from vllm.platforms import current_platform

    if getattr(ops.cutlass_scaled_mm, "_vllm_turing", False):
        return
    cap = current_platform.get_device_capability()
    if cap is None or cap.to_int() != 100:
        return
    orig = ops.cutlass_scaled_mm

    def cutlass_scaled_mm(a, b, scale_a, scale_b, out_dtype, bias=None):
        if not (b.shape[0] % 16 == 0 and b.shape[1] % 16 == 0):
            return orig(a, b, scale_a, scale_b, out_dtype, bias)
        return scaled_mm(a, b, scale_a, scale_b, out_dtype, bias)

    cutlass_scaled_mm._vllm_turing = True
    cutlass_scaled_mm._orig = orig
    ops.cutlass_scaled_mm = cutlass_scaled_mm

"""Per-token dynamic int8 quantisation of W8A8 activations, and the fused residual add + RMSNorm + quantisation.

quant_torch is the reference's formula (vllm_turing/quantfuse.py:18-24: float32 absmax per row, scale = absmax / 127,
round-half-even of x * (127 / absmax), clamped); while torch.compile traces, vLLM's scaled_int8_quant is replaced by it
so inductor fuses it into the producer kernel (quantfuse.py:35-43). Eager calls of the dynamic symmetric case run the
sm_100a kernel vt_scaled_int8_quant, bit-exact to quant_torch (torch evaluates 127 / absmax as
absmax.reciprocal() * 127; the kernel does the same two roundings). rms_norm_dynamic_per_token_quant is the B200
kernel behind the call the reference makes at vllm_turing/tailoverlap.py:200. VLLM_TURING_QUANTFUSE=0 disables.
"""
import os

import torch

from . import _build

ENABLED = os.environ.get("VLLM_TURING_QUANTFUSE", "1") != "0"


def quant_torch(x: torch.Tensor):
    """Per-row dynamic symmetric int8 quantisation: (int8 like x, float32 scales [rows, 1])."""
    shape = x.shape
    xf = x.reshape(-1, shape[-1]).float()
    absmax = xf.abs().amax(dim=-1, keepdim=True)
    q = torch.round(xf * (127.0 / absmax)).clamp(-128.0, 127.0).to(torch.int8)
    return q.reshape(shape), absmax / 127.0


def _code(dt):
    if dt not in (torch.float16, torch.bfloat16):
        raise TypeError(f"vllm_turing_b200: unsupported dtype {dt}")
    return 0 if dt == torch.float16 else 1


def scaled_int8_quant_cuda(x: torch.Tensor):
    """(int8 [rows, N], float32 [rows, 1]) on the GPU."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    M, N = x2.shape
    q = torch.empty(M, N, dtype=torch.int8, device=x.device)
    s = torch.empty(M, 1, dtype=torch.float32, device=x.device)
    rc = _build.load().vt_scaled_int8_quant(x2.data_ptr(), q.data_ptr(), s.data_ptr(), M, N, _code(x.dtype),
                                            torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"vt_scaled_int8_quant failed: {rc}")
    return q.view(x.shape), s


def rms_norm_dynamic_per_token_quant(x, weight, eps, residual, normed=None, q=None, s=None):
    """residual += x (in place); returns (q int8, scales float32 [rows, 1]) of RMSNorm(residual) * weight.
    The contract of vLLM's op as the reference calls it (vllm_turing/tailoverlap.py:200-201); q / s are written in
    place when given (static buffers of a captured step)."""
    M, N = residual.shape
    q = q if q is not None else torch.empty(M, N, dtype=torch.int8, device=x.device)
    s = s if s is not None else torch.empty(M, 1, dtype=torch.float32, device=x.device)
    if q.shape != (M, N) or q.dtype != torch.int8 or not q.is_contiguous() or s.numel() != M:
        raise ValueError("rms_norm_dynamic_per_token_quant: q must be int8 [M, N] contiguous and s hold M floats")
    rc = _build.load().vt_rms_norm_quant(x.data_ptr(), residual.data_ptr(), weight.data_ptr(), float(eps),
                                         q.data_ptr(), s.data_ptr(), normed.data_ptr() if normed is not None else None,
                                         M, N, _code(x.dtype), torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"vt_rms_norm_quant failed: {rc}")
    return q, s


def install():
    if not ENABLED:
        return
    from vllm import _custom_ops as ops
    if getattr(ops.scaled_int8_quant, "_vllm_turing", False):
        return
    orig = ops.scaled_int8_quant

    def scaled_int8_quant(input, scale=None, azp=None, symmetric=True):
        if scale is None and azp is None and symmetric:
            if torch.compiler.is_compiling():
                q, s = quant_torch(input)
                return q, s, None
            if input.is_cuda and input.dtype in (torch.float16, torch.bfloat16) and input.shape[-1] % 4 == 0 \
                    and torch.cuda.get_device_capability(input.device) == (10, 0):
                q, s = scaled_int8_quant_cuda(input)
                return q, s, None
        return orig(input, scale, azp, symmetric)

    scaled_int8_quant._vllm_turing = True
    scaled_int8_quant._orig = orig
    ops.scaled_int8_quant = scaled_int8_quant

    # the traced graphs differ from upstream's: their own AOT compile cache key (quantfuse.py:45-55)
    try:
        from vllm.compilation import caching
    except ImportError:
        return
    if hasattr(caching, "aot_compile_hash_factors") and not getattr(caching, "_vllm_turing_quantfuse", False):
        orig_factors = caching.aot_compile_hash_factors

        def aot_compile_hash_factors(vllm_config):
            return [*orig_factors(vllm_config), "vllm_turing_quantfuse"]

        caching.aot_compile_hash_factors = aot_compile_hash_factors
        caching._vllm_turing_quantfuse = True

"""The per-token tail of a tensor-parallel decoder layer (out_proj -> all-reduce -> residual add + RMSNorm + int8
quant -> gate_up -> SiLU * up + quant -> down_proj -> all-reduce) as one opaque op, chunked for prefill so the
all-reduces of chunk i overlap the GEMMs of chunk i + 1 (the reference's vllm_turing/tailoverlap.py:153-259).

B200 version of each step: the GEMMs are w8a8.scaled_mm (tcgen05 / GEMV kernels), the all-reduces go through the
P2P communicator of the TP group (hostar: one-shot / two-shot kernels, which take a handful of SMs and no NCCL), the
post-attention norm + residual add + quantisation is quantfuse.rms_norm_dynamic_per_token_quant (csrc/norm_quant.cu)
and SiLU * up + quantisation is silu_mul_quant (csrc/norm_quant.cu). For decode-sized batches the TP all-reduce and
the norm are fused further into one kernel (fused.row_linear_norm_quant) when the communicator is available.

Chunk bounds at the fractions VLLM_TURING_TAIL_SPLIT of the batch (default 1/6, 1/2, 5/6; batches under 4096 tokens:
halves, tailoverlap.py:220-224), the side stream at high priority (tailoverlap.py:139-144). VLLM_TURING_TAIL=1
enables; VLLM_TURING_TAIL_MIN (default 2048) is the smallest batch chunked; VLLM_TURING_TAIL_FUSED=0 keeps the model's
own norm and activation.
"""
import logging
import os
import types

import torch

from . import _build

logger = logging.getLogger("vllm.turing")
ENABLED = os.environ.get("VLLM_TURING_TAIL", "0") == "1"
SPLIT = sorted(float(f) for f in os.environ.get("VLLM_TURING_TAIL_SPLIT", "0.16667,0.5,0.83333").split(",") if f)
SPLIT = tuple(f for f in SPLIT if 0.0 < f < 1.0) or (0.5,)
MAX_PART = max(b - a for a, b in zip((0.0, *SPLIT), (*SPLIT, 1.0)))
MIN_TOKENS = int(os.environ.get("VLLM_TURING_TAIL_MIN", "2048"))
FUSED = os.environ.get("VLLM_TURING_TAIL_FUSED", "1") != "0"
_REG = []
_STREAMS = {}


def silu_mul_quant(gate_up: torch.Tensor, q=None, sc=None):
    """(M, 2I) fp16 / bf16 -> int8 (M, I) of SiLU(gate) * up and its per-row scales (M, 1) float32, written into q / sc
    when given (e.g. the static buffers of a captured decode step)."""
    M, I2 = gate_up.shape
    q = q if q is not None else torch.empty(M, I2 // 2, dtype=torch.int8, device=gate_up.device)
    sc = sc if sc is not None else torch.empty(M, 1, dtype=torch.float32, device=gate_up.device)
    if q.shape != (M, I2 // 2) or q.dtype != torch.int8 or not q.is_contiguous() or sc.numel() != M:
        raise ValueError("silu_mul_quant: q must be int8 [M, I] contiguous and sc hold M floats")
    code = 0 if gate_up.dtype == torch.float16 else 1
    rc = _build.load().vt_silu_mul_quant(gate_up.data_ptr(), q.data_ptr(), sc.data_ptr(), M, I2 // 2, code,
                                         torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"silu_mul_quant failed: {rc}")
    return q, sc


def chunk_bounds(n):
    """Row bounds of the chunks of an n-token batch (multiples of 16, as tailoverlap.py:220-224)."""
    fr = SPLIT if n >= 4096 else (0.5,)
    b = [0] + [int(f * n) // 16 * 16 for f in fr] + [n]
    return [x for i, x in enumerate(b) if i == 0 or x > b[i - 1]]


def _side_stream(dev):
    s = _STREAMS.get(dev)
    if s is None:
        s = _STREAMS[dev] = torch.cuda.Stream(device=dev, priority=-1)
    return s


def _proj(linear, x):
    """The GEMM of a RowParallelLinear without its all-reduce (this rank's partial sum)."""
    bias = None if (linear.tp_rank > 0 or linear.skip_bias_add) else linear.bias
    return linear.quant_method.apply(linear, x, bias)


def _w8a8_params(layer):
    kernel = getattr(layer.quant_method, "kernel", None) or getattr(getattr(layer, "scheme", None), "kernel", None)
    if kernel is None or not hasattr(kernel, "_get_layer_params"):
        return None
    w_q, w_s, i_s, i_zp, azp = kernel._get_layer_params(layer)
    if i_s is not None or i_zp is not None or azp is not None or w_q.dtype != torch.int8:
        return None
    return w_q, w_s


class _Tail:
    def __init__(self, layer):
        attn = layer.linear_attn if layer.layer_type == "linear_attention" else layer.self_attn
        self.out_proj = attn.out_proj if layer.layer_type == "linear_attention" else attn.o_proj
        self.norm = layer.post_attention_layernorm
        self.mlp = layer.mlp
        self.fused = None

    def _decide(self):
        from . import w8a8
        self.fused = False
        norm_type = type(self.norm).__name__
        if FUSED and norm_type in ("GemmaRMSNorm", "RMSNorm") and self.mlp.gate_up_proj.bias is None:
            p = _w8a8_params(self.mlp.gate_up_proj)
            if p is not None:
                w = self.norm.weight.data
                self.w1 = (1.0 + w.float()).to(w.dtype) if norm_type == "GemmaRMSNorm" else w
                self.w_q, self.w_s = p
                self.actq = False
                dp = self.mlp.down_proj
                if type(self.mlp.act_fn).__name__ == "SiluAndMul" and dp.bias is None:
                    pd = _w8a8_params(dp)
                    if pd is not None:
                        self.wd_q, self.wd_s = pd
                        self.actq = True
                self.fused = True
        self._mm = w8a8.scaled_mm
        logger.info("vllm_turing_b200: layer tail (chunks %s, min %d tokens, fused norm+quant %s)", SPLIT,
                    MIN_TOKENS, self.fused)

    def mlp_partial(self, h, res):
        """res += h in place; the MLP of the normed sum -> this rank's partial down projection."""
        if self.fused is None:
            self._decide()
        if self.fused:
            from .quantfuse import rms_norm_dynamic_per_token_quant
            x_q, x_s = rms_norm_dynamic_per_token_quant(h, self.w1, self.norm.variance_epsilon, res)
            gate_up = self._mm(x_q, self.w_q, x_s, self.w_s, h.dtype)
            if self.actq:
                a_q, a_s = silu_mul_quant(gate_up)
                return self._mm(a_q, self.wd_q, a_s, self.wd_s, h.dtype)
            return _proj(self.mlp.down_proj, self.mlp.act_fn(gate_up))
        x, r = self.norm(h, res)
        if r.data_ptr() != res.data_ptr():
            res.copy_(r)
        gate_up, _ = self.mlp.gate_up_proj(x)
        return _proj(self.mlp.down_proj, self.mlp.act_fn(gate_up))

    def plain(self, attn, residual):
        from vllm.distributed import tensor_model_parallel_all_reduce as ar
        res = residual.clone()
        h = ar(_proj(self.out_proj, attn))
        return ar(self.mlp_partial(h, res)), res

    def chunked(self, attn, residual):
        from vllm.distributed import tensor_model_parallel_all_reduce as ar
        bounds = chunk_bounds(attn.shape[0])
        cur = torch.cuda.current_stream(attn.device)
        comm = _side_stream(attn.device)
        res = residual.clone()
        mid = torch.empty_like(residual)
        out = torch.empty_like(residual)
        held = []

        def reduce_async(y, dst):
            ev = torch.cuda.Event()
            ev.record(cur)
            comm.wait_event(ev)
            held.append(y)
            with torch.cuda.stream(comm):
                dst.copy_(ar(y))
                done = torch.cuda.Event()
                done.record(comm)
            return done

        first = [reduce_async(_proj(self.out_proj, attn[a:b]), mid[a:b]) for a, b in zip(bounds, bounds[1:])]
        for (a, b), done in zip(zip(bounds, bounds[1:]), first):
            cur.wait_event(done)
            reduce_async(self.mlp_partial(mid[a:b], res[a:b]), out[a:b])
        cur.wait_stream(comm)
        held.clear()
        return out, res


_frag = torch.library.Library("vllm_turing", "FRAGMENT")
_frag.define("layer_tail(Tensor attn, Tensor residual, int idx) -> (Tensor, Tensor)")


@torch.library.impl(_frag, "layer_tail", "CUDA")
def _layer_tail(attn, residual, idx):
    t = _REG[idx]
    if attn.shape[0] < MIN_TOKENS or torch.cuda.is_current_stream_capturing():
        return t.plain(attn, residual)
    return t.chunked(attn, residual)


@torch.library.register_fake("vllm_turing::layer_tail")
def _layer_tail_fake(attn, residual, idx):
    return torch.empty_like(residual), torch.empty_like(residual)


def _register(self):
    self._turing_tail = -1
    mlp = getattr(self, "mlp", None)
    if (getattr(self, "use_attn_reduce_scatter_for_moe", False) or getattr(self, "layer_scale", False)
            or mlp is None or not hasattr(mlp, "gate_up_proj") or getattr(mlp, "expert_gate", None) is not None
            or getattr(self, "layer_type", None) not in ("linear_attention", "full_attention")):
        return
    t = _Tail(self)
    if t.out_proj.tp_size > 1 and t.out_proj.reduce_results and mlp.down_proj.reduce_results:
        self._turing_tail = len(_REG)
        _REG.append(t)
        t.out_proj.forward = types.MethodType(lambda m, x: (x, None), t.out_proj)


def _patch_layer_class(L):
    if "_vllm_turing_tail" in L.__dict__:
        return
    L._vllm_turing_tail = True
    if "__init__" in L.__dict__:
        orig_init = L.__init__

        def __init__(self, *args, **kwargs):
            orig_init(self, *args, **kwargs)
            _register(self)

        L.__init__ = __init__
    if "forward" not in L.__dict__:
        return
    orig_fwd = L.forward

    def forward(self, hidden_states, residual, positions, **kwargs):
        if getattr(self, "_turing_tail", -1) < 0:
            return orig_fwd(self, hidden_states, residual, positions, **kwargs)
        if residual is None:
            residual = hidden_states
            hidden_states = self.input_layernorm(hidden_states)
        else:
            hidden_states, residual = self.input_layernorm(hidden_states, residual)
        if self.layer_type == "linear_attention":
            attn = self.linear_attn(hidden_states=hidden_states)
        else:
            attn = self.self_attn(hidden_states=hidden_states, positions=positions)
        return torch.ops.vllm_turing.layer_tail(attn, residual, self._turing_tail)

    L.forward = forward


def install():
    if not ENABLED:
        return
    try:
        from vllm.model_executor.models import qwen3_5, qwen3_next
    except ImportError:
        return
    _patch_layer_class(qwen3_next.Qwen3NextDecoderLayer)
    _patch_layer_class(qwen3_5.Qwen3_5DecoderLayer)
    try:
        from vllm.compilation import caching
    except ImportError:
        return
    if hasattr(caching, "aot_compile_hash_factors") and not getattr(caching, "_vllm_turing_tail", False):
        orig_factors = caching.aot_compile_hash_factors

        def aot_compile_hash_factors(vllm_config):
            return [*orig_factors(vllm_config), "vllm_turing_tail"]

        caching.aot_compile_hash_factors = aot_compile_hash_factors
        caching._vllm_turing_tail = True

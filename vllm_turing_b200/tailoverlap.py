"""The per-token tail of a tensor-parallel decoder layer -- out_proj -> all-reduce -> residual add + RMSNorm + int8
quant -> gate_up -> SiLU * up + int8 quant -> down_proj -> all-reduce -- as the opaque op
vllm_turing::layer_tail(attn, residual, idx) -> (mlp_out, new_residual), the contract of the reference's
vllm_turing/tailoverlap.py:207-217 (op schema, VLLM_TURING_TAIL* switches, chunk fractions).

How it runs here (a plan per layer, resolved at the first call, when the checkpoint has been loaded and processed):

* fused (W8A8 int8 projections with dynamic per-token activation scales, an RMSNorm, SiLU * up, and the TP group's P2P
  communicator from hostar.install): five launches per layer and no separate all-reduce or norm kernel --
    quant(attn) -> TPComm.row_linear(o_proj, residual, norm)    one fused row-linear: GEMM + all-reduce + residual add
                                                                 + RMSNorm + int8 quant (decode: one kernel, prefill:
                                                                 GEMM with the reduce-scatter in its epilogue + reduce
                                                                 / all-gather / norm kernel; from four ranks up the
                                                                 GEMM -> two-shot -> norm chain, measured faster there)
    -> scaled_mm(gate_up) -> silu_mul_quant -> TPComm.row_linear(down_proj)   GEMM + all-reduce, no norm
  The overlap of communication with the GEMMs happens inside those kernels, tile by tile, so no chunking is needed.
* staged (anything else, or a token count the fused kernels do not take): the model's own modules, with each
  row-parallel projection's all-reduce issued on a high-priority side stream; batches of at least
  VLLM_TURING_TAIL_MIN tokens are cut into row chunks (VLLM_TURING_TAIL_SPLIT) so that chunk i's all-reduces overlap
  chunk i + 1's GEMMs (the reference's scheme, kept as the fallback).

VLLM_TURING_TAIL=1 enables the layer patch; VLLM_TURING_TAIL_FUSED=0 forces the staged path.
"""
import logging
import os

import torch

from . import _build

logger = logging.getLogger("vllm.turing")
ENABLED = os.environ.get("VLLM_TURING_TAIL", "0") == "1"
SPLIT = sorted(float(f) for f in os.environ.get("VLLM_TURING_TAIL_SPLIT", "0.16667,0.5,0.83333").split(",") if f)
SPLIT = tuple(f for f in SPLIT if 0.0 < f < 1.0) or (0.5,)
MAX_PART = max(b - a for a, b in zip((0.0, *SPLIT), (*SPLIT, 1.0)))
MIN_TOKENS = int(os.environ.get("VLLM_TURING_TAIL_MIN", "2048"))
FUSED = os.environ.get("VLLM_TURING_TAIL_FUSED", "1") != "0"
_PLANS = []   # index = the idx argument of vllm_turing::layer_tail


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
    """Row bounds of the staged path's chunks of an n-token batch: the SPLIT fractions for n >= 4096, else halves,
    each bound a multiple of 16 rows (the reference's chunking, vllm_turing/tailoverlap.py:220-224)."""
    fr = SPLIT if n >= 4096 else (0.5,)
    b = [0] + [int(f * n) // 16 * 16 for f in fr] + [n]
    return [x for i, x in enumerate(b) if i == 0 or x > b[i - 1]]


class Int8Operands:
    """One W8A8 linear as the B200 kernels take it: w int8 [N, K] row-major (vLLM keeps its [K, N] transposed view)
    and the per-output-channel float32 scales s [N]."""
    __slots__ = ("w", "s")

    def __init__(self, w, s):
        self.w, self.s = w, s

    @staticmethod
    def of(linear):
        """The operands of a vLLM int8 linear with dynamic symmetric per-token activations, else None."""
        scheme = getattr(linear, "scheme", None)
        kernel = getattr(linear.quant_method, "kernel", None) or getattr(scheme, "kernel", None)
        if kernel is None or not hasattr(kernel, "_get_layer_params") or getattr(linear, "bias", None) is not None:
            return None
        w_q, w_s, i_s, i_zp, azp = kernel._get_layer_params(linear)
        if i_s is not None or i_zp is not None or azp is not None or w_q.dtype != torch.int8:
            return None
        w = w_q.t()
        if not w.is_contiguous():
            return None
        return Int8Operands(w, w_s.reshape(-1).float().contiguous())


def _partial(linear, x):
    """A RowParallelLinear's GEMM on x without its all-reduce: this rank's partial sum (bias on rank 0 only)."""
    bias = linear.bias if (linear.tp_rank == 0 and not linear.skip_bias_add) else None
    return linear.quant_method.apply(linear, x, bias)


def _tp_comm():
    try:
        from vllm.distributed import get_tp_group
        return getattr(get_tp_group().device_communicator, "turing_comm", None)
    except Exception:   # noqa: BLE001
        return None


class _SideStream:
    """Per device: the high-priority stream the staged path's all-reduces run on (the block scheduler then hands SMs
    freed by the GEMMs to the all-reduce first)."""
    _streams = {}

    @classmethod
    def of(cls, dev):
        s = cls._streams.get(dev)
        if s is None:
            s = cls._streams[dev] = torch.cuda.Stream(device=dev, priority=-1)
        return s


class TailPlan:
    """One decoder layer's tail. `comm` (a TPComm) and `reduce` (an all-reduce function) may be given; by default
    they come from vLLM's TP group at the first call."""

    def __init__(self, out_proj, norm, mlp, comm=None, reduce=None):
        self.out_proj, self.norm, self.mlp = out_proj, norm, mlp
        self._comm, self._reduce = comm, reduce
        self.fused = None   # resolved at the first call

    # ---- resolution ------------------------------------------------------------------------------------------------
    def _resolve(self):
        if self._comm is None:
            self._comm = _tp_comm()
        if self._reduce is None:
            if self._comm is not None:
                self._reduce = lambda y: self._comm.all_reduce(y)
            else:
                from vllm.distributed import tensor_model_parallel_all_reduce
                self._reduce = tensor_model_parallel_all_reduce
        self.fused = False
        kind = type(self.norm).__name__
        if not (FUSED and self._comm is not None and kind in ("RMSNorm", "GemmaRMSNorm")
                and getattr(self.norm, "variance_size_override", None) is None
                and type(self.mlp.act_fn).__name__ == "SiluAndMul"):
            return
        ops = [Int8Operands.of(x) for x in (self.out_proj, self.mlp.gate_up_proj, self.mlp.down_proj)]
        if any(o is None for o in ops):
            return
        self.o, self.gu, self.dn = ops
        w = self.norm.weight.data
        # GemmaRMSNorm multiplies by 1 + w (float32); the fused kernels take the weight they multiply by
        self.norm_w = (1.0 + w.float()).to(w.dtype) if kind == "GemmaRMSNorm" else w
        self.eps = float(self.norm.variance_epsilon)
        self.fused = True
        logger.info("vllm_turing_b200: layer tail on the fused row-linear kernels (TP %d)", self._comm.world)

    def _fused_ok(self, attn):
        M = attn.shape[0]
        c = self._comm
        if M <= 32:
            return M * attn.shape[1] * 2 <= c.ll_capacity
        return M % (128 * c.world) == 0

    # ---- the fused path --------------------------------------------------------------------------------------------
    def _fused(self, attn, residual):
        from . import w8a8
        from .quantfuse import scaled_int8_quant_cuda
        c = self._comm
        res = residual.clone()
        a_q, a_s = scaled_int8_quant_cuda(attn)
        x_q, x_s = c.row_linear(a_q, self.o.w, a_s, self.o.s, residual=res, norm_w=self.norm_w, eps=self.eps)
        gate_up = w8a8.scaled_mm(x_q, self.gu.w.t(), x_s, self.gu.s.view(-1, 1), attn.dtype)
        h_q, h_s = silu_mul_quant(gate_up)
        out = c.row_linear(h_q, self.dn.w, h_s, self.dn.s,
                           reduced=torch.empty(attn.shape[0], self.dn.w.shape[0], dtype=attn.dtype,
                                               device=attn.device))
        return out, res

    # ---- the staged path -------------------------------------------------------------------------------------------
    def _mlp_partial(self, h, res):
        """res += h (in place); the MLP of RMSNorm(res) -> this rank's partial down projection."""
        x, r = self.norm(h, res)
        if r.data_ptr() != res.data_ptr():
            res.copy_(r)
        gate_up, _ = self.mlp.gate_up_proj(x)
        return _partial(self.mlp.down_proj, self.mlp.act_fn(gate_up))

    def _staged(self, attn, residual, bounds):
        """Two stages per row chunk, each a GEMM on the compute stream followed by its all-reduce on the side stream:
        stage 1 out_proj -> mid[chunk], stage 2 (after its chunk's stage-1 reduction) the MLP -> out[chunk]. The
        compute stream runs every chunk's stage 1 first, so their reductions overlap the later GEMMs."""
        compute = torch.cuda.current_stream(attn.device)
        side = _SideStream.of(attn.device)
        res = residual.clone()
        mid, out = torch.empty_like(residual), torch.empty_like(residual)
        keep = []   # partial sums the side stream still reads, released only after the compute stream waited for it

        def reduce_on_side(y, dst):
            ready = torch.cuda.Event()
            ready.record(compute)
            side.wait_event(ready)
            keep.append(y)
            with torch.cuda.stream(side):
                dst.copy_(self._reduce(y))
                done = torch.cuda.Event()
                done.record(side)
            return done

        chunks = list(zip(bounds, bounds[1:]))
        firsts = [reduce_on_side(_partial(self.out_proj, attn[a:b]), mid[a:b]) for a, b in chunks]
        for (a, b), done in zip(chunks, firsts):
            compute.wait_event(done)
            reduce_on_side(self._mlp_partial(mid[a:b], res[a:b]), out[a:b])
        compute.wait_stream(side)
        keep.clear()
        return out, res

    def __call__(self, attn, residual):
        if self.fused is None:
            self._resolve()
        if self.fused and self._fused_ok(attn):
            return self._fused(attn, residual)
        if attn.shape[0] < MIN_TOKENS or torch.cuda.is_current_stream_capturing():
            return self._staged(attn, residual, [0, attn.shape[0]])
        return self._staged(attn, residual, chunk_bounds(attn.shape[0]))


_frag = torch.library.Library("vllm_turing", "FRAGMENT")
_frag.define("layer_tail(Tensor attn, Tensor residual, int idx) -> (Tensor, Tensor)")


@torch.library.impl(_frag, "layer_tail", "CUDA")
def _layer_tail(attn, residual, idx):
    return _PLANS[idx](attn, residual)


@torch.library.register_fake("vllm_turing::layer_tail")
def _layer_tail_fake(attn, residual, idx):
    return torch.empty_like(residual), torch.empty_like(residual)


def register_plan(plan):
    """Adds a TailPlan; returns the idx that vllm_turing::layer_tail takes for it."""
    _PLANS.append(plan)
    return len(_PLANS) - 1


# ---- vLLM integration: Qwen3-Next / Qwen3.5 decoder layers ------------------------------------------------------------
class _ProjInTail(torch.nn.Module):
    """Stands in for the attention module's out_proj: returns its input (and no bias), so the attention module ends
    before the projection and the projection runs inside the tail (the original module is kept by the plan)."""

    def __init__(self, inner):
        super().__init__()
        self.inner_ref = [inner]   # not a submodule: its parameters stay registered where they were

    def forward(self, x):
        return x, None


def _attn_module(layer):
    return layer.linear_attn if layer.layer_type == "linear_attention" else layer.self_attn


def _eligible(layer):
    mlp = getattr(layer, "mlp", None)
    if getattr(layer, "layer_type", None) not in ("linear_attention", "full_attention") or mlp is None:
        return False
    if not hasattr(mlp, "gate_up_proj") or getattr(mlp, "expert_gate", None) is not None:
        return False   # mixture-of-experts layers keep their own forward
    if getattr(layer, "use_attn_reduce_scatter_for_moe", False) or getattr(layer, "layer_scale", False):
        return False
    proj = _attn_module(layer).out_proj if layer.layer_type == "linear_attention" else _attn_module(layer).o_proj
    return proj.tp_size > 1 and proj.reduce_results and mlp.down_proj.reduce_results


def attach(layer):
    """Gives an eligible decoder layer a plan (sets layer._turing_tail to its idx, -1 otherwise) and moves its
    out_proj into the tail."""
    layer._turing_tail = -1
    if not _eligible(layer):
        return
    attn = _attn_module(layer)
    name = "out_proj" if layer.layer_type == "linear_attention" else "o_proj"
    proj = getattr(attn, name)
    layer._turing_tail = register_plan(TailPlan(proj, layer.post_attention_layernorm, layer.mlp))
    setattr(attn, name, _ProjInTail(proj))


def _tail_forward(orig_forward):
    def forward(self, hidden_states, residual, positions, **kwargs):
        if getattr(self, "_turing_tail", -1) < 0:
            return orig_forward(self, hidden_states, residual, positions, **kwargs)
        if residual is None:
            residual, hidden_states = hidden_states, self.input_layernorm(hidden_states)
        else:
            hidden_states, residual = self.input_layernorm(hidden_states, residual)
        if self.layer_type == "linear_attention":
            core = self.linear_attn(hidden_states=hidden_states)
        else:
            core = self.self_attn(hidden_states=hidden_states, positions=positions)
        return torch.ops.vllm_turing.layer_tail(core, residual, self._turing_tail)
    return forward


def _patch(cls):
    """Attach plans after the class's own __init__ and route its own forward through the tail (a subclass that
    inherits either one inherits the patched version; the mark is checked in the class's own namespace)."""
    if cls.__dict__.get("_vllm_turing_tail"):
        return
    cls._vllm_turing_tail = True
    if "__init__" in cls.__dict__:
        init = cls.__init__

        def __init__(self, *args, **kwargs):
            init(self, *args, **kwargs)
            attach(self)

        cls.__init__ = __init__
    if "forward" in cls.__dict__:
        cls.forward = _tail_forward(cls.forward)


def install():
    if not ENABLED:
        return
    try:
        from vllm.model_executor.models import qwen3_5, qwen3_next
    except ImportError:
        return
    for cls in (qwen3_next.Qwen3NextDecoderLayer, qwen3_5.Qwen3_5DecoderLayer):
        _patch(cls)
    # the compiled layer forward differs from vLLM's: a separate key for vLLM's AOT compile cache
    try:
        from vllm.compilation import caching
    except ImportError:
        return
    factors = getattr(caching, "aot_compile_hash_factors", None)
    if factors is not None and not getattr(factors, "_vllm_turing", False):
        def aot_compile_hash_factors(vllm_config):
            return [*factors(vllm_config), "vllm_turing_tail"]

        aot_compile_hash_factors._vllm_turing = True
        caching.aot_compile_hash_factors = aot_compile_hash_factors

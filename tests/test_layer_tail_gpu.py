"""vllm_turing::layer_tail (tailoverlap.py) on a stand-in decoder layer, on ONE GPU (world-1 communicator):
  - the fused plan (W8A8 projections, RMSNorm, SiLU * up): quant -> fused o_proj row-linear + all-reduce + residual add +
    RMSNorm + int8 quant -> gate_up -> SiLU * up + quant -> fused down row-linear + all-reduce, at a decode size (the
    one-kernel tail) and a prefill size (the GEMM + reduce/all-gather/norm pair); the new residual bit-exact to the
    oracle chain (vllm_turing/tailoverlap.py:138-163 is the reference's sequence), the output within the tolerance the
    +-1 LSB of the re-quantised activations allows;
  - the staged plan (the model's own modules, all-reduces on the side stream), unchunked and chunked into row blocks:
    chunked bit-identical to unchunked, and both close to the fused plan.
The stand-in modules expose what vLLM's do to the plan: RowParallelLinear attributes, a W8A8 kernel with
_get_layer_params, an RMSNorm(x, residual) -> (normed, residual) and SiluAndMul."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist

from oracle import oracle as O

pytestmark = pytest.mark.gpu


class _Kernel:
    def _get_layer_params(self, layer):
        return layer.weight, layer.weight_scale, None, None, None


class _W8A8Method:
    """vLLM's dynamic per-token int8 linear: quantise the input rows, then the W8A8 GEMM."""
    kernel = _Kernel()

    def apply(self, layer, x, bias=None):
        from vllm_turing_b200 import w8a8
        from vllm_turing_b200.quantfuse import scaled_int8_quant_cuda
        q, s = scaled_int8_quant_cuda(x)
        return w8a8.scaled_mm(q, layer.weight, s, layer.weight_scale, x.dtype, bias)


class _RowLinear(torch.nn.Module):
    def __init__(self, w, s):
        super().__init__()
        self.weight = w.t()                      # vLLM's [K, N] view of the row-major [N, K] int8 weight
        self.weight_scale = s.view(-1, 1)
        self.bias = None
        self.tp_rank, self.tp_size, self.reduce_results, self.skip_bias_add = 0, 2, True, False
        self.quant_method = _W8A8Method()

    def forward(self, x):
        return self.quant_method.apply(self, x), None


class RMSNorm(torch.nn.Module):
    def __init__(self, w, eps):
        super().__init__()
        self.weight = torch.nn.Parameter(w, requires_grad=False)
        self.variance_epsilon = eps

    def forward(self, x, residual):
        h = (x.float() + residual.float()).to(x.dtype)
        hf = h.float()
        y = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return (y * self.weight.float()).to(x.dtype), h


class SiluAndMul(torch.nn.Module):
    def forward(self, gu):
        g, u = gu.chunk(2, dim=-1)
        return (torch.nn.functional.silu(g.float()) * u.float()).to(gu.dtype)


class _MLP(torch.nn.Module):
    def __init__(self, gu, dn):
        super().__init__()
        self.gate_up_proj, self.down_proj, self.act_fn = gu, dn, SiluAndMul()


@pytest.fixture(scope="module")
def comm1():
    from vllm_turing_b200 import w8a8  # noqa: F401  (registers vllm_turing::scaled_mm_)
    from vllm_turing_b200.comm import TPComm
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29621")
        dist.init_process_group("gloo", rank=0, world_size=1)
    torch.cuda.set_device(0)
    c = TPComm(dist.group.WORLD, torch.device("cuda", 0))
    yield c
    c.close()


H, I = 1024, 2048


def _layer(seed):
    from vllm_turing_b200.synthetic import quant_per_channel
    g = torch.Generator().manual_seed(seed)
    mats = {}
    for name, (n, k) in (("o", (H, H)), ("gu", (2 * I, H)), ("dn", (H, I))):
        w, s = quant_per_channel(torch.randn(n, k, generator=g) * 0.02)
        mats[name] = (w.contiguous(), s.contiguous())
    norm_w = (1.0 + torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    return mats, norm_w


def _plan(mats, norm_w, comm, allow_fused=True):
    from vllm_turing_b200 import tailoverlap
    d = {k: (w.cuda(), s.cuda()) for k, (w, s) in mats.items()}
    o_proj = _RowLinear(*d["o"])
    mlp = _MLP(_RowLinear(*d["gu"]), _RowLinear(*d["dn"]))
    norm = RMSNorm(norm_w.cuda(), 1e-6)
    plan = tailoverlap.TailPlan(o_proj, norm, mlp, comm=comm)
    if not allow_fused:
        plan._resolve()
        plan.fused = False
    return plan, tailoverlap.register_plan(plan)


def _oracle_tail(attn, residual, mats, norm_w, big):
    """The reference's tail sequence on the CPU oracle: quant(attn) -> o_proj -> (world 1: no all-reduce) -> residual
    add + RMSNorm + quant -> gate_up -> SiLU * up + quant -> down."""
    mm = (lambda a, w, sa, sw: O.dequant_big(O.gemm_s32(a, w), sa, sw, 1)) if big else \
        (lambda a, w, sa, sw: O.scaled_mm(a, w, sa, sw, None, 1))
    a_q, a_s = O.quant_rows(O.to_bits(attn), 1)
    h = mm(a_q, mats["o"][0].numpy(), a_s, mats["o"][1].numpy())
    res, x_q, x_s, _ = O.add_rms_norm_quant(h, O.to_bits(residual), O.to_bits(norm_w), 1e-6, 1)
    gu = mm(x_q, mats["gu"][0].numpy(), x_s, mats["gu"][1].numpy())
    h_q, h_s = O.silu_mul_quant(gu, 1)
    return mm(h_q, mats["dn"][0].numpy(), h_s, mats["dn"][1].numpy()), res


def _close(got, want_bits, tol):
    g = got.float().cpu()
    w = O.from_bits(want_bits, torch.bfloat16).float()
    return (g - w).abs().max().item() / max(w.abs().max().item(), 1e-6) <= tol


@pytest.mark.parametrize("M", [5, 256])
def test_layer_tail_fused_vs_oracle(comm1, M):
    mats, norm_w = _layer(M)
    plan, idx = _plan(mats, norm_w, comm1)
    g = torch.Generator().manual_seed(100 + M)
    attn = torch.randn(M, H, generator=g).to(torch.bfloat16)
    residual = torch.randn(M, H, generator=g).to(torch.bfloat16)
    out, res = torch.ops.vllm_turing.layer_tail(attn.cuda(), residual.cuda(), idx)
    torch.cuda.synchronize()
    comm1.check()
    assert plan.fused, "the stand-in layer should take the fused plan"
    want_out, want_res = _oracle_tail(attn, residual, mats, norm_w, big=M > 32)
    assert np.array_equal(O.to_bits(res.cpu()), want_res), "new residual"
    assert _close(out, want_out, 2e-2), "tail output"


def test_layer_tail_staged_plain_and_chunked(comm1, monkeypatch):
    from vllm_turing_b200 import tailoverlap
    M = 256
    mats, norm_w = _layer(7)
    g = torch.Generator().manual_seed(8)
    attn = torch.randn(M, H, generator=g).to(torch.bfloat16).cuda()
    residual = torch.randn(M, H, generator=g).to(torch.bfloat16).cuda()
    plan, idx = _plan(mats, norm_w, comm1, allow_fused=False)
    out_plain, res_plain = torch.ops.vllm_turing.layer_tail(attn, residual, idx)   # M < MIN_TOKENS: one chunk
    monkeypatch.setattr(tailoverlap, "MIN_TOKENS", 64)
    out_chunk, res_chunk = torch.ops.vllm_turing.layer_tail(attn, residual, idx)   # two row chunks, side stream
    assert tailoverlap.chunk_bounds(M) == [0, 128, 256]
    fplan, fidx = _plan(mats, norm_w, comm1)
    out_fused, res_fused = torch.ops.vllm_turing.layer_tail(attn, residual, fidx)
    torch.cuda.synchronize()
    assert not plan.fused and fplan.fused
    assert torch.equal(out_chunk, out_plain) and torch.equal(res_chunk, res_plain), "chunking changed the result"
    assert torch.equal(res_plain, res_fused), "staged and fused residuals"
    assert _close(out_plain, O.to_bits(out_fused.cpu()), 3e-2), "staged vs fused output"

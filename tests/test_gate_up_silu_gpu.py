"""The fused gate/up GEMM + SiLU * up + per-token int8 quant (csrc/gate_up_silu.cu) against the two-op chain it
replaces -- the tcgen05 decode GEMM with the plain weight (scaled_mm_) then silu_mul_quant: bit-identical, since both
round at the same points (bf16 gate / up, bf16 SiLU, bf16 product, the quantiser of quantfuse.py:18-24) -- and
against the oracle chain (O.scaled_mm then O.silu_mul_quant; int8 within 1 LSB, the host's expf may differ from the
device's by an ulp)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import q_off, rand_int8, rand_scales

pytestmark = pytest.mark.gpu


def _chain(a, w, sa, sw, dtype):
    """scaled_mm_ (plain weight) -> silu_mul_quant, on the GPU"""
    from vllm_turing_b200 import w8a8
    from vllm_turing_b200.tailoverlap import silu_mul_quant
    M = a.shape[0]
    out = torch.empty(M, w.shape[0], dtype=dtype, device="cuda")
    w8a8.mma(out, a, w.t(), sa, sw, None)
    return silu_mul_quant(out)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,I,K", [(5, 17408, 5120), (1, 64, 128), (16, 2176, 5120), (24, 8704, 5120),
                                   (32, 1088, 256), (3, 4352, 5136)])
def test_fused_equals_chain(M, I, K, dtype):
    from vllm_turing_b200 import w8a8
    code = 0 if dtype == torch.float16 else 1
    a, w = rand_int8((M, K), M + I), rand_int8((2 * I, K), I + K)
    sa, sw = rand_scales(M, 3, 2e-2), rand_scales(2 * I, 4, 2e-4)
    ac, wc, sac, swc = a.cuda(), w.cuda(), sa.cuda().view(-1, 1), sw.cuda().view(-1, 1)
    wi, si = w8a8.interleave_gate_up(wc, swc)
    q, s = w8a8.gate_up_silu_quant(ac, wi, sac, si, dtype=dtype)
    q0, s0 = _chain(ac, wc, sac, swc, dtype)
    torch.cuda.synchronize()
    assert torch.equal(q, q0), f"{(q != q0).sum().item()} int8 values differ from the chain"
    assert torch.equal(s.view(-1), s0.view(-1))
    gu = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), None, code)
    qo, so = O.silu_mul_quant(gu, code)
    assert q_off(q.cpu().numpy(), qo) <= 1
    assert np.max(np.abs(s.cpu().numpy().reshape(-1) - so) / np.maximum(so, 1e-12)) < 1e-2
    assert w8a8.lib().vt_status(1) == 0


def test_back_to_back_and_workspace_zero():
    """12 calls with different inputs and no host sync: each call's row maxima are tagged with its own epoch (a stale
    word of an earlier call is never read as this call's), and the split-K slots read zero afterwards."""
    from vllm_turing_b200 import w8a8
    M, I, K = 5, 4352, 5120
    w = rand_int8((2 * I, K), 7)
    sw = rand_scales(2 * I, 8, 2e-4)
    wc, swc = w.cuda(), sw.cuda().view(-1, 1)
    wi, si = w8a8.interleave_gate_up(wc, swc)
    ins, outs = [], []
    for r in range(12):
        a = rand_int8((M, K), 100 + r).cuda()
        sa = rand_scales(M, 200 + r, 2e-2).cuda().view(-1, 1)
        ins.append((a, sa))
        outs.append(w8a8.gate_up_silu_quant(a, wi, sa, si))
    torch.cuda.synchronize()
    for (a, sa), (q, s) in zip(ins, outs):
        q0, s0 = _chain(a, wc, sa, swc, torch.bfloat16)
        assert torch.equal(q, q0) and torch.equal(s.view(-1), s0.view(-1))
    ws = next(iter(w8a8._silu_ws.values()))
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    slot_bytes = sms * ((M + 1) // 2) * 128 * 16   # [status 256][slots]...
    torch.cuda.synchronize()
    assert int(ws[256:256 + slot_bytes].count_nonzero().item()) == 0

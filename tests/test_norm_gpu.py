"""Row-wise epilogue kernels (csrc/norm_quant.cu) against the oracle and the golden vectors of the reference's own
quant_torch: per-token quant bit-exact, residual add bit-exact, normalised rows within 1e-2 relative, int8 within 1 LSB
(the mean-of-squares summation order is the only free rounding point)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bits_equal, q_off

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("code", [1, 0])
@pytest.mark.parametrize("shape", [(1, 64), (5, 5120), (30, 136)])
def test_quant_golden(golden, code, shape):
    from vllm_turing_b200.quantfuse import scaled_int8_quant_cuda
    key = f"quant_{code}_{shape[0]}x{shape[1]}"
    dt = torch.bfloat16 if code else torch.float16
    x = O.from_bits(golden[key + "_x"], dt).cuda()
    q, s = scaled_int8_quant_cuda(x)
    assert np.array_equal(q.cpu().numpy(), golden[key + "_q"])
    assert np.array_equal(s.cpu().numpy().reshape(-1), golden[key + "_s"])


@pytest.mark.parametrize("M,N", [(1, 5120), (7, 4096), (300, 5120), (2048, 5120)])
def test_quant_vs_oracle(M, N):
    from vllm_turing_b200.quantfuse import scaled_int8_quant_cuda
    x = (torch.randn(M, N, generator=torch.Generator().manual_seed(M)) * 3).to(torch.bfloat16)
    x[0, 3] = 0.5 * x[0].float().abs().max()          # exact ties exercise the rounding order
    q, s = scaled_int8_quant_cuda(x.cuda())
    qo, so = O.quant_rows(O.to_bits(x), 1)
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy().reshape(-1), so)


@pytest.mark.parametrize("shape", [(1, 512), (5, 5120), (24, 1024)])
def test_rms_norm_quant_golden(golden, shape):
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant
    key = f"norm_{shape[0]}x{shape[1]}"
    dt = torch.bfloat16
    x = O.from_bits(golden[key + "_x"], dt).cuda()
    r = O.from_bits(golden[key + "_r"], dt).cuda()
    w = O.from_bits(golden[key + "_w"], dt).cuda()
    normed = torch.empty_like(x)
    q, s = rms_norm_dynamic_per_token_quant(x, w, 1e-6, r, normed)
    assert_bits_equal(r, golden[key + "_h"], "residual")
    yf, yr = O.bits_to_float(O.to_bits(normed.cpu()), 1), O.bits_to_float(golden[key + "_y"], 1)
    assert np.max(np.abs(yf - yr) / (np.abs(yr) + 1e-3)) < 1e-2
    assert q_off(q.cpu().numpy(), golden[key + "_q"]) <= 1
    so = s.cpu().numpy().reshape(-1)
    assert np.max(np.abs(so - golden[key + "_s"]) / golden[key + "_s"]) < 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N", [(5, 5120), (300, 5120), (8192, 5120), (64, 4096), (7, 16384), (33, 512),
                                 (40, 1000), (3, 20480)])
def test_rms_norm_quant_vs_oracle(M, N, dtype):
    """the register-resident kernel (N % 8 == 0, N <= 16384) and the shared-memory one (N = 1000, 20480)"""
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant
    code = 0 if dtype == torch.float16 else 1
    g = torch.Generator().manual_seed(N + M)
    x = (torch.randn(M, N, generator=g) * 3).to(dtype)
    r = torch.randn(M, N, generator=g).to(dtype)
    w = (1 + torch.randn(N, generator=g) * 0.1).to(dtype)
    rc = r.cuda()
    q, s = rms_norm_dynamic_per_token_quant(x.cuda(), w.cuda(), 1e-6, rc)
    ro, qo, so, _ = O.add_rms_norm_quant(O.to_bits(x), O.to_bits(r), O.to_bits(w), 1e-6, code)
    assert_bits_equal(rc, ro, "residual")
    assert q_off(q.cpu().numpy(), qo) <= 1
    assert (q.cpu().numpy() != qo).mean() < 1e-2
    assert np.max(np.abs(s.cpu().numpy().reshape(-1) - so) / so) < 1e-2   # one bf16 ulp of the row's absmax


def test_silu_mul_quant_reference_abi():
    """silu_mul_quant with the reference's signature, fp16, incl. an all-zero row (tests/test_silu_quant.py:29-33)."""
    from vllm_turing_b200 import _build
    for M, I in ((1, 8704), (7, 8704), (5, 136)):
        gu = (torch.randn(M, 2 * I, generator=torch.Generator().manual_seed(I + M)) * 3).half()
        gu[0, :I] = 0
        q = torch.empty(M, I, dtype=torch.int8, device="cuda")
        s = torch.empty(M, dtype=torch.float32, device="cuda")
        g = gu.cuda()
        assert _build.load().silu_mul_quant(g.data_ptr(), q.data_ptr(), s.data_ptr(), M, I,
                                            torch.cuda.current_stream().cuda_stream) == 0
        qo, so = O.silu_mul_quant(O.to_bits(gu), 0)
        assert q_off(q.cpu().numpy(), qo) <= 1 and (q.cpu().numpy() != qo).mean() < 1e-3
        assert np.max(np.abs(s.cpu().numpy() - so) / np.maximum(so, 1e-12)) < 1e-3
        assert s[0].item() == 0.0 and not q[0].any().item()


@pytest.mark.parametrize("M,I", [(1, 17408), (5, 17408), (5, 2176), (24, 8704), (64, 136), (100, 4352), (5, 4352),
                                 (3, 4100)])
def test_silu_mul_quant_bf16_row_split(M, I):
    """bf16 SiLU-mul-quant at decode shapes -- rows split over 4..17 CTAs (the row absmax combined through epoch-tagged
    words; 4100 takes the scalar loads, the others the 8-element vectors) or one CTA per row (2176, and 100 rows) --
    ten back-to-back calls with different inputs and no host sync in between: a call never takes an earlier call's
    words for its own."""
    from vllm_turing_b200 import _build
    L = _build.load()
    ins, outs = [], []
    for rep in range(10):
        gu = (torch.randn(M, 2 * I, generator=torch.Generator().manual_seed(31 * rep + M + I)) * 3).to(torch.bfloat16)
        if rep == 3:
            gu[M - 1, :I] = 0   # an all-zero SiLU row: scale 0, q 0
        q = torch.empty(M, I, dtype=torch.int8, device="cuda")
        s = torch.empty(M, dtype=torch.float32, device="cuda")
        g = gu.cuda()
        assert L.vt_silu_mul_quant(g.data_ptr(), q.data_ptr(), s.data_ptr(), M, I, 1,
                                   torch.cuda.current_stream().cuda_stream) == 0
        ins.append((gu, g))
        outs.append((q, s))
    torch.cuda.synchronize()
    for (gu, _), (q, s) in zip(ins, outs):
        qo, so = O.silu_mul_quant(O.to_bits(gu), 1)
        assert q_off(q.cpu().numpy(), qo) <= 1 and (q.cpu().numpy() != qo).mean() < 1e-3
        assert np.max(np.abs(s.cpu().numpy() - so) / np.maximum(so, 1e-12)) < 1e-3
    assert outs[3][1][M - 1].item() == 0.0 and not outs[3][0][M - 1].any().item()
    assert L.vt_status(1) == 0

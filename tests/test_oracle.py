"""The CPU oracle pinned against the golden vectors made by the reference's own code and its tests' formulas
(tests/golden/make_golden.py). CPU only."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden.make_golden import MM_CASES, mm_case_inputs


def sha(x):
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


@pytest.mark.parametrize("code", [1, 0])
@pytest.mark.parametrize("shape", [(1, 64), (5, 5120), (30, 136)])
def test_quant_matches_reference_quant_torch(golden, code, shape):
    key = f"quant_{code}_{shape[0]}x{shape[1]}"
    q, s = O.quant_rows(golden[key + "_x"], code)
    assert np.array_equal(s, golden[key + "_s"])           # vllm_turing/quantfuse.py:18-24, bit-exact
    assert np.array_equal(q, golden[key + "_q"])


@pytest.mark.parametrize("case", MM_CASES)
def test_gemm_and_dequant(golden, case):
    M, N, K = case
    a, w, sa, sw = mm_case_inputs(M, N, K)
    key = f"mm_{M}x{N}x{K}"
    assert str(golden[key + "_in_sha"]) == sha(a.numpy()) + sha(w.numpy()) + sha(sa.numpy()) + sha(sw.numpy())
    acc = O.gemm_s32(a.numpy(), w.numpy())
    assert np.array_equal(acc, golden[key + "_acc"])         # exact int32
    for code in (1, 0):
        out = O.dequant(acc, sa.numpy(), sw.numpy(), None, code)
        assert np.array_equal(out, golden[f"{key}_out{code}"])
        out2 = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), None, code)
        assert np.array_equal(out2, out)


def test_dequant_bias_and_per_tensor_scale():
    """bias and per-tensor scales (tests/test_w8a8_mma.py:63-64) against a float64 restatement."""
    g = torch.Generator().manual_seed(5)
    a = torch.randint(-128, 128, (3, 96), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (40, 96), generator=g, dtype=torch.int8)
    sa = torch.rand(1, generator=g) * 1e-2
    sw = torch.rand(40, generator=g) * 1e-3
    bias = torch.randn(40, generator=g).to(torch.bfloat16)
    out = O.scaled_mm(a.numpy(), w.numpy(), sa.numpy(), sw.numpy(), O.to_bits(bias), 1)
    ref = (a.double() @ w.double().t()) * sa.double() * sw.double().view(1, -1) + bias.double()
    got = O.from_bits(out, torch.bfloat16).double()
    assert ((got - ref).abs() / (ref.abs() + 1e-3)).max().item() < 2e-2     # tests/test_w8a8_mma.py:97-99


@pytest.mark.parametrize("nr", [2, 4, 8])
def test_all_reduce(golden, nr):
    parts = list(golden[f"ar_{nr}_parts"])
    assert np.array_equal(O.all_reduce(parts, 1), golden[f"ar_{nr}_out"])


@pytest.mark.parametrize("shape", [(1, 512), (5, 5120), (24, 1024)])
def test_add_rms_norm_quant(golden, shape):
    key = f"norm_{shape[0]}x{shape[1]}"
    res, q, s, y = O.add_rms_norm_quant(golden[key + "_x"], golden[key + "_r"], golden[key + "_w"], 1e-6, 1,
                                        want_normed=True)
    assert np.array_equal(res, golden[key + "_h"])            # bf16 residual add, exact
    yf = O.bits_to_float(y, 1)
    yr = O.bits_to_float(golden[key + "_y"], 1)
    assert np.max(np.abs(yf - yr) / (np.abs(yr) + 1e-3)) < 1e-2   # mean-of-squares order differs in the last bit
    assert np.max(np.abs(s - golden[key + "_s"]) / golden[key + "_s"]) < 1e-2
    assert np.abs(q.astype(np.int32) - golden[key + "_q"].astype(np.int32)).max() <= 1


def test_config0_chain(golden):
    """BASELINE config 0 (M=16, K_local=8704, N=5120, 2 ranks, seed 0): every exact stage bit-exact, the requantised
    activations within one LSB."""
    from vllm_turing_b200.synthetic import make_layer_inputs
    M, N, K = 16, 5120, 8704
    lis = [make_layer_inputs(M, N, K, seed=0, rank=r) for r in range(2)]
    parts = []
    for r, li in enumerate(lis):
        acc = O.gemm_s32(li.a.numpy(), li.w.numpy())
        assert sha(acc) == str(golden[f"cfg0_r{r}_acc_sha"])
        part = O.dequant(acc, li.sa.numpy(), li.sw.numpy(), None, 1)
        assert sha(part) == str(golden[f"cfg0_r{r}_part_sha"])
        parts.append(part)
    red = O.all_reduce(parts, 1)
    assert sha(red) == str(golden["cfg0_reduced_sha"])
    res, q, s, _ = O.add_rms_norm_quant(red, O.to_bits(lis[0].residual), O.to_bits(lis[0].norm_w), 1e-6, 1)
    assert sha(res) == str(golden["cfg0_residual_sha"])
    assert np.abs(q.astype(np.int32) - golden["cfg0_q"].astype(np.int32)).max() <= 1
    assert np.max(np.abs(s - golden["cfg0_s"]) / golden["cfg0_s"]) < 1e-3
    # the one-call chain gives the same
    res2, q2, s2, red2 = O.row_linear_tp([li.a.numpy() for li in lis], [li.w.numpy() for li in lis],
                                         [li.sa.numpy() for li in lis], [li.sw.numpy() for li in lis],
                                         O.to_bits(lis[0].residual), O.to_bits(lis[0].norm_w), 1e-6, 1)
    assert np.array_equal(red2, red) and np.array_equal(res2, res) and np.array_equal(q2, q)


def test_weight_quant_formula():
    """scripts/w8a8_convert.py:165-166 restated, against the synthetic generator's torch version of it."""
    from vllm_turing_b200.synthetic import quant_per_channel
    w = torch.randn(33, 200, generator=torch.Generator().manual_seed(3)) * 0.02
    w[4] = 0.0
    q, s = O.weight_quant(w.numpy())
    qt, st = quant_per_channel(w)
    assert np.array_equal(q, qt.numpy()) and np.array_equal(s, st.numpy())


def test_silu_mul_quant_zero_row():
    """silu_quant.cu semantics incl. an all-zero activation row (tests/test_silu_quant.py:30)."""
    g = torch.Generator().manual_seed(9)
    M, I = 4, 136
    gu = (torch.randn(M, 2 * I, generator=g) * 3).half()
    gu[0, :I] = 0
    q, s = O.silu_mul_quant(O.to_bits(gu), 0)
    assert s[0] == 0.0 and not q[0].any()
    act = (torch.nn.functional.silu(gu[:, :I].float()).half() * gu[:, I:]).float()
    am = act.abs().amax(-1)
    assert np.allclose(s[1:], (am / 127.0).numpy()[1:], rtol=1e-6)


def test_all_gather():
    ps = [np.full(37, r + 1, np.uint8) for r in range(4)]
    g = O.all_gather(ps)
    assert g.size == 4 * 37 and all((g[r * 37:(r + 1) * 37] == r + 1).all() for r in range(4))


LM_CASES = [(1, 64, 256), (5, 300, 1040), (17, 136, 512)]


@pytest.mark.parametrize("code", [0, 1])
@pytest.mark.parametrize("case", LM_CASES)
def test_lmhead_quant_matches_reference_quantize_rows(golden, code, case):
    """vllm_turing/lmhead.py:52-61 (the reference's own function made the golden q, s), incl. an all-zero row."""
    key = f"lm_{code}_{case[0]}x{case[1]}x{case[2]}"
    w = O.bits_to_float(golden[key + "_w"], code)
    q, s = O.lmhead_quant(w)                      # torch's CPU semantics, which made the golden vectors
    assert np.array_equal(s, golden[key + "_s"])
    assert np.array_equal(q, golden[key + "_q"])
    qc, sc = O.lmhead_quant(w, device="cuda")      # the GPU form: scales within one float32 ulp
    assert np.all(np.abs(sc.view(np.int32) - s.view(np.int32)) <= 1)
    assert np.abs(qc.astype(np.int32) - q.astype(np.int32)).max() <= 1


@pytest.mark.parametrize("code", [0, 1])
@pytest.mark.parametrize("case", LM_CASES)
def test_w8a16_formula(golden, code, case):
    """The W8A16 arithmetic of vllm_turing/csrc/w8a16_gemv.cu:64-106: the exact sum (float64 here and in the golden
    vectors, in different orders) and the one-rounding epilogue fma(acc, s, b)."""
    key = f"lm_{code}_{case[0]}x{case[1]}x{case[2]}"
    out, acc, mag = O.w8a16(golden[key + "_x"], golden[key + "_q"], golden[key + "_s"], golden[key + "_b"], code,
                            want_acc=True)
    np.testing.assert_allclose(acc, golden[key + "_acc"], rtol=1e-12, atol=1e-9)
    assert (mag >= np.abs(acc)).all()
    assert np.array_equal(out, golden[key + "_out"])
    # the tolerance check used by the GPU tests accepts the oracle itself and rejects a planted error
    assert O.w8a16_close(out, golden[key + "_out"], mag, golden[key + "_s"], code) == 0.0
    bad = out.copy()
    bad[0, 0] ^= 0x0100                                        # a wrong exponent bit
    assert O.w8a16_close(bad, golden[key + "_out"], mag, golden[key + "_s"], code) > 1.0


def test_w8a16_matches_reference_large_m_path(golden):
    """Above 256 rows the reference dequantises the head to fp16 and multiplies (lmhead.py:104-110); that differs from
    the kernels' arithmetic only by the fp16 rounding of the dequantised weights."""
    out = O.w8a16(golden["lmbig_x"], golden["lmbig_q"], golden["lmbig_s"], None, 0)
    got = O.bits_to_float(out, 0).astype(np.float64)
    ref = O.bits_to_float(golden["lmbig_out"], 0).astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-3


def _ar8_torch(x):
    """The reference's AR8 quantiser (vllm_turing/csrc/host_ar.cu:138-160) restated with torch CPU ops: an independent
    check of the C oracle."""
    g = x.float().view(-1, 128)
    sh = (g.abs().amax(1) / 127.0).half()
    sc = sh.float()
    inv = torch.where(sc > 0, 1.0 / sc, torch.zeros_like(sc))
    q = torch.round(g * inv[:, None]).clamp(-127, 127).to(torch.int8)
    return q.view(-1), sh


def test_ar8_quant_and_sum():
    g = torch.Generator().manual_seed(8)
    xs = [(torch.randn(2048, generator=g) * 3).half() for _ in range(4)]
    xs[0][:128] = 0                                    # an all-zero group: scale 0, values 0
    xs[1][128:256] *= 1e-4                             # tiny values: a subnormal fp16 scale
    xs[2][256] = 6e4                                   # a near-overflow value
    blocks = []
    for x in xs:
        b = O.ar8_quant(O.to_bits(x))
        q, sh = _ar8_torch(x)
        assert np.array_equal(b[:2048].view(np.int8), q.numpy())
        assert np.array_equal(b[2048:].view(np.uint16), O.to_bits(sh))
        blocks.append(b)
    for w in (1, 2, 4):
        out = O.from_bits(O.ar8_dequant_sum(blocks[:w]), torch.float16).float()
        deq = [torch.from_numpy(b[:2048].view(np.int8).copy()).float().view(-1, 128) *
               O.from_bits(b[2048:].view(np.uint16).copy(), torch.float16).float()[:, None] for b in blocks[:w]]
        acc = deq[0]
        for d in deq[1:]:
            acc = acc + d                              # float32, rank order
        assert torch.equal(out, acc.view(-1).half().float())
        # error bound of the lossy format: half a scale step per rank
        ref = sum(x.float() for x in xs[:w])
        step = sum(O.from_bits(b[2048:].view(np.uint16).copy(), torch.float16).float().repeat_interleave(128)
                   for b in blocks[:w])
        assert ((out - ref).abs() <= step / 2 + ref.abs() * 2e-3 + 1e-6).all()

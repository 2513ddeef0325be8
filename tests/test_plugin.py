"""The plugin boundary on CPU with vLLM importable: register() / install() semantics, the reference's switches, the
dispatch predicates, and the pure host logic (chunk bounds, all-reduce algorithm choice)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _py(code, env=None):
    e = dict(os.environ)
    e.update(env or {})
    e["PYTHONPATH"] = REPO + os.pathsep + e.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=e, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return r.stdout.strip().splitlines()[-1]


def test_disable_switch():
    out = _py("import vllm_turing_b200 as v; v.register(); from vllm import _custom_ops as o; "
              "print(getattr(o.scaled_int8_quant, '_vllm_turing', False))", {"VLLM_TURING_DISABLE": "1"})
    assert out == "False"


def test_register_idempotent_and_capability_gated():
    """On a non-B200 platform (here: no GPU) the GEMM and all-reduce hooks stay off, the capability-independent
    quantfuse and custom-AR hooks go on (the reference gates the same way on cap 75, w8a8.py:132-134)."""
    out = _py("import vllm_turing_b200 as v; v.register(); v.register(); from vllm import _custom_ops as o; "
              "from vllm.distributed.device_communicators.cuda_communicator import CudaCommunicator as C; "
              "from vllm.distributed.device_communicators.custom_all_reduce import CustomAllreduce as A; "
              "print(getattr(o.scaled_int8_quant, '_vllm_turing', False), "
              "getattr(o.cutlass_scaled_mm, '_vllm_turing', False), getattr(C, '_vllm_turing_har', False), "
              "getattr(A, '_vllm_turing_copy', False))")
    assert out == "True False False True"


def test_entry_point_declared():
    txt = open(os.path.join(REPO, "pyproject.toml")).read()
    assert '[project.entry-points."vllm.general_plugins"]' in txt and 'turing = "vllm_turing_b200:register"' in txt


def test_quant_torch_matches_oracle():
    from oracle import oracle as O
    from vllm_turing_b200.quantfuse import quant_torch
    x = (torch.randn(7, 640, generator=torch.Generator().manual_seed(1)) * 3).to(torch.bfloat16)
    q, s = quant_torch(x)
    qo, so = O.quant_rows(O.to_bits(x), 1)
    assert np.array_equal(q.numpy(), qo) and np.array_equal(s.numpy().reshape(-1), so)


def test_scaled_mm_op_registered():
    import vllm_turing_b200.w8a8  # noqa: F401
    assert hasattr(torch.ops.vllm_turing, "scaled_mm_")
    import vllm_turing_b200.tailoverlap  # noqa: F401
    assert hasattr(torch.ops.vllm_turing, "layer_tail")


def test_gemv_ok_predicates():
    """The layout checks of vllm_turing/w8a8.py:38-66 on CPU tensors (no kernel call)."""
    from vllm_turing_b200 import w8a8
    M, N, K = 5, 64, 128
    a = torch.zeros(M, K, dtype=torch.int8)
    w = torch.zeros(N, K, dtype=torch.int8)
    sa, sb = torch.ones(M, 1), torch.ones(N, 1)
    out = torch.empty(M, N, dtype=torch.bfloat16)
    def ok(*t):
        return w8a8.gemv_ok(*t, max_m=8)
    assert ok(out, a, w.t(), sa, sb, None)
    assert not ok(out, a, w, sa, sb, None)                               # not the transposed view
    a9 = torch.zeros(9, K, dtype=torch.int8)
    assert not ok(torch.empty(9, N, dtype=torch.bfloat16), a9, w.t(), torch.ones(9, 1), sb, None)
    assert not ok(out.float(), a, w.t(), sa, sb, None)                   # fp32 output not served
    assert w8a8.gemv_ok(out, a, w.t(), sa, sb, None) == (w8a8.MAX_M >= M)  # the GEMV is off by default


def test_chunk_bounds_match_reference_formula():
    """tailoverlap.py:220-224: bounds at 1/6, 1/2, 5/6 rounded down to 16 for >= 4096 tokens, halves below."""
    from vllm_turing_b200.tailoverlap import chunk_bounds
    for n in (2048, 4095, 4096, 6720, 8192, 32768):
        fr = (0.16667, 0.5, 0.83333) if n >= 4096 else (0.5,)
        ref = [0] + [int(f * n) // 16 * 16 for f in fr] + [n]
        assert chunk_bounds(n) == ref


def test_allreduce_algorithm_choice():
    from vllm_turing_b200 import hostar

    class C:
        ll_bytes = 512 << 10

        def should_use(self, t):
            return t.numel() % 8 == 0

    c = C()
    assert hostar.choose_algo(None, torch.empty(5120, dtype=torch.bfloat16)) == 0
    assert hostar.choose_algo(c, torch.empty(5 * 5120, dtype=torch.bfloat16)) == 1       # 51 KB: one-shot
    assert hostar.choose_algo(c, torch.empty(8192 * 5120, dtype=torch.bfloat16)) == 2    # 84 MB: two-shot
    assert hostar.choose_algo(c, torch.empty(5121, dtype=torch.bfloat16)) == 0           # odd: vLLM's path
    # AR8 (VLLM_TURING_AR8=1): large fp16 messages only, above the one-shot size
    c.ar8_ok = lambda t: t.dtype == torch.float16 and t.numel() % 1024 == 0
    old = hostar.AR8
    try:
        hostar.AR8 = True
        assert hostar.choose_algo(c, torch.empty(8192 * 5120, dtype=torch.float16)) == 3
        assert hostar.choose_algo(c, torch.empty(8192 * 5120, dtype=torch.bfloat16)) == 2
        assert hostar.choose_algo(c, torch.empty(5 * 5120, dtype=torch.float16)) == 1
    finally:
        hostar.AR8 = old


def test_synthetic_inputs_are_deterministic():
    from vllm_turing_b200.synthetic import make_layer_inputs
    a = make_layer_inputs(5, 64, 128, seed=3, rank=1)
    b = make_layer_inputs(5, 64, 128, seed=3, rank=1)
    c = make_layer_inputs(5, 64, 128, seed=3, rank=0)
    assert torch.equal(a.a, b.a) and torch.equal(a.w, b.w) and not torch.equal(a.w, c.w)
    assert torch.equal(a.residual, c.residual) and torch.equal(a.norm_w, c.norm_w)   # shared across ranks


@pytest.mark.parametrize("mod", ["w8a8", "hostar", "quantfuse", "customar", "dmaag", "tailoverlap", "comm", "lmhead",
                                 "convert"])
def test_modules_import_without_gpu(mod):
    __import__(f"vllm_turing_b200.{mod}")


def test_interleave_gate_up_order():
    """tile t of the interleaved weight = gate rows 64t..64t+63, then up rows 64t..64t+63 (CPU, no kernel)"""
    from vllm_turing_b200 import w8a8
    I, K = 192, 32
    w = torch.arange(2 * I, dtype=torch.int32).view(-1, 1).expand(2 * I, K).to(torch.int16)
    s = torch.arange(2 * I, dtype=torch.float32)
    wi, si = w8a8.interleave_gate_up(w, s)
    rows = wi[:, 0].tolist()
    for t in range(I // 64):
        assert rows[128 * t:128 * t + 64] == list(range(64 * t, 64 * t + 64))
        assert rows[128 * t + 64:128 * t + 128] == list(range(I + 64 * t, I + 64 * t + 64))
    assert si.tolist() == [float(r) for r in rows]


def test_w8a16_op_registered_and_quantize_rows_matches_oracle():
    """vllm_turing::w8a16_mm exists (the reference's op name, lmhead.py:80-81) and the package's quantize_rows is the
    oracle's restatement of the reference's formula (bit-exact on CPU)."""
    from oracle import oracle as O
    from vllm_turing_b200 import lmhead
    assert hasattr(torch.ops.vllm_turing, "w8a16_mm")
    w = (torch.randn(40, 96, generator=torch.Generator().manual_seed(4)) * 0.02).half()
    w[2] = 0
    q, s = lmhead.quantize_rows(w)
    qo, so = O.lmhead_quant(w.float().numpy())
    assert np.array_equal(q.numpy(), qo) and np.array_equal(s.numpy(), so)


class _FakeComm:
    """The communicator's all-gather contract on CPU tensors: fills the peers' blocks from the given peers' inputs."""

    def __init__(self, xs, rank, ll=1 << 20):
        self.xs, self.rank, self.world, self.ll_capacity = xs, rank, len(xs), ll
        self.calls = []

    def all_gather_rows(self, out, rows, row_bytes, ld_bytes):
        self.calls.append("rows")
        b = out.view(-1).view(torch.uint8).view(rows, ld_bytes)
        for r, x in enumerate(self.xs):
            if r != self.rank:
                b[:, r * row_bytes:(r + 1) * row_bytes] = x.reshape(rows, -1).view(torch.uint8)
        return out

    def all_gather(self, g, m):
        self.calls.append("slots")
        for r, x in enumerate(self.xs):
            if r != self.rank:
                g[r * m:(r + 1) * m] = x.reshape(-1).view(torch.uint8)
        return g


@pytest.mark.parametrize("shape,dim", [((5, 24), -1), ((2, 3, 8), -1), ((6, 16), 0), ((4, 6, 8), 1), ((3, 5), -1),
                                       ((4, 6), -1)])
@pytest.mark.parametrize("world", [2, 4])
def test_all_gather_dim_layout(shape, dim, world):
    """dmaag.all_gather_dim gives vLLM's all_gather(dim) result (torch.cat of the ranks' tensors along dim) for every
    layout path: row-strided in place (last dim), contiguous slots (dim 0), slots + movedim (other dims, or payloads
    whose row is not a multiple of 8 bytes)."""
    from vllm_turing_b200 import dmaag
    g = torch.Generator().manual_seed(world)
    xs = [torch.randn(*shape, generator=g).to(torch.bfloat16) for _ in range(world)]
    want = torch.cat(xs, dim=dim)
    m = xs[0].numel() * 2
    for rank in range(world):
        fc = _FakeComm(xs, rank)
        got = dmaag.all_gather_dim(fc, xs[rank], dim)
        if m % 8:                                      # no 8-byte words: left to vLLM's all-gather
            assert got is None and fc.calls == []
            continue
        assert got is not None and torch.equal(got, want), (rank, fc.calls)
        last = dim in (-1, len(shape) - 1)
        assert fc.calls == (["rows"] if last and (shape[-1] * 2) % 8 == 0 else ["slots"])


def test_all_gather_dim_large_last_dim_uses_slots():
    from vllm_turing_b200 import dmaag
    xs = [torch.full((3, 64), float(r)).to(torch.bfloat16) for r in range(2)]
    fc = _FakeComm(xs, 1, ll=128)                                     # payload 384 B > the one-shot capacity
    got = dmaag.all_gather_dim(fc, xs[1], -1)
    assert torch.equal(got, torch.cat(xs, -1)) and fc.calls == ["slots"]


@pytest.mark.parametrize("M,ll", [(5, 1 << 20), (5, 256), (70, 1 << 20)])
def test_logits_gathered_paths(monkeypatch, M, ll):
    """lmhead.logits_gathered on CPU with the kernel and the communicator faked: in place + row-strided gather when the
    payload fits the one-shot capacity and M <= 64, else the shard through the op + contiguous slots + transpose;
    both give the ranks' logits concatenated along the vocabulary."""
    from vllm_turing_b200 import lmhead
    world, Vs, K = 3, 40, 32
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    heads = [torch.randn(Vs, K, generator=g) for _ in range(world)]
    logits = [(x.float() @ h.t()).to(torch.bfloat16) for h in heads]
    want = torch.cat(logits, dim=1)
    calls = []

    def fake_mm_into(out, x_, w, s, bias=None, ldo=None):
        calls.append("kernel")
        r = int(w[0, 0].item())
        out[:, :Vs] = logits[r]          # the view starts at this rank's columns; the row stride is out's
        return out

    monkeypatch.setattr(lmhead, "mm_into", fake_mm_into)
    monkeypatch.setattr(lmhead, "kernel_ok", lambda x_, w: True)
    monkeypatch.setattr(lmhead, "shard_logits", lambda x_, w, s, b=None: (calls.append("op"), logits[int(w[0, 0])])[1])
    for rank in range(world):
        fc = _FakeComm([lg for lg in logits], rank, ll=ll)
        w_tag = torch.full((Vs, K), float(rank))   # the fakes read the rank from the weight
        got = lmhead.logits_gathered(x, w_tag, None, comm=fc)
        assert torch.equal(got, want)
        fits = M <= 64 and M * Vs * 2 <= ll
        assert fc.calls == (["rows"] if fits else ["slots"])
    assert set(calls) == ({"kernel"} if M <= 64 and M * Vs * 2 <= ll else {"op"})


def test_logits_gathered_rejects_a_mismatched_out():
    """A caller-supplied out is written through its pointer with row stride world * Vs: a wrong shape, dtype or a
    non-contiguous view is refused instead of being mis-written."""
    from vllm_turing_b200 import lmhead
    M, Vs, K = 4, 40, 32
    x = torch.randn(M, K).to(torch.bfloat16)
    w = torch.zeros(Vs, K, dtype=torch.int8)
    for bad in (torch.empty(M, Vs + 8, dtype=torch.bfloat16), torch.empty(M, Vs, dtype=torch.float16),
                torch.empty(Vs, M, dtype=torch.bfloat16).t()):
        with pytest.raises(ValueError):
            lmhead.logits_gathered(x, w, None, out=bad)

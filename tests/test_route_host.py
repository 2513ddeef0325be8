"""Which path TPComm.row_linear takes, on CPU with the device calls stubbed: decode shapes (M <= 32) always go to the
fused row-linear entry (vt_tp_row_linear); prefill shapes go to the fused prefill tail below
comm.PREFILL_CHAIN_WORLD ranks and to the three-kernel chain (GEMM into the reduced buffer, all-reduce in place,
residual + RMSNorm + quant) from there up, unless `route` forces one; a chain the prefill GEMM cannot take falls back
to the fused entry; an unknown route is an error. No GPU is used."""
import types

import pytest
import torch

from vllm_turing_b200 import comm as C
from vllm_turing_b200 import quantfuse, w8a8


class _Lib:
    def __init__(self, log):
        self.log = log

    def vt_tp_row_linear(self, *args):
        self.log.append("fused")
        return 0


@pytest.fixture
def rig(monkeypatch):
    log = []
    r = types.SimpleNamespace(big_ok=True, log=log)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: types.SimpleNamespace(cuda_stream=0))
    monkeypatch.setattr(w8a8, "big_ok", lambda out, a, b, sa, sb, bias: r.big_ok)
    monkeypatch.setattr(w8a8, "big", lambda out, a, b, sa, sb: log.append(("gemm", out.data_ptr())))
    monkeypatch.setattr(quantfuse, "rms_norm_dynamic_per_token_quant",
                        lambda x, w, eps, res, normed=None, q=None, s=None: log.append(("norm", x.data_ptr())))

    def make(world):
        c = object.__new__(C.TPComm)
        c.L, c.world, c.rank, c.handle = _Lib(log), world, 0, 0xABC
        c.all_reduce = lambda t, out=None, algo=0: log.append(("all_reduce", t.data_ptr(), out.data_ptr()))
        return c

    r.make = make
    return r


def _call(c, M, route="auto", residual=True, N=64, K=32):
    a = torch.zeros(M, K, dtype=torch.int8)
    w = torch.zeros(N, K, dtype=torch.int8)
    sa, sw = torch.ones(M), torch.ones(N)
    red = torch.empty(M, N, dtype=torch.bfloat16)
    kw = dict(residual=torch.zeros(M, N, dtype=torch.bfloat16), norm_w=torch.ones(N, dtype=torch.bfloat16)) \
        if residual else {}
    c.row_linear(a, w, sa, sw, reduced=red, route=route, **kw)
    return red


def _kinds(log):
    return [e if isinstance(e, str) else e[0] for e in log]


@pytest.mark.parametrize("world,M,route,want", [
    (1, 256, "auto", "fused"), (2, 256, "auto", "fused"), (4, 256, "auto", "chain"), (8, 512, "auto", "chain"),
    (4, 5, "auto", "fused"), (8, 32, "chain", "fused"),            # decode shapes: always the fused entry
    (4, 256, "fused", "fused"), (2, 256, "chain", "chain"), (1, 33, "chain", "chain")])
def test_route(rig, world, M, route, want):
    assert C.PREFILL_CHAIN_WORLD == 4
    red = _call(rig.make(world), M, route)
    if want == "fused":
        assert rig.log == ["fused"]
    else:
        p = red.data_ptr()   # the GEMM writes the caller's reduced buffer, reduced in place, then normalised
        assert rig.log == [("gemm", p), ("all_reduce", p, p), ("norm", p)]


def test_chain_without_residual_returns_reduced(rig):
    c = rig.make(4)
    a = torch.zeros(64, 32, dtype=torch.int8)
    out = c.row_linear(a, torch.zeros(16, 32, dtype=torch.int8), torch.ones(64), torch.ones(16))
    assert _kinds(rig.log) == ["gemm", "all_reduce"] and out.shape == (64, 16) and out.dtype == torch.bfloat16


def test_chain_falls_back_when_the_gemm_cannot_take_the_shape(rig):
    rig.big_ok = False
    _call(rig.make(4), 256)
    assert rig.log == ["fused"]


def test_unknown_route_rejected(rig):
    with pytest.raises(ValueError):
        _call(rig.make(2), 256, route="fast")
    assert rig.log == []

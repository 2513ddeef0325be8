"""Seeded synthetic inputs for the row-parallel W8A8 layer (no checkpoint or dataset is available offline).

Shapes and value distributions follow the benchmark configuration of the reference's TP path: activations N(0, 1) in
bf16 quantised per token (symmetric absmax, the formula of vllm_turing/quantfuse.py:18-24), weights N(0, 0.02)
quantised per output channel (scripts/w8a8_convert.py:165-166), residual N(0, 1) bf16, RMSNorm weight 1 + N(0, 0.1).
Generation runs on the CPU with torch.Generator, so every machine with this torch build produces the same bytes.
Per-rank tensors (the activation K-slice and the weight K-slice) use the seed `seed * 1000 + rank`; tensors every rank
holds identically (residual, norm weight) use `seed * 1000 + 999`.
"""
from dataclasses import dataclass

import torch


def quant_per_token(x: torch.Tensor):
    """(int8 like x, float32 [rows]) -- vllm_turing/quantfuse.py:18-24 with the all-zero-row rule of
    vllm_turing/csrc/silu_quant.cu:57 (scale 0, q 0)."""
    xf = x.reshape(-1, x.shape[-1]).float()
    absmax = xf.abs().amax(dim=-1, keepdim=True)
    inv = torch.where(absmax > 0, 127.0 / absmax, torch.zeros_like(absmax))
    q = torch.round(xf * inv).clamp(-128.0, 127.0).to(torch.int8)
    return q.reshape(x.shape), (absmax / 127.0).reshape(-1)


def quant_per_channel(w: torch.Tensor):
    """(int8 [N, K], float32 [N]) -- scripts/w8a8_convert.py:165-166."""
    w = w.float()
    scale = w.abs().amax(dim=1, keepdim=True).clamp(min=1e-12) / 127.0
    q = torch.round(w / scale).clamp(-128, 127).to(torch.int8)
    return q, scale.reshape(-1)


@dataclass
class LayerInputs:
    a: torch.Tensor         # int8 [M, K]   this rank's activation slice, quantised
    sa: torch.Tensor        # float32 [M]
    w: torch.Tensor         # int8 [N, K]   this rank's weight slice (row-major [N, K])
    sw: torch.Tensor        # float32 [N]
    residual: torch.Tensor  # [M, N] dtype, identical on every rank
    norm_w: torch.Tensor    # [N] dtype, identical on every rank
    eps: float = 1e-6


def make_layer_inputs(M: int, N: int, K: int, seed: int = 0, rank: int = 0, dtype=torch.bfloat16,
                      with_norm: bool = True) -> LayerInputs:
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    x = torch.randn(M, K, generator=g).to(dtype)
    a, sa = quant_per_token(x)
    w, sw = quant_per_channel(torch.randn(N, K, generator=g) * 0.02)
    if with_norm:
        gs = torch.Generator().manual_seed(seed * 1000 + 999)
        residual = torch.randn(M, N, generator=gs).to(dtype)
        norm_w = (1.0 + torch.randn(N, generator=gs) * 0.1).to(dtype)
    else:
        residual = torch.empty(0, dtype=dtype)
        norm_w = torch.empty(0, dtype=dtype)
    return LayerInputs(a.contiguous(), sa.contiguous(), w.contiguous(), sw.contiguous(), residual, norm_w)

"""The checkpoint converter (vllm_turing_b200/convert.py) against the reference's own scripts/w8a8_convert.py, whose
outputs on a tiny seeded bf16 checkpoint are the golden vectors (tests/golden/make_golden.py runs it on the CPU):
every stored tensor bit for bit and the quantization_config, for W8A8, --w8a16 64 and --mixed, and with SmoothQuant
folding (--smooth, alpha 0.5 and 0.8) on a checkpoint of an attention layer, a GDN layer and the MTP layer with
seeded calibration maxima. Plus: the W8A8 weights are the oracle's per-channel quantiser
(scripts/w8a8_convert.py:165-166) and feed the W8A8 GEMM's row-major layout unchanged. CPU only."""
import json
import os

import numpy as np
import pytest
import torch

from tests.golden.make_golden import (CKPT_MODES, CKPT_SHARDS, SMOOTH_ALPHAS, SMOOTH_SHARDS, smooth_checkpoint,
                                     tiny_checkpoint)


def _np(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


@pytest.mark.parametrize("mode", list(CKPT_MODES))
def test_convert_matches_reference_script(tmp_path, golden, mode):
    from safetensors import safe_open
    from vllm_turing_b200 import convert
    src, dst = str(tmp_path / "src"), str(tmp_path / mode)
    tiny_checkpoint(src)
    convert.main([src, dst, "cpu", *CKPT_MODES[mode]])
    names = set()
    for shard in CKPT_SHARDS:
        with safe_open(os.path.join(dst, shard), framework="pt") as f:
            for name in f.keys():
                names.add(name)
                want = golden[f"cv_{mode}_{name}"]
                got = _np(f.get_tensor(name))
                assert got.dtype == want.dtype and np.array_equal(got, want), name
    assert names == {k[len(f"cv_{mode}_"):] for k in golden.files if k.startswith(f"cv_{mode}_")} - \
        {"quantization_config"}
    cfg = json.load(open(os.path.join(dst, "config.json")))
    assert json.dumps(cfg["quantization_config"], sort_keys=True) == str(golden[f"cv_{mode}_quantization_config"])
    assert os.path.exists(os.path.join(dst, "tokenizer_config.json"))
    idx = json.load(open(os.path.join(dst, "model.safetensors.index.json")))
    assert set(idx["weight_map"]) == names


def test_w8a8_weights_are_the_oracle_quantiser_in_gemm_layout(tmp_path):
    """The converted [N, K] int8 weight and [N, 1] scales are orc_weight_quant's, and they are exactly what
    scaled_mm_ takes (b = weight.t(), b_scales = scale) -- the oracle's GEMM on them equals the float64 reference."""
    from safetensors import safe_open
    from oracle import oracle as O
    from vllm_turing_b200 import convert
    src, dst = str(tmp_path / "src"), str(tmp_path / "dst")
    tiny_checkpoint(src)
    convert.convert(src, dst, "cpu", log=lambda *a: None)
    name = "model.language_model.layers.0.mlp.gate_proj.weight"
    with safe_open(os.path.join(src, "model-00001-of-00002.safetensors"), framework="pt") as f:
        w = f.get_tensor(name).float()
    with safe_open(os.path.join(dst, "model-00001-of-00002.safetensors"), framework="pt") as f:
        q, s = f.get_tensor(name), f.get_tensor(name + "_scale")
    qo, so = O.weight_quant(w.numpy())
    assert q.dtype == torch.int8 and q.shape == w.shape and s.shape == (w.shape[0], 1)
    assert np.array_equal(q.numpy(), qo) and np.array_equal(s.view(-1).numpy(), so)
    a = torch.randint(-128, 128, (3, w.shape[1]), generator=torch.Generator().manual_seed(1), dtype=torch.int8)
    assert np.array_equal(O.gemm_s32(a.numpy(), q.numpy()), (a.double() @ q.double().t()).to(torch.int32).numpy())


@pytest.mark.parametrize("alpha", SMOOTH_ALPHAS)
def test_smoothquant_matches_reference_script(tmp_path, alpha):
    """Every tensor of the --smooth conversion equals the reference script's: the smoothed, quantised linears and
    their scales, the folded norms and producer rows (float32), in_proj_a / b (smoothed, kept unquantised), and the
    untouched tensors (lm_head) as stored."""
    from safetensors import safe_open
    from vllm_turing_b200 import convert
    golden = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_smooth.npz"))
    src, calib, dst = str(tmp_path / "src"), str(tmp_path / "calib"), str(tmp_path / "dst")
    smooth_checkpoint(src, calib)
    convert.main([src, dst, "cpu", "--smooth", calib, "--alpha", str(alpha)])
    names = set()
    for shard in SMOOTH_SHARDS:
        with safe_open(os.path.join(dst, shard), framework="pt") as f:
            for name in f.keys():
                names.add(name)
                want = golden[f"sm{alpha}_{name}"]
                got = _np(f.get_tensor(name))
                assert got.dtype == want.dtype and np.array_equal(got, want), name
    assert names == {k[len(f"sm{alpha}_"):] for k in golden.files if k.startswith(f"sm{alpha}_")}
    # the folding moved scale between producers and consumers: some norm became float32, a v_proj row changed
    assert golden[f"sm{alpha}_model.language_model.layers.0.input_layernorm.weight"].dtype == np.float32


def test_smoothquant_preserves_the_layer_function(tmp_path):
    """Folding is exact in real arithmetic: the smoothed norm and consumer give the same pre-quantisation product as
    the originals for any activation (float64 check on the attention layer's q_proj and its input norm)."""
    from safetensors import safe_open
    from vllm_turing_b200 import convert
    src, calib = str(tmp_path / "src"), str(tmp_path / "calib")
    smooth_checkpoint(src, calib)
    sm = convert.Smoothing(src, calib, 0.5, "cpu", list(SMOOTH_SHARDS), log=lambda *a: None)
    get = {}
    for shard in SMOOTH_SHARDS:
        with safe_open(os.path.join(src, shard), framework="pt") as f:
            for name in f.keys():
                get[name] = f.get_tensor(name)
    pre = "model.language_model.layers.0."
    nw, wq = get[pre + "input_layernorm.weight"].double(), get[pre + "self_attn.q_proj.weight"].double()
    nw2 = sm.apply(pre + "input_layernorm.weight", get[pre + "input_layernorm.weight"]).double()
    wq2 = sm.apply(pre + "self_attn.q_proj.weight", get[pre + "self_attn.q_proj.weight"]).double()
    x = torch.randn(3, nw.numel(), generator=torch.Generator().manual_seed(4), dtype=torch.float64)
    ref = (x * (1 + nw)) @ wq.t()
    got = (x * (1 + nw2)) @ wq2.t()
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_convert_smooth_needs_a_directory():
    from vllm_turing_b200 import convert
    with pytest.raises(SystemExit):
        convert.main(["a", "b", "--smooth"])

#!/usr/bin/env python3
"""Generate the committed golden vectors that pin the CPU oracle to the reference.

Run in a container where the reference tree is present (it is NOT needed at test time):
    python tests/golden/make_golden.py [--ref <reference tree>]
(default: VLLM_TURING_REFERENCE, else the directory `reference` beside this repository)
Writes tests/golden/golden.npz. Every output is produced by the reference's own code where it is Python, and by the
exact formulas the reference's tests compute where the reference is CUDA:

  quant      vllm_turing.quantfuse.quant_torch, imported from the reference tree (quantfuse.py:18-24)
  gemm       float64 matmul of the int8 operands, "exact for int8 sums" (tests/test_w8a8_mma.py:42-45)
  dequant    (float)acc * sa * sw rounded to the 16-bit type, in the order of vllm_turing/csrc/w8a8_gemv.cu:91
  allreduce  (x0.float() + x1.float()).half() (tests/bench_devll.py:28-36), rank order for more ranks
  norm+quant h = x + r; h.float() * rsqrt(mean(h^2) + eps) * w; quant_torch  (tests/test_quantfuse.py:45-48)
  lm head    vllm_turing.lmhead.quantize_rows, imported from the reference tree (lmhead.py:52-61), on fp16 / bf16
             heads; the W8A16 GEMM as the reference's kernel computes it (vllm_turing/csrc/w8a16_gemv.cu:64-106:
             products exact in fp32, the sum, then acc * s + b in one fp32 rounding), with the sum in float64; and
             the reference's large-M path (lmhead.py:104-110: dequantise to the activation dtype, matmul), run on CPU
  convert    the reference's scripts/w8a8_convert.py itself (run on the CPU) on a tiny seeded bf16 checkpoint, W8A8,
             --w8a16 64 and --mixed: every stored tensor and the quantization_config
  smooth     the same script with --smooth (SmoothQuant folding) on a tiny seeded checkpoint of one attention layer,
             one GDN layer and the MTP layer, with seeded calibration maxima in the two-rank files its calibration run
             writes, at alpha 0.5 and 0.8 (tests/golden/golden_smooth.npz; --smooth-only writes just that file)
  config 0   the whole chain at BASELINE config 0 (M=16, K_local=8704, N=5120, 2 ranks, seed 0): digests of the
             exact parts plus the int8 / scales arrays
Inputs come from seeded torch CPU generators (vllm_turing_b200.synthetic for config 0) and are stored (small cases)
or regenerated from the seed (config 0).
"""
import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sha(x):
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


# int8 GEMM cases: the operands are regenerated from a per-case seed (tests/test_oracle.py uses the same function and
# checks the input digests first), as in tests/test_w8a8_mma.py:84-88 (randint int8, rand * 1e-2 / 1e-3 scales)
MM_CASES = ((1, 64, 64), (5, 136, 5136), (16, 256, 1024), (24, 40, 256), (32, 300, 5168))


def mm_case_inputs(M, N, K):
    g = torch.Generator().manual_seed(M * 1000003 + N * 1009 + K)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    sa = torch.rand(M, generator=g) * 1e-2
    sw = torch.rand(N, generator=g) * 1e-3
    return a, w, sa, sw


# a tiny synthetic checkpoint for the converter (scripts/w8a8_convert.py): names from its quantised and kept sets
CKPT_SHARDS = {
    "model-00001-of-00002.safetensors": {
        "model.language_model.layers.0.mlp.gate_proj.weight": (48, 256),
        "model.language_model.layers.0.mlp.down_proj.weight": (64, 128),
        "model.language_model.layers.0.self_attn.o_proj.weight": (32, 128),
        "model.language_model.layers.0.linear_attn.in_proj_a.weight": (16, 64),   # kept (ignore list)
        "model.language_model.norm.weight": (64,),
    },
    "model-00002-of-00002.safetensors": {
        "mtp.layers.0.mlp.up_proj.weight": (32, 128),
        "lm_head.weight": (100, 64),                                              # kept (ignore list)
    },
}
CKPT_MODES = {"w8a8": [], "w8a16": ["--w8a16", "64"], "mixed": ["--mixed"]}

# a tiny checkpoint for SmoothQuant folding: an attention layer (q with its gate, GQA), a GDN layer and the MTP layer,
# with the norms and producers the folding touches; dims of the config's text_config
SMOOTH_CFG = {"hidden_size": 64, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16,
              "linear_num_value_heads": 4, "linear_value_head_dim": 16}


def _smooth_tensors():
    H, I = 64, 96
    t = {}
    for pre in ("model.language_model.layers.0.", "mtp.layers.0."):
        t.update({pre + "input_layernorm.weight": (H,), pre + "post_attention_layernorm.weight": (H,),
                  pre + "self_attn.q_proj.weight": (128, H), pre + "self_attn.k_proj.weight": (32, H),
                  pre + "self_attn.v_proj.weight": (32, H), pre + "self_attn.o_proj.weight": (H, 64),
                  pre + "mlp.gate_proj.weight": (I, H), pre + "mlp.up_proj.weight": (I, H),
                  pre + "mlp.down_proj.weight": (H, I)})
    pre = "model.language_model.layers.1."
    t.update({pre + "input_layernorm.weight": (H,), pre + "post_attention_layernorm.weight": (H,),
              pre + "linear_attn.in_proj_qkv.weight": (160, H), pre + "linear_attn.in_proj_z.weight": (64, H),
              pre + "linear_attn.in_proj_a.weight": (4, H), pre + "linear_attn.in_proj_b.weight": (4, H),
              pre + "linear_attn.out_proj.weight": (H, 64), pre + "linear_attn.norm.weight": (16,),
              pre + "mlp.gate_proj.weight": (I, H), pre + "mlp.up_proj.weight": (I, H),
              pre + "mlp.down_proj.weight": (H, I), "lm_head.weight": (50, H)})
    names = sorted(t)
    half = len(names) // 2
    return {"model-00001-of-00002.safetensors": {n: t[n] for n in names[:half]},
            "model-00002-of-00002.safetensors": {n: t[n] for n in names[half:]}}


SMOOTH_SHARDS = _smooth_tensors()
SMOOTH_ALPHAS = (0.5, 0.8)


def smooth_checkpoint(path, calib):
    """Writes the seeded bf16 checkpoint for the SmoothQuant case into `path` and the calibration maxima into `calib`
    (rank{0,1}.pt for the text layers, rank{0,1}_m1.pt for the MTP layer, keyed by vLLM's fused module names;
    row-parallel inputs as each rank's K-shard)."""
    import json as _json
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    os.makedirs(calib, exist_ok=True)
    g = torch.Generator().manual_seed(78)
    wmap = {}
    for shard, tensors in SMOOTH_SHARDS.items():
        out = {}
        for name, shape in tensors.items():
            if len(shape) == 1:   # norm weights: zero-centred (Qwen's 1 + w) or plain
                t = (torch.randn(*shape, generator=g) * 0.1).to(torch.bfloat16)
            else:
                t = (torch.randn(*shape, generator=g) * 0.05).to(torch.bfloat16)
                t[:, 3] *= 8                     # an input channel with large weights
            out[name] = t
            wmap[name] = shard
        save_file(out, os.path.join(path, shard), metadata={"format": "pt"})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        _json.dump({"metadata": {"total_size": 0}, "weight_map": wmap}, f)
    with open(os.path.join(path, "config.json"), "w") as f:
        _json.dump({"architectures": ["Qwen3_5ForConditionalGeneration"], "text_config": dict(SMOOTH_CFG)}, f)
    keys = {"language_model.model.layers.0.self_attn.qkv_proj": 64, "language_model.model.layers.0.self_attn.o_proj": 32,
            "language_model.model.layers.0.mlp.gate_up_proj": 64, "language_model.model.layers.0.mlp.down_proj": 48,
            "language_model.model.layers.1.linear_attn.in_proj_qkvz": 64,
            "language_model.model.layers.1.linear_attn.out_proj": 32,
            "language_model.model.layers.1.mlp.gate_up_proj": 64, "language_model.model.layers.1.mlp.down_proj": 48}
    keys_m1 = {"model.layers.0.self_attn.qkv_proj": 64, "model.layers.0.self_attn.o_proj": 32,
               "model.layers.0.mlp.gate_up_proj": 64, "model.layers.0.mlp.down_proj": 48}
    for tag, ks in (("", keys), ("_m1", keys_m1)):
        for r in (0, 1):
            d = {}
            for k, n in ks.items():
                x = torch.randn(n, generator=g).abs() * 2 + 1e-6
                x[min(7, n - 1)] *= 40            # an activation outlier channel
                d[k] = x
            torch.save(d, os.path.join(calib, f"rank{r}{tag}.pt"))


def tiny_checkpoint(path):
    """Writes the synthetic bf16 checkpoint (seeded) into `path`."""
    import json as _json
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    g = torch.Generator().manual_seed(77)
    wmap = {}
    for shard, tensors in CKPT_SHARDS.items():
        out = {}
        for name, shape in tensors.items():
            t = (torch.randn(*shape, generator=g) * 0.05).to(torch.bfloat16)
            if len(shape) == 2 and shape[0] > 5:
                t[5] = 0                       # an all-zero output channel: scale clamps at 1e-12 / 127
            out[name] = t
            wmap[name] = shard
        save_file(out, os.path.join(path, shard), metadata={"format": "pt"})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        _json.dump({"metadata": {"total_size": 0}, "weight_map": wmap}, f)
    with open(os.path.join(path, "config.json"), "w") as f:
        _json.dump({"architectures": ["Qwen3_5ForConditionalGeneration"], "text_config": {"hidden_size": 64}}, f)
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        f.write("{}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("VLLM_TURING_REFERENCE")
                    or os.path.join(os.path.dirname(REPO), "reference"))
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    ap.add_argument("--smooth-only", action="store_true", help="write only golden_smooth.npz")
    args = ap.parse_args()
    if args.smooth_only:
        return smooth_golden(args.ref, os.path.join(HERE, "golden_smooth.npz"))
    sys.path.insert(0, args.ref)
    from vllm_turing.quantfuse import quant_torch  # the reference's own quantiser
    sys.path.insert(0, REPO)
    from vllm_turing_b200.synthetic import make_layer_inputs

    g = torch.Generator().manual_seed(20240601)
    out = {}

    # ---- quant: the reference's quant_torch on bf16 and fp16 rows ------------------------------------------------
    for dt, code in ((torch.bfloat16, 1), (torch.float16, 0)):
        for M, N in ((1, 64), (5, 5120), (30, 136)):
            x = (torch.randn(M, N, generator=g) * 3).to(dt)
            if M > 1:
                x[1, 7] = 200.0                      # an outlier channel
            if M == 30:
                x[0] = 0.0                           # an all-zero row (tests/test_silu_quant.py:30 covers the same)
            q, s = quant_torch(x)
            key = f"quant_{code}_{M}x{N}"
            out[key + "_x"] = bits(x)
            out[key + "_q"] = q.numpy()
            out[key + "_s"] = s.reshape(-1).numpy()

    # ---- gemm + dequant -------------------------------------------------------------------------------------------
    for M, N, K in MM_CASES:
        a, w, sa, sw = mm_case_inputs(M, N, K)
        acc = (a.double() @ w.double().t())                 # exact (tests/test_w8a8_mma.py:42-43)
        acc32 = acc.to(torch.int32)
        for dt, code in ((torch.bfloat16, 1), (torch.float16, 0)):
            deq = ((acc32.float() * sa.view(-1, 1)) * sw.view(1, -1)).to(dt)   # w8a8_gemv.cu:91 order
            out[f"mm_{M}x{N}x{K}_out{code}"] = bits(deq)
        key = f"mm_{M}x{N}x{K}"
        out[key + "_acc"] = acc32.numpy()
        out[key + "_in_sha"] = np.array(sha(a.numpy()) + sha(w.numpy()) + sha(sa.numpy()) + sha(sw.numpy()))

    # ---- all-reduce -------------------------------------------------------------------------------------------------
    for nr in (2, 4, 8):
        parts = [(torch.randn(5 * 64, generator=g) * 4).to(torch.bfloat16) for _ in range(nr)]
        s = parts[0].float()
        for p in parts[1:]:
            s = s + p.float()
        out[f"ar_{nr}_parts"] = np.stack([bits(p) for p in parts])
        out[f"ar_{nr}_out"] = bits(s.to(torch.bfloat16))

    # ---- residual add + RMSNorm + quant -----------------------------------------------------------------------------
    for M, N in ((1, 512), (5, 5120), (24, 1024)):
        x = (torch.randn(M, N, generator=g) * 3).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g).to(torch.bfloat16)
        w = (1.0 + torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
        h = x + r                                             # in bf16, as tests/test_quantfuse.py:46
        v = h.float().pow(2).mean(-1, keepdim=True)
        y = (h.float() * torch.rsqrt(v + 1e-6) * w.float()).to(torch.bfloat16)
        q, s = quant_torch(y)
        key = f"norm_{M}x{N}"
        out[key + "_x"], out[key + "_r"], out[key + "_w"] = bits(x), bits(r), bits(w)
        out[key + "_h"], out[key + "_y"] = bits(h), bits(y)
        out[key + "_q"], out[key + "_s"] = q.numpy(), s.reshape(-1).numpy()

    # ---- LM head: the reference's row quantiser and the W8A16 arithmetic -----------------------------------------
    from vllm_turing import lmhead   # the reference's module (its CUDA libraries are loaded lazily, not here)
    for dt, code in ((torch.float16, 0), (torch.bfloat16, 1)):
        for M, N, K in ((1, 64, 256), (5, 300, 1040), (17, 136, 512)):
            w = (torch.randn(N, K, generator=g) * 0.02).to(dt)
            w[3, 11] = 0.5                           # an outlier weight: its row's scale follows it
            w[7] = 0.0                               # an all-zero row: scale clamps at 1e-12 / 127
            q, sc = lmhead.quantize_rows(w)
            x = torch.randn(M, K, generator=g).to(dt)
            b = (torch.randn(N, generator=g) * 0.1).to(dt)
            acc = x.double() @ q.double().t()
            o = ((acc.float().double() * sc.double().view(1, -1) + b.double().view(1, -1)).float()).to(dt)
            key = f"lm_{code}_{M}x{N}x{K}"
            out[key + "_w"], out[key + "_q"], out[key + "_s"] = bits(w), q.numpy(), sc.numpy()
            out[key + "_x"], out[key + "_b"] = bits(x), bits(b)
            out[key + "_acc"], out[key + "_out"] = acc.numpy(), bits(o)
    # the reference's own op above GEMV_MAX_M rows (dequantise, matmul), fp16, on CPU
    Mb, Nb, Kb = 300, 40, 256
    wb16 = (torch.randn(Nb, Kb, generator=g) * 0.02).half()
    qb, sb = lmhead.quantize_rows(wb16)
    xb = torch.randn(Mb, Kb, generator=g).half()
    ob = lmhead._w8a16_mm(xb, qb, sb, None)
    out["lmbig_x"], out["lmbig_q"], out["lmbig_s"], out["lmbig_out"] = bits(xb), qb.numpy(), sb.numpy(), bits(ob)

    # ---- M=16, K_local=8704, N=5120, 2 ranks, seed 0 ---------------------------------------------
    M, N, K = 16, 5120, 8704
    parts = []
    for rank in range(2):
        li = make_layer_inputs(M, N, K, seed=0, rank=rank)
        # the activation quantiser must agree with the reference's own quant_torch on these inputs
        gx = torch.Generator().manual_seed(0 * 1000 + rank)
        x = torch.randn(M, K, generator=gx).to(torch.bfloat16)
        qr, sr = quant_torch(x)
        assert torch.equal(qr, li.a) and torch.equal(sr.reshape(-1), li.sa), "synthetic quantiser != quant_torch"
        acc = (li.a.double() @ li.w.double().t()).to(torch.int32)
        part = ((acc.float() * li.sa.view(-1, 1)) * li.sw.view(1, -1)).to(torch.bfloat16)
        out[f"cfg0_r{rank}_acc_sha"] = np.array(sha(acc.numpy()))
        out[f"cfg0_r{rank}_part_sha"] = np.array(sha(bits(part)))
        out[f"cfg0_r{rank}_acc_head"] = acc[:2, :16].numpy()
        parts.append(part)
        res0, nw = li.residual, li.norm_w
    red = (parts[0].float() + parts[1].float()).to(torch.bfloat16)
    h = red + res0
    v = h.float().pow(2).mean(-1, keepdim=True)
    y = (h.float() * torch.rsqrt(v + 1e-6) * nw.float()).to(torch.bfloat16)
    q, s = quant_torch(y)
    out["cfg0_reduced_sha"] = np.array(sha(bits(red)))
    out["cfg0_residual_sha"] = np.array(sha(bits(h)))
    out["cfg0_q"] = q.numpy()
    out["cfg0_s"] = s.reshape(-1).numpy()

    # ---- checkpoint conversion: the reference's own script on the tiny checkpoint, on the CPU -----------------------
    import json as _json
    import subprocess
    import tempfile
    from safetensors import safe_open
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "src")
        tiny_checkpoint(src)
        for mode, flags in CKPT_MODES.items():
            dst = os.path.join(tmp, mode)
            subprocess.run([sys.executable, os.path.join(args.ref, "scripts", "w8a8_convert.py"), src, dst, "cpu",
                            *flags], check=True, capture_output=True)
            for shard in CKPT_SHARDS:
                with safe_open(os.path.join(dst, shard), framework="pt") as f:
                    for name in f.keys():
                        t = f.get_tensor(name)
                        out[f"cv_{mode}_{name}"] = bits(t) if t.dtype == torch.bfloat16 else t.numpy()
            cfg = _json.load(open(os.path.join(dst, "config.json")))
            out[f"cv_{mode}_quantization_config"] = np.array(_json.dumps(cfg["quantization_config"], sort_keys=True))

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out) / 1024:.0f} KiB")
    smooth_golden(args.ref, os.path.join(HERE, "golden_smooth.npz"))


def smooth_golden(ref, path):
    """The reference's scripts/w8a8_convert.py --smooth on the SmoothQuant checkpoint (CPU): every stored tensor."""
    import subprocess
    import tempfile
    from safetensors import safe_open
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        src, calib = os.path.join(tmp, "src"), os.path.join(tmp, "calib")
        smooth_checkpoint(src, calib)
        for alpha in SMOOTH_ALPHAS:
            dst = os.path.join(tmp, f"a{alpha}")
            subprocess.run([sys.executable, os.path.join(ref, "scripts", "w8a8_convert.py"), src, dst, "cpu",
                            "--smooth", calib, "--alpha", str(alpha)], check=True, capture_output=True)
            for shard in SMOOTH_SHARDS:
                with safe_open(os.path.join(dst, shard), framework="pt") as f:
                    for name in f.keys():
                        t = f.get_tensor(name)
                        out[f"sm{alpha}_{name}"] = bits(t) if t.dtype == torch.bfloat16 else t.numpy()
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()

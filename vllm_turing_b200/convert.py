"""Data-free checkpoint conversion into the format this package's GEMMs load: a 16-bit HF safetensors checkpoint ->
an INT8 W8A8 compressed-tensors checkpoint for vLLM (the reference's scripts/w8a8_convert.py:1-243, same on-disk
format, same quantised tensors, same quantization_config), or weight-only INT8 (W8A16, pack-quantized) with --w8a16.

W8A8 (default): the Linear weights of the text layers and the MTP layer become int8 with one float32 scale per output
channel, scale = max(amax(|w|), 1e-12) / 127, q = round(w / scale) clamped to [-128, 127] (w8a8_convert.py:165-166);
activations are quantised per token at run time (config only). The weight is stored row-major [N, K], which is the
layout the tcgen05 decode kernels stream (one TMA box = 128 rows x 128 bytes): vLLM hands it to cutlass_scaled_mm
as the [K, N] view the plugin expects, so no re-layout happens at load time.
W8A16 (--w8a16 [group], default 128; 0 = per channel): int8 per group of K, stored as vLLM's pack-quantized format
(q + 128 as unsigned bytes, four per int32 along K, fp16 scales [N, K / group], weight_shape) (w8a8_convert.py:155-174).
--mixed: W8A16 for down_proj / o_proj / out_proj, W8A8 for the rest (w8a8_convert.py:19-22, 220-227).
Kept as stored: embeddings, lm_head, norms, the vision tower, conv1d, mtp.fc, in_proj_a / in_proj_b (the reference's
ignore list).
--smooth <calibration dir> [--alpha a] (default 0.5): SmoothQuant folding before quantisation (w8a8_convert.py:60-143),
from the per-input-channel activation maxima a calibration run wrote (rank{0,1}.pt, rank{0,1}_m1.pt for the MTP
layer, keyed by vLLM's fused module names). For every group of linears reading one input X (q/k/v, in_proj_qkv/z/a/b,
gate/up, down, o, out), per input channel j: s_j = clamp(max|X_j|^a / max|W_j|^(1 - a), 0.01, 100) with both maxima
clamped at 1e-5, W[:, j] *= s_j in every consumer, and the producer of X absorbs 1 / s_j -- a zero-centred RMSNorm
(Qwen's 1 + w) becomes (1 + w) / s - 1, the GDN output norm w / s (s shared over the value heads), up_proj's rows / s
for down_proj, v_proj's rows / s for o_proj (s shared over the query heads of a key-value head). Changed tensors that
stay unquantised are stored as float32.

Streams one input shard at a time; quantises on `device` (a GPU when given, else the CPU).

usage: python -m vllm_turing_b200.convert <src dir> <dst dir> [device] [--w8a16 [group] | --mixed]
       [--smooth <calibration dir> [--alpha a]]
"""
import json
import os
import re
import shutil
import sys

import torch

# the Linears that are quantised (w8a8_convert.py:55-57): Qwen3.x text layers (GDN, attention, MLP) and the MTP layer
QUANT = re.compile(r"^(model\.language_model\.layers\.\d+\.(linear_attn\.(in_proj_qkv|in_proj_z|out_proj)"
                   r"|self_attn\.(q_proj|k_proj|v_proj|o_proj)|mlp\.(gate_proj|up_proj|down_proj))"
                   r"|mtp\.layers\.\d+\.(self_attn\.(q_proj|k_proj|v_proj|o_proj)|mlp\.(gate_proj|up_proj|down_proj)))"
                   r"\.weight$")
MIXED_W16 = re.compile(r"\.(down_proj|o_proj|out_proj)\.weight$")
IGNORE = ["lm_head", "re:.*visual.*", "re:.*conv1d.*", "re:.*mtp\\.fc.*", "re:.*linear_attn\\.in_proj_(a|b)$"]


def quant_channel(w):
    """float32 [N, K] -> (int8-valued float [N, K], float32 scale [N, 1])."""
    scale = w.abs().amax(dim=1, keepdim=True).clamp(min=1e-12) / 127.0
    return torch.round(w / scale).clamp(-128, 127), scale


def quant_group(w, group):
    """float32 [N, K] -> (int8-valued float [N, K], float32 scale [N, K / group])."""
    N, K = w.shape
    wg = w.view(N, K // group, group)
    scale = wg.abs().amax(dim=2, keepdim=True).clamp(min=1e-12) / 127.0
    q = torch.round(wg / scale).clamp(-128, 127).view(N, K)
    return q, scale.view(N, K // group)


def pack_w16(q, scale, N, K):
    """vLLM's pack-quantized int8 tensors: q + 128 as bytes, four per int32 along K (little-endian)."""
    return {"weight_packed": (q + 128).to(torch.uint8).contiguous().view(torch.int32).cpu(),
            "weight_scale": scale.to(torch.float16).contiguous().cpu(),
            "weight_shape": torch.tensor([N, K], dtype=torch.int64)}


def quantization_config(w8a16=False, group=128, mixed=False):
    """The config.json quantization_config of the converted checkpoint (w8a8_convert.py:194-228)."""
    w16_group = {
        "targets": ["Linear"],
        "weights": {"num_bits": 8, "type": "int", "symmetric": True, "strategy": "group" if group else "channel",
                    "dynamic": False, "group_size": group if group else None, "observer": "minmax"},
        "input_activations": None,
        "output_activations": None,
        "format": "pack-quantized",
    }
    w8a8_group = {
        "targets": ["Linear"],
        "weights": {"num_bits": 8, "type": "int", "symmetric": True, "strategy": "channel", "dynamic": False,
                    "group_size": None, "observer": "minmax"},
        "input_activations": {"num_bits": 8, "type": "int", "symmetric": True, "strategy": "token",
                              "dynamic": True, "observer": None},
        "output_activations": None,
        "format": "int-quantized",
    }
    qc = {
        "quant_method": "compressed-tensors",
        "format": "int-quantized",
        "quantization_status": "compressed",
        "config_groups": {"group_0": w8a8_group},
        "ignore": list(IGNORE),
        "kv_cache_scheme": None,
        "sparsity_config": {},
        "global_compression_ratio": None,
    }
    if w8a16:
        qc["format"] = "pack-quantized"
        qc["config_groups"] = {"group_0": w16_group}
    elif mixed:
        qc["format"] = "mixed-precision"
        qc["config_groups"] = {
            "group_0": dict(w16_group, targets=["re:.*down_proj$", "re:.*o_proj$", "re:.*out_proj$"]),
            "group_1": w8a8_group,
        }
    return qc


class Smoothing:
    """SmoothQuant scales of one checkpoint (see the module docstring): per tensor name, the column scales of a
    consumer, the row scales of a producing linear, or the fold of a producing norm."""

    def __init__(self, src, calib, alpha, device, shards, log=print):
        cfg = json.load(open(os.path.join(src, "config.json")))
        tc = cfg.get("text_config", cfg)
        n_q, n_kv, hd = tc["num_attention_heads"], tc["num_key_value_heads"], tc["head_dim"]
        n_vh, vhd = tc["linear_num_value_heads"], tc["linear_value_head_dim"]
        self.device = device
        stats = {}
        # the calibration files: text layers (vLLM's "language_model.model.layers.*") and the MTP layer ("model.*")
        for tag, prefix in (("", ("language_model.model.layers.", "model.language_model.layers.")),
                            ("_m1", ("model.layers.", "mtp.layers."))):
            ranks = [torch.load(os.path.join(calib, f"rank{r}{tag}.pt")) for r in (0, 1)]
            for key in ranks[0]:
                name = key.replace(prefix[0], prefix[1], 1)
                if key.rsplit(".", 1)[1] in ("o_proj", "down_proj", "out_proj"):
                    stats[name] = torch.cat([ranks[0][key], ranks[1][key]]).float()   # row-parallel: K shards
                else:
                    stats[name] = torch.maximum(ranks[0][key], ranks[1][key]).float()
        groups = []   # (input, consumers, producer, fold, channel reduction)
        for key in stats:
            mod, role = key.rsplit(".", 1)
            layer = mod.rsplit(".", 1)[0] + "."
            if role == "qkv_proj":
                groups.append((key, [f"{mod}.{p}.weight" for p in ("q_proj", "k_proj", "v_proj")],
                               layer + "input_layernorm.weight", "zc", None))
            elif role == "in_proj_qkvz":
                groups.append((key, [f"{mod}.{p}.weight" for p in ("in_proj_qkv", "in_proj_z", "in_proj_a",
                                                                     "in_proj_b")],
                               layer + "input_layernorm.weight", "zc", None))
            elif role == "gate_up_proj":
                groups.append((key, [f"{mod}.gate_proj.weight", f"{mod}.up_proj.weight"],
                               layer + "post_attention_layernorm.weight", "zc", None))
            elif role == "down_proj":
                groups.append((key, [f"{mod}.down_proj.weight"], f"{mod}.up_proj.weight", "rows", None))
            elif role == "o_proj":
                groups.append((key, [f"{mod}.o_proj.weight"], f"{mod}.v_proj.weight", "rows", "gqa"))
            elif role == "out_proj":
                groups.append((key, [f"{mod}.out_proj.weight"], f"{mod}.norm.weight", "plain", "heads"))
        wanted = {c for g in groups for c in g[1]}
        wmax = {}   # per input channel max |W| of every consumer (a first pass over the shards)
        from safetensors import safe_open
        for shard in shards:
            with safe_open(os.path.join(src, shard), framework="pt") as f:
                for name in f.keys():
                    if name in wanted:
                        wmax[name] = f.get_tensor(name).to(device, torch.float32).abs().amax(dim=0).cpu()
        self.cols, self.rows, self.norms = {}, {}, {}
        for key, consumers, producer, fold, reduce in groups:
            x = stats[key]
            w = torch.stack([wmax[c] for c in consumers]).amax(dim=0)
            if reduce == "gqa":      # o_proj input channel h * hd + d is produced by v head h // (n_q / n_kv)
                x = x.view(n_kv, n_q // n_kv, hd).amax(dim=1)
                w = w.view(n_kv, n_q // n_kv, hd).amax(dim=1)
            elif reduce == "heads":  # the GDN output norm's weight is one per dimension, shared by the value heads
                x = x.view(n_vh, vhd).amax(dim=0)
                w = w.view(n_vh, vhd).amax(dim=0)
            sc = (x.clamp(min=1e-5) ** alpha / w.clamp(min=1e-5) ** (1 - alpha)).clamp(1e-2, 1e2)
            if reduce == "gqa":
                s_cols, s_prod = sc.repeat_interleave(n_q // n_kv, dim=0).flatten(), sc.flatten()
            elif reduce == "heads":
                s_cols, s_prod = sc.repeat(n_vh), sc
            else:
                s_cols = s_prod = sc
            for c in consumers:
                self.cols[c] = s_cols
            if fold == "rows":
                self.rows[producer] = s_prod
            else:
                self.norms[producer] = (s_prod, fold)
        log(f"smoothing (alpha {alpha}): {len(groups)} groups, {len(self.cols)} consumer weights")

    def apply(self, name, t):
        """float32 smoothed tensor, or None when `name` is untouched."""
        if name not in self.cols and name not in self.rows and name not in self.norms:
            return None
        w = t.to(self.device, torch.float32)
        if name in self.cols:
            w = w * self.cols[name].to(self.device)[None, :]
        if name in self.rows:
            w = w / self.rows[name].to(self.device)[:, None]
        if name in self.norms:
            sc, fold = self.norms[name]
            sc = sc.to(self.device)
            w = (1 + w) / sc - 1 if fold == "zc" else w / sc
        return w


def convert_tensor(name, t, device, w8a16=False, group=128, mixed=False, smoothing=None):
    """-> ({name: tensor} to store, relative reconstruction error or None) for one checkpoint tensor."""
    ts = smoothing.apply(name, t) if smoothing is not None else None
    if not QUANT.match(name):
        return ({name: ts.cpu()} if ts is not None else {name: t}), None
    assert t.dim() == 2, name
    w = ts if ts is not None else t.to(device, torch.float32)
    N, K = w.shape
    w16 = w8a16 or (mixed and MIXED_W16.search(name) is not None)
    if w16 and group:
        q, scale = quant_group(w, group)
        dq = (q.view(N, K // group, group) * scale.view(N, K // group, 1)).view(N, K)
    else:
        q, scale = quant_channel(w)
        dq = q * scale
    err = ((dq - w).norm() / w.norm().clamp(min=1e-12)).item()
    if w16:
        base = name[: -len(".weight")]
        return {base + "." + k: v for k, v in pack_w16(q, scale, N, K).items()}, err
    return {name: q.to(torch.int8).cpu(), name + "_scale": scale.cpu()}, err


def convert(src, dst, device="cpu", w8a16=False, group=128, mixed=False, log=print, smooth=None, alpha=0.5):
    """Convert the checkpoint in `src` into `dst` (SmoothQuant folding first when `smooth` names a calibration
    directory); returns (tensors quantised, mean and max relative error)."""
    from safetensors import safe_open
    from safetensors.torch import save_file

    os.makedirs(dst, exist_ok=True)
    index = json.load(open(os.path.join(src, "model.safetensors.index.json")))
    shards = sorted(set(index["weight_map"].values()))
    smoothing = Smoothing(src, smooth, alpha, device, shards, log) if smooth else None
    new_map, total, errs = {}, 0, []
    for si, shard in enumerate(shards):
        out = {}
        with safe_open(os.path.join(src, shard), framework="pt") as f:
            for name in f.keys():
                tensors, err = convert_tensor(name, f.get_tensor(name), device, w8a16, group, mixed, smoothing)
                out.update(tensors)
                if err is not None:
                    errs.append(err)
        for name, t in out.items():
            new_map[name] = shard
            total += t.numel() * t.element_size()
        save_file(out, os.path.join(dst, shard), metadata={"format": "pt"})
        log(f"[{si + 1}/{len(shards)}] {shard}: {len(out)} tensors, {len(errs)} quantized so far, "
            f"max rel err {max(errs) if errs else 0.0:.4f}")
    with open(os.path.join(dst, "model.safetensors.index.json"), "w") as fh:
        json.dump({"metadata": {"total_size": total}, "weight_map": new_map}, fh, indent=2)
    for fn in os.listdir(src):   # tokenizer / processor files
        if fn.endswith(".safetensors") or fn in ("model.safetensors.index.json", "config.json") or fn.startswith("."):
            continue
        shutil.copy2(os.path.join(src, fn), os.path.join(dst, fn))
    cfg = json.load(open(os.path.join(src, "config.json")))
    cfg["quantization_config"] = quantization_config(w8a16, group, mixed)
    with open(os.path.join(dst, "config.json"), "w") as fh:
        json.dump(cfg, fh, indent=2)
    mean = sum(errs) / max(len(errs), 1)
    log(f"done: {len(errs)} tensors quantized, mean rel err {mean:.4f}, max {max(errs) if errs else 0.0:.4f}, "
        f"{total / 2**30:.2f} GiB -> {dst}")
    return len(errs), mean, (max(errs) if errs else 0.0)


def main(argv=None):
    args = list(sys.argv[1:] if argv is None else argv)
    mixed = "--mixed" in args
    if mixed:
        args.remove("--mixed")
    w8a16, group = "--w8a16" in args, 128
    if w8a16:
        i = args.index("--w8a16")
        if i + 1 < len(args) and args[i + 1].isdigit():
            group = int(args.pop(i + 1))
        args.pop(i)
    smooth, alpha = None, 0.5
    if "--smooth" in args:
        i = args.index("--smooth")
        if i + 1 >= len(args):
            raise SystemExit("vllm_turing_b200.convert: --smooth needs the calibration directory")
        smooth = args[i + 1]
        del args[i:i + 2]
    if "--alpha" in args:
        i = args.index("--alpha")
        alpha = float(args[i + 1])
        del args[i:i + 2]
    if len(args) < 2:
        raise SystemExit(__doc__)
    device = args[2] if len(args) > 2 else ("cuda" if torch.cuda.is_available() else "cpu")
    convert(args[0], args[1], device, w8a16, group, mixed, smooth=smooth, alpha=alpha)


if __name__ == "__main__":
    main()

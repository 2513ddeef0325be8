#!/usr/bin/env python3
"""Benchmark of the tensor-parallel W8A8 linear layer on B200 (one process per GPU).

Workload (BASELINE.json config 1 at N = 1, the same layer tensor-parallel at N > 1, config 2's split): one "layer" is a
decode MLP through the public API, each kernel's output feeding the next:
  gate_up : column-parallel W8A8 linear, M tokens, [5120 -> 34816 / N] (vllm_turing::scaled_mm_, the
            cutlass_scaled_mm replacement: the tcgen05 decode kernel)
  silu    : SiLU(gate) * up and per-token int8 quantisation (silu_mul_quant); --mlp fused runs gate_up and silu as one
            kernel instead (w8a8.gate_up_silu_quant)
  down    : row-parallel W8A8 linear, [17408 / N -> 5120], fused with the TP all-reduce, residual add, RMSNorm and
            per-token int8 re-quantisation (TPComm.row_linear -> vt_tp_row_linear; at N = 1 the "fused epilogue without
            collective"), whose int8 output is the next layer's input
One step = a 64-layer decode stack of such layers (the depth of config 4), every layer with its own weight buffers, so
each step streams 64 x 267 MB / N of weights from HBM (inputs far larger than L2), captured once as a CUDA graph and
replayed (as vLLM replays its captured decode forward). M = 5 tokens (1 + 4 MTP drafts) by default. Strong scaling:
the layer's total work is fixed, N ranks split it. Inputs: seeded synthetic tensors of the config's shapes and
distributions (no checkpoint offline; the per-layer buffers are copies of a few generated sets).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

Prints one JSON line (rank 0). value = whole-job int8 TOPS of the layer; us_per_layer and bus_gbs are the other two
figures of the metric. --impl reference times the reference algorithm's CPU restatement (oracle/, C + OpenMP) on the
host cores instead (the reference's own path is CUDA for sm_75 only; there is no other CPU implementation of it).
"""
import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "W8A8 linear+TP all-reduce µs/layer, TOPS & bus GB/s at 1/2/4/8 B200"
HIDDEN, INTER = 5120, 17408
VOCAB = 151936                   # config 4's LM head: int8 [5120 -> 151936], logits all-gathered
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
LAYERS = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=None, help="tokens per step (decode default 5, prefill 8192)")
    ap.add_argument("--mode", default="decode", choices=["decode", "prefill", "allreduce", "lmhead", "p2p", "gemv",
                                                         "stack"],
                    help="decode: the 64-layer MLP stack (the headline, config 1/2); prefill: the row-parallel layer "
                         "tail at config 3 (down GEMM -> two-shot all-reduce -> residual add + RMSNorm + int8 quant); "
                         "allreduce: config 4's size sweep, 1 KB .. 256 MB, against NCCL on the same ranks")
    ap.add_argument("--proj", default="down", choices=["down", "o_proj"], help="prefill: K = 17408 or 6144 (per TP)")
    ap.add_argument("--tail", default="fused", choices=["fused", "chain"],
                    help="prefill: the fused tail (TPComm.row_linear: GEMM with the reduce-scatter in its epilogue, then "
                         "reduce + all-gather + RMSNorm + quant; default) or the unfused chain of three kernels")
    ap.add_argument("--blocked", action="store_true",
                    help="decode gate_up on the tile-blocked weight layout (w8a8.block_weight / mma_blocked)")
    ap.add_argument("--mlp", default="unfused", choices=["fused", "unfused"],
                    help="decode: gate_up then SiLU*up + quant as the reference's two ops (scaled_mm_, silu_mul_quant; "
                         "default) or as one kernel (w8a8.gate_up_silu_quant; measured ~1 us per layer slower)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="short run for ncu: no clocks, e2e or CPU baseline")
    a = ap.parse_args()
    if a.tokens is None:
        a.tokens = 8192 if a.mode == "prefill" else 5
    return a


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:   # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


FALLBACK_NVLINK_GBS = 770.0   # the pool's earlier peer-copy measurement per direction (nominal 900)


def nvlink_peak():
    """(GB/s per direction, kind): the peer-copy bandwidth measured by `bench.py --mode p2p` on this pool and committed
    in profiles/nvlink_peak.txt (`peer_copy_gbs <value>`), else the pool's earlier figure."""
    try:
        with open(os.path.join(HERE, "profiles", "nvlink_peak.txt")) as f:
            for ln in f:
                p = ln.split()
                if len(p) >= 2 and p[0] == "peer_copy_gbs":
                    return float(p[1]), "measured peer copy per direction (profiles/nvlink_peak.txt)"
    except (OSError, ValueError):
        pass
    return FALLBACK_NVLINK_GBS, "fallback: the pool's earlier peer-copy figure per direction"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms from warm-up through the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-i", str(self.index),
                   "-lms", "100"]
            if shutil.which("stdbuf"):
                cmd = ["stdbuf", "-oL"] + cmd   # line-buffered: a terminated sampler loses nothing
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:   # noqa: BLE001
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:   # noqa: BLE001
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:   # noqa: BLE001
        return os.cpu_count() or 1


def layer_ops(M, world):
    """int8 ops of one layer, all ranks together (strong scaling: independent of the rank count)."""
    return 2.0 * M * (2 * INTER * HIDDEN + HIDDEN * INTER)


# ---- CPU: the oracle restatement ------------------------------------------------------------------------------------
def time_oracle_layer(M, threads, budget_s=12.0, max_steps=20):
    """The same layer (TP1) on the host cores via the C oracle -- gate_up, silu_mul_quant, down + RMSNorm + quant, the
    layer's output feeding the next step; returns (seconds per layer, steps, threads)."""
    from oracle import oracle as O
    from vllm_turing_b200.synthetic import make_layer_inputs
    O.set_threads(threads)
    gu = make_layer_inputs(M, 2 * INTER, HIDDEN, seed=1, rank=0, with_norm=False)
    dn = make_layer_inputs(M, HIDDEN, INTER, seed=0, rank=0)
    w_gu, sw_gu, w_dn, sw_dn = gu.w.numpy(), gu.sw.numpy(), dn.w.numpy(), dn.sw.numpy()
    nw = O.to_bits(dn.norm_w)
    st = {"x": gu.a.numpy(), "xs": gu.sa.numpy(), "res": O.to_bits(dn.residual)}

    def step():
        h = O.scaled_mm(st["x"], w_gu, st["xs"], sw_gu, None, 1)
        hq, hs = O.silu_mul_quant(h, 1)
        st["res"], st["x"], st["xs"], _ = O.row_linear_tp([hq], [w_dn], [hs], [sw_dn], st["res"], nw, 1e-6, 1)

    step()
    n, t0 = 0, time.perf_counter()
    while n < max_steps and (n < 2 or time.perf_counter() - t0 < budget_s):
        step()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return dt, n, threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M = args.tokens
    threads = cpu_cores()
    steps = max(1, min(args.steps, 20))
    if args.mode == "prefill":
        return run_reference_prefill(args, threads, steps)
    if args.mode == "lmhead":
        return run_reference_lmhead(args, threads, steps)
    dt, n, threads = time_oracle_layer(M, threads, budget_s=60.0, max_steps=steps)
    tops = layer_ops(M, 1) / dt / 1e12
    sample = (f"{n} full layers (M={M}, gate_up 5120->34816 + silu_mul_quant + down 17408->5120 + RMSNorm + "
              f"quant), TP1")
    line = {
        "metric": METRIC, "value": tops, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus, "steps": n,
        "warmup": 1, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic", "us_per_layer": dt * 1e6, "bus_gbs": 0.0,
        "config": {"workload": f"decode W8A8 MLP layer M={M}, hidden 5120, intermediate 17408 (BASELINE config 1)",
                   "tokens": M, "tp": 1, "device": "cpu"},
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own path is CUDA for sm_75 only; this arm is its CPU restatement (oracle/)",
    }
    print(json.dumps(line), flush=True)


def run_reference_prefill(args, threads, steps, sample_rows=256):
    """The prefill row-parallel tail (config 3) through the C oracle on the host cores, TP1, on a bounded sample of
    the batch's rows (the per-row work is identical, so time scales with rows); reported for the full batch."""
    from oracle import oracle as O
    from vllm_turing_b200.synthetic import make_layer_inputs
    O.set_threads(threads)
    M = args.tokens
    K = INTER if args.proj == "down" else 6144
    rows = min(M, sample_rows)
    li = make_layer_inputs(rows, HIDDEN, K, seed=300, rank=0)
    a, w, sa, sw = li.a.numpy(), li.w.numpy(), li.sa.numpy(), li.sw.numpy()
    res, nw = O.to_bits(li.residual), O.to_bits(li.norm_w)
    O.row_linear_tp([a], [w], [sa], [sw], res, nw, 1e-6, 1)
    n, t0 = 0, time.perf_counter()
    while n < steps and (n < 2 or time.perf_counter() - t0 < 30.0):
        O.row_linear_tp([a], [w], [sa], [sw], res, nw, 1e-6, 1)
        n += 1
    dt = (time.perf_counter() - t0) / n * (M / rows)   # seconds for the full batch
    tops = 2.0 * M * HIDDEN * K / dt / 1e12
    sample = f"{n} tails of {rows} of the {M} rows ({args.proj} K={K} -> 5120 + RMSNorm + quant), TP1, scaled by rows"
    line = {
        "metric": METRIC, "value": tops, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus, "steps": n,
        "warmup": 1, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic", "mode": "prefill", "us_per_layer": dt * 1e6, "bus_gbs": 0.0,
        "config": {"workload": f"prefill row-parallel tail M={M} (BASELINE config 3)", "tokens": M, "tp": 1,
                   "device": "cpu"},
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own path is CUDA for sm_75 only; this arm is its CPU restatement (oracle/)",
    }
    print(json.dumps(line), flush=True)


def time_oracle_lmhead(M, threads, budget_s=12.0, max_steps=20, sample_rows=8192):
    """The W8A16 LM head through the C oracle on the host cores (TP1), on a bounded sample of the vocabulary's rows
    (the per-row work is identical); returns (seconds for the full 151936-row head, calls, rows sampled)."""
    import torch
    from oracle import oracle as O
    O.set_threads(threads)
    g = torch.Generator().manual_seed(600)
    x = O.to_bits(torch.randn(M, HIDDEN, generator=g).to(torch.bfloat16))
    w = torch.randint(-128, 128, (sample_rows, HIDDEN), generator=g, dtype=torch.int8).numpy()
    sc = (torch.rand(sample_rows, generator=g) * 1e-3).numpy()
    O.w8a16(x, w, sc, None, 1)
    n, t0 = 0, time.perf_counter()
    while n < max_steps and (n < 2 or time.perf_counter() - t0 < budget_s):
        O.w8a16(x, w, sc, None, 1)
        n += 1
    return (time.perf_counter() - t0) / n * (VOCAB / sample_rows), n, sample_rows


def run_reference_lmhead(args, threads, steps):
    M = args.tokens
    dt, n, rows = time_oracle_lmhead(M, threads, budget_s=30.0, max_steps=steps)
    gbs = VOCAB * HIDDEN / dt / 1e9
    sample = f"{n} W8A16 calls on {rows} of the {VOCAB} head rows (M={M}, K=5120), TP1, scaled by rows"
    line = {
        "metric": "int8 LM head (W8A16) + logits all-gather, us per step", "value": dt * 1e6, "unit": "us",
        "impl": "reference", "n_gpus": args.gpus, "steps": n, "warmup": 1, "ms_per_step": dt * 1e3,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 x int8 -> fp32",
        "data": "synthetic", "mode": "lmhead", "weight_gbs": gbs,
        "config": {"workload": f"LM head int8 [5120 -> {VOCAB}] W8A16, M={M} (BASELINE config 4)", "tokens": M,
                   "tp": 1, "device": "cpu"},
        "cpu_baseline": {"value": dt * 1e6, "unit": "us", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": dt * 1e6, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own W8A16 kernels are CUDA; this arm is their arithmetic restated in C (oracle/)",
    }
    print(json.dumps(line), flush=True)


# ---- GPU ------------------------------------------------------------------------------------------------------------
def read_traffic():
    """DRAM bytes per launch of the kernels, from the committed ncu summary profiles/traffic.txt (`key bytes` lines,
    from `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum`). Empty when absent."""
    out = {}
    try:
        with open(os.path.join(HERE, "profiles", "traffic.txt")) as f:
            for ln in f:
                p = ln.split()
                if len(p) >= 2 and not ln.startswith("#"):
                    try:
                        out[p[0]] = float(p[1])
                    except ValueError:
                        pass
    except OSError:
        pass
    return out


def dist_setup(args):
    """One process per GPU: (world, rank, local rank, device, gloo group for set-up and barriers)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29655")
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    else:
        dist.init_process_group("gloo", rank=0, world_size=1)
        gloo = dist.group.WORLD
    return world, rank, local, dev, gloo


def torch_tail_reference(parts, residual, norm_w, eps):
    """A plain torch float32 restatement of the row-parallel tail from every rank's bf16 partial (all-gathered, exact):
    reduced = the float32 sum in rank order rounded once; residual' = bf16(reduced + residual); y = bf16(h * rsqrt(
    mean(h^2) + eps) * w); (q, scale) = per-token int8 quantisation of y (vllm_turing/quantfuse.py:18-24)."""
    import torch
    s = parts[0].float()
    for p in parts[1:]:
        s = s + p.float()
    red = s.to(residual.dtype)
    h = (red.float() + residual.float()).to(residual.dtype)
    hf = h.float()
    v = hf.pow(2).mean(-1, keepdim=True)
    y = (hf * torch.rsqrt(v + eps) * norm_w.float()).to(residual.dtype).float()
    amax = y.abs().amax(-1, keepdim=True)
    q = torch.round(y * (amax.reciprocal() * 127.0)).clamp(-128, 127).to(torch.int8)
    return red, h, q, amax / 127.0


def tail_parity(world, gloo_pg, partial, fused, chain=None):
    """Correctness of one row-parallel tail call, computed on the device and agreed over the ranks (NCCL).
    partial: this rank's bf16 [M, N] GEMM partial (vllm_turing::scaled_mm_, oracle-pinned on one GPU);
    fused / chain: dicts {reduced, residual, q} of the path under test and (optionally) of the unfused chain, both
    started from the same residual. The reference is torch_tail_reference over the all-gathered partials.
    Returns {reduced_bitexact, residual_bitexact, q_max_lsb, ranks_identical[, chain_*]} (worst over ranks)."""
    import torch
    import torch.distributed as dist
    parts = [torch.empty_like(partial) for _ in range(world)]
    if world > 1:
        dist.all_gather(parts, partial)
    else:
        parts[0].copy_(partial)
    res0 = fused["residual0"]
    red, h, q, _ = torch_tail_reference(parts, res0, fused["norm_w"], fused["eps"])

    def cmp(d):
        out = {"reduced_bitexact": bool(torch.equal(d["reduced"].view(torch.int16), red.view(torch.int16)))
               if d.get("reduced") is not None else None,
               "residual_bitexact": bool(torch.equal(d["residual"].view(torch.int16), h.view(torch.int16))),
               "q_max_lsb": int((d["q"].int() - q.int()).abs().max().item())}
        return out

    res = cmp(fused)
    # identical on every rank: compare rank 0's q and residual with this rank's
    qq = fused["q"].clone()
    rr = fused["residual"].clone()
    if world > 1:
        dist.broadcast(qq, src=0)
        dist.broadcast(rr, src=0)
    res["ranks_identical"] = bool(torch.equal(qq, fused["q"]) and torch.equal(rr, fused["residual"]))
    if chain is not None:
        for k, v in cmp(chain).items():
            res["chain_" + k] = v
    # worst over ranks: booleans by MIN, LSB counts by MAX
    keys = sorted(res)
    vals = torch.tensor([(-1.0 if res[k] is None else float(res[k])) for k in keys], dtype=torch.float64,
                        device=partial.device)
    neg = torch.tensor([0.0 if k.endswith("lsb") else 1.0 for k in keys], dtype=torch.float64, device=partial.device)
    signed = torch.where(neg > 0, -vals, vals)   # MAX of -bool = -MIN(bool)
    if world > 1:
        dist.all_reduce(signed, op=dist.ReduceOp.MAX)
    out = {}
    for k, v, n in zip(keys, signed.tolist(), neg.tolist()):
        x = -v if n > 0 else v
        out[k] = None if res[k] is None else (int(x) if k.endswith("lsb") else bool(x >= 1.0))
    out["reference"] = "torch float32 restatement over the all-gathered scaled_mm_ partials"
    return out


PREFILL_SETS = 3   # distinct layer buffers cycled by the captured step: every step's inputs are cold in L2


def prefill_kernel_name():
    """The prefill GEMM kernel the library picks (VLLM_TURING_PREFILL_WIDE=0: the 128 x 256 tiles)."""
    if os.environ.get("VLLM_TURING_PREFILL_WIDE", "1") == "0":
        return "tc_gemm_kernel (prefill, 128 x 256 tiles)"
    return "tc_gemm_wide_kernel (prefill, 256 x 256 tiles, last round as 128-row halves)"


def run_prefill(args, world, rank, local, dev, gloo):
    """Config 3: the row-parallel tail of a prefill layer -- this rank's W8A8 GEMM (tcgen05, 256 x 256 tiles) ->
    two-shot all-reduce over NVLink P2P -> residual add + RMSNorm + per-token int8 quant -- through the public API
    (vllm_turing::scaled_mm_, TPComm.all_reduce, quantfuse.rms_norm_dynamic_per_token_quant), captured in a CUDA graph.
    value = whole-job int8 TOPS of the GEMM part; us_per_layer, bus_gbs (the all-reduce's nccl-tests convention)."""
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build, w8a8
    from vllm_turing_b200.comm import TPComm
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant
    from vllm_turing_b200.synthetic import make_layer_inputs

    _build.load()
    M, N = args.tokens, HIDDEN
    K_full = INTER if args.proj == "down" else 6144
    assert K_full % world == 0
    K = K_full // world
    sets = []
    for i in range(PREFILL_SETS):
        li = make_layer_inputs(M, N, K, seed=300 + i, rank=rank)
        sets.append(dict(a=li.a.to(dev), w=li.w.to(dev), sa=li.sa.to(dev).view(-1, 1), sw=li.sw.to(dev).view(-1, 1),
                         res=li.residual.to(dev), nw=li.norm_w.to(dev),
                         out=torch.empty(M, N, dtype=torch.bfloat16, device=dev),
                         q=torch.empty(M, N, dtype=torch.int8, device=dev),
                         s=torch.empty(M, 1, dtype=torch.float32, device=dev)))
        del li
    comm = TPComm(gloo, dev, big_bytes=2 * M * N)
    stream = torch.cuda.current_stream()

    def gemm(st):
        torch.ops.vllm_turing.scaled_mm_(st["out"], st["a"], st["w"].t(), st["sa"], st["sw"], None)

    def allreduce(st):
        comm.all_reduce(st["out"], out=st["out"])

    def norm(st):
        rms_norm_dynamic_per_token_quant(st["out"], st["nw"], 1e-6, st["res"], q=st["q"], s=st["s"])

    def fused(st):   # one call: GEMM with the reduce-scatter in its epilogue, then reduce + all-gather + row epilogue
        comm.row_linear(st["a"], st["w"], st["sa"], st["sw"], residual=st["res"], norm_w=st["nw"], eps=1e-6,
                        q=st["q"], scales=st["s"], route="fused")

    STEP = (fused,) if args.tail == "fused" else (gemm, allreduce, norm)

    def run(fns):
        for st in sets:
            for fn in fns:
                fn(st)

    def barrier():
        torch.cuda.synchronize()
        dist.barrier(group=gloo)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def timed(fn, n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        barrier()
        return max_over_ranks(a.elapsed_time(b) / n) / 1e3

    K_steps, W = args.steps, max(args.warmup, 3)
    if args.profile:
        for _ in range(W + K_steps):
            run(STEP)
        barrier()
        comm.check()
        if rank == 0:
            print(json.dumps({"profile": True, "mode": "prefill", "steps": K_steps}), flush=True)
        comm.close()
        dist.destroy_process_group()
        return
    for _ in range(2):
        run(STEP)
    barrier()
    comm.check()

    # parity self-check (untimed) on set 0: the fused tail and the unfused chain (scaled_mm_ partial -> two-shot
    # vt_all_reduce -> vt_rms_norm_quant) against a torch float32 restatement over all ranks' partials
    st0 = sets[0]
    partial = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    torch.ops.vllm_turing.scaled_mm_(partial, st0["a"], st0["w"].t(), st0["sa"], st0["sw"], None)
    fz = dict(residual=st0["res"].clone(), residual0=st0["res"].clone(), norm_w=st0["nw"], eps=1e-6,
              reduced=torch.empty(M, N, dtype=torch.bfloat16, device=dev),
              q=torch.empty(M, N, dtype=torch.int8, device=dev))
    comm.row_linear(st0["a"], st0["w"], st0["sa"], st0["sw"], residual=fz["residual"], norm_w=st0["nw"], eps=1e-6,
                    q=fz["q"], scales=torch.empty(M, 1, dtype=torch.float32, device=dev), reduced=fz["reduced"])
    chk = dict(reduced=comm.all_reduce(partial.clone()), residual=st0["res"].clone())
    chk["q"], _ = rms_norm_dynamic_per_token_quant(chk["reduced"], st0["nw"], 1e-6, chk["residual"])
    barrier()
    comm.check()
    parity = tail_parity(world, gloo, partial, fz, chk)
    del partial, chk, fz

    def capture(fns):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run(fns)
        return g

    g_step = capture(STEP)
    g_k = {"gemm": capture((gemm,)), "allreduce": capture((allreduce,)), "norm": capture((norm,))}
    if args.tail == "fused":
        g_k["fused"] = capture((fused,))
    barrier()
    with ClockSampler(local) as clk:
        t_w = time.perf_counter()
        i = 0
        while i < W or time.perf_counter() - t_w < 1.0:
            g_step.replay()
            i += 1
            if i % 4 == 0:
                torch.cuda.synchronize()
        barrier()
        t_step = timed(g_step.replay, K_steps)
    W = max(W, i)
    t_layer = t_step / PREFILL_SETS
    t_k = {k: timed(g.replay, max(1, min(K_steps, 10))) / PREFILL_SETS for k, g in g_k.items()}
    comm.check()

    # end to end: the layer's activation (int8 + scales) and residual from pinned host memory, outputs read back
    e2e = None
    if not args.no_e2e:
        st0 = sets[0]
        h_a, h_sa, h_res = st0["a"].cpu().pin_memory(), st0["sa"].cpu().pin_memory(), st0["res"].cpu().pin_memory()
        o_q, o_s, o_res = (torch.empty_like(st0["q"], device="cpu").pin_memory(),
                           torch.empty_like(st0["s"], device="cpu").pin_memory(), torch.empty_like(h_res).pin_memory())
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            for fn in STEP:
                fn(st0)

        def e2e_step():
            st0["a"].copy_(h_a, non_blocking=True)
            st0["sa"].copy_(h_sa, non_blocking=True)
            st0["res"].copy_(h_res, non_blocking=True)
            g1.replay()
            o_q.copy_(st0["q"], non_blocking=True)
            o_s.copy_(st0["s"], non_blocking=True)
            o_res.copy_(st0["res"], non_blocking=True)

        for _ in range(2):
            e2e_step()
        t_e2e = timed(e2e_step, max(1, min(K_steps, 10)))
        h2d = h_a.numel() + h_sa.numel() * 4 + h_res.numel() * 2
        d2h = o_q.numel() + o_s.numel() * 4 + o_res.numel() * 2
        e2e = {"value": 2.0 * M * N * K_full / t_e2e / 1e12, "unit": "TOPS", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "us_per_layer": t_e2e * 1e6,
               "api": ("TPComm.row_linear (fused prefill tail)" if args.tail == "fused" else
                       "scaled_mm_ + TPComm.all_reduce + rms_norm_dynamic_per_token_quant") + ", captured; host copies"}
        del g1

    # roofline. The GEMM alone: int8 dense on the tensor cores against 2x the measured bf16 GEMM rate. The fused tail:
    # its floor is the slower of the GEMM and the NVLink bus bytes 2 (n - 1) / n x 2 M N (the reduce-scatter inside the
    # GEMM plus the all-gather) at the measured peer-copy bandwidth per direction; achieved = floor / measured time.
    ops_rank = 2.0 * M * N * K
    S = 2 * M * N
    bus_bytes = 2.0 * (world - 1) / world * S
    nvl, nvl_kind = nvlink_peak()
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            int8_peak, pk = 2.0 * float(json.load(f)["bf16_tflops"]), "2x measured bf16 GEMM"
    except Exception:   # noqa: BLE001
        int8_peak, pk = 2.0 * 1590.0, "2x fallback bf16"
    t_tail = t_k["fused"] if args.tail == "fused" else t_k["gemm"] + t_k["allreduce"] + t_k["norm"]
    bus = bus_bytes / t_tail / 1e9 if world > 1 else 0.0
    floor = max(ops_rank / (int8_peak * 1e12), bus_bytes / (nvl * 1e9))
    gemm_ach = ops_rank / t_k["gemm"] / 1e12
    if args.tail == "fused":
        roof = {"bound": "tensor" if ops_rank / (int8_peak * 1e12) >= bus_bytes / (nvl * 1e9) else "nvlink",
                "kernel": "tp_prefill_gemm_kernel + tp_prefill_tail_kernel (fused prefill tail)",
                "achieved": floor / t_tail, "peak": 1.0, "unit": "fraction of max(GEMM floor, NVLink floor)",
                "frac": floor / t_tail, "traffic": None, "floor_us": floor * 1e6,
                "gemm_floor_us": ops_rank / (int8_peak * 1e12) * 1e6, "nvlink_floor_us": bus_bytes / (nvl * 1e9) * 1e6,
                "gemm_alone": {"achieved": gemm_ach, "peak": int8_peak, "unit": "TOP/s", "frac": gemm_ach / int8_peak,
                               "peak_kind": pk},
                "nvlink_peak_gbs": nvl, "nvlink_peak_kind": nvl_kind, "peak_kind": pk}
    elif t_k["gemm"] >= t_k["allreduce"] or world == 1:
        roof = {"bound": "tensor", "kernel": prefill_kernel_name(), "achieved": gemm_ach,
                "peak": int8_peak, "unit": "TOP/s", "frac": gemm_ach / int8_peak, "traffic": None, "peak_kind": pk}
    else:
        ar_bus = bus_bytes / t_k["allreduce"] / 1e9
        roof = {"bound": "nvlink", "kernel": "ar_twoshot_kernel", "achieved": ar_bus, "peak": nvl, "unit": "GB/s",
                "frac": ar_bus / nvl, "traffic": None, "peak_kind": nvl_kind}
    line = {
        "metric": METRIC, "value": 2.0 * M * N * K_full / t_layer / 1e12, "unit": "TOPS", "n_gpus": world,
        "steps": K_steps, "warmup": W, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic", "mode": "prefill",
        "us_per_layer": t_layer * 1e6, "bus_gbs": bus,
        "config": {"workload": f"prefill row-parallel tail M={M}: {args.proj} GEMM {K_full}/{world} -> {N} + two-shot "
                               f"all-reduce + residual add + RMSNorm + int8 quant (BASELINE config 3), "
                               + ("fused: reduce-scatter in the GEMM epilogue, reduce + all-gather + norm in one kernel"
                                  if args.tail == "fused" else "unfused chain of three kernels"),
                   "tokens": M, "tp": world, "K_local": K, "N": N, "layers_cycled": PREFILL_SETS, "tail": args.tail,
                   "l2": "inputs larger than L2 (three layer buffer sets cycled)", "launch": "CUDA graph",
                   "parallelism": f"tp{world}"},
        "kernel_us": {k: v * 1e6 for k, v in t_k.items()},
        "roofline": roof, "clocks": clk.summary(),
        "gpu_launches": len(STEP) * PREFILL_SETS * K_steps * (2 if args.tail == "fused" else 1), "e2e": e2e,
        "cpu_baseline": None, "parity": parity,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g_step, g_k
    comm.close()
    dist.destroy_process_group()


LMHEAD_SETS = 3   # distinct head buffers cycled by the captured step: at TP8 one shard (97 MB) would fit in L2


def run_lmhead(args, world, rank, local, dev, gloo):
    """Config 4's LM head: int8 [5120 -> 151936] W8A16, vocabulary-parallel over the ranks (151936 / N rows each),
    logits all-gathered on every rank -- lmhead.logits_gathered: the tcgen05 kernel writes this rank's columns of the
    [M, 151936] logits in place, the row-strided P2P all-gather fills the peers' columns -- captured in a CUDA graph.
    value = us per step (lower is better)."""
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build, lmhead
    from vllm_turing_b200.comm import TPComm

    _build.load()
    M, K = args.tokens, HIDDEN
    assert VOCAB % world == 0
    Vs = VOCAB // world
    g = torch.Generator().manual_seed(700 + rank)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(701)).to(torch.bfloat16).to(dev)
    heads = []
    for i in range(LMHEAD_SETS):
        w = torch.randint(-128, 128, (Vs, K), generator=g, dtype=torch.int8).to(dev)
        sc = (torch.rand(Vs, generator=g) * 1e-3 + 1e-5).to(dev)
        heads.append((w, sc, torch.empty(M, VOCAB, dtype=torch.bfloat16, device=dev)))
    # one-shot capacity for this rank's logits (TP2 at M = 5: 760 KB, above the 512 KB default)
    ll = max(512 << 10, ((M * Vs * 2 + 4095) // 4096) * 4096)
    comm = TPComm(gloo, dev, ll_bytes=ll) if world > 1 else None
    stream = torch.cuda.current_stream()

    def step_set(h):
        lmhead.logits_gathered(x, h[0], h[1], comm=comm, out=h[2])

    def kernel_set(h):
        lmhead.mm_into(h[2][:, rank * Vs:], x, h[0], h[1], None, ldo=VOCAB)

    def gather_set(h):
        if comm is not None:
            comm.all_gather_rows(h[2], M, Vs * 2, VOCAB * 2)

    def run(fn):
        for h in heads:
            fn(h)

    def barrier():
        torch.cuda.synchronize()
        dist.barrier(group=gloo)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def timed(fn, n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        barrier()
        return max_over_ranks(a.elapsed_time(b) / n) / 1e3

    K_steps, W = args.steps, max(args.warmup, 3)
    for _ in range(2):
        run(step_set)
    barrier()
    if comm is not None:
        comm.check()
    if args.profile:
        for _ in range(W + K_steps):
            run(step_set)
        barrier()
        if rank == 0:
            print(json.dumps({"profile": True, "mode": "lmhead", "steps": K_steps}), flush=True)
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
        return

    def capture(fn):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            run(fn)
        return gr

    g_step, g_kern = capture(step_set), capture(kernel_set)
    g_gath = capture(gather_set) if comm is not None else None
    barrier()
    with ClockSampler(local) as clk:
        t_w = time.perf_counter()
        i = 0
        while i < W or time.perf_counter() - t_w < 1.0:
            g_step.replay()
            i += 1
            if i % 8 == 0:
                torch.cuda.synchronize()
        barrier()
        t_step = timed(g_step.replay, K_steps) / LMHEAD_SETS
    W = max(W, i)
    n_k = max(1, min(K_steps, 20))
    t_kern = timed(g_kern.replay, n_k) / LMHEAD_SETS
    t_gath = timed(g_gath.replay, n_k) / LMHEAD_SETS if g_gath is not None else 0.0
    if comm is not None:
        comm.check()

    # end to end: the hidden states from pinned host memory, the gathered logits read back (what the sampler takes)
    e2e = None
    if not args.no_e2e:
        h_x = x.cpu().pin_memory()
        o_l = torch.empty(M, VOCAB, dtype=torch.bfloat16).pin_memory()
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            step_set(heads[0])

        def e2e_step():
            x.copy_(h_x, non_blocking=True)
            g1.replay()
            o_l.copy_(heads[0][2], non_blocking=True)

        for _ in range(2):
            e2e_step()
        t_e2e = timed(e2e_step, n_k)
        e2e = {"value": t_e2e * 1e6, "unit": "us", "h2d_bytes_per_step": int(h_x.numel() * 2),
               "d2h_bytes_per_step": int(o_l.numel() * 2),
               "api": "lmhead.logits_gathered (vt_w8a16_mm + vt_all_gather_rows), captured; host copies"}
        del g1

    # roofline: the W8A16 kernel streams this rank's head once per call (HBM bound at decode M)
    alg = Vs * K + Vs * 4 + M * K * 2 + M * Vs * 2   # weights, row scales, activations, logits
    hbm_peak, pk = peaks()
    ach = alg / t_kern / 1e9
    limbs = M <= 8 and os.environ.get("VLLM_TURING_W8A16_LIMBS", "1") != "0"   # csrc/w8a16_tc.cu's choice
    kname = "w8a16_limb_kernel (int8 tcgen05 on exact activation limbs)" if limbs else "w8a16_tc_kernel"
    tr = read_traffic().get(f"w8a16_limb_tp{world}_m{M}" if limbs else f"w8a16_tp{world}_m{M}")
    roof = {"bound": "hbm", "kernel": kname, "achieved": ach, "peak": hbm_peak, "unit": "GB/s",
            "frac": ach / hbm_peak, "traffic": tr, "alg_bytes": alg, "peak_kind": pk}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, n, rows = time_oracle_lmhead(M, cpu_cores())
        cpu = {"value": dt * 1e6, "unit": "us", "cores": cpu_cores(), "kind": "port",
               "sample": f"{n} W8A16 calls on {rows} of the {VOCAB} head rows (M={M}), C oracle, scaled by rows"}
    line = {
        "metric": "int8 LM head (W8A16) + logits all-gather, us per step", "value": t_step * 1e6, "unit": "us",
        "n_gpus": world, "steps": K_steps, "warmup": W, "ms_per_step": t_step * 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 x int8 -> fp32", "data": "synthetic",
        "mode": "lmhead", "weight_gbs": Vs * K / t_kern / 1e9,
        "config": {"workload": f"LM head int8 [5120 -> {VOCAB}] W8A16, vocabulary-parallel, logits all-gathered "
                               f"(BASELINE config 4), M={M}", "tokens": M, "tp": world, "rows_per_rank": Vs,
                   "l2": "inputs larger than L2 (three head buffer sets cycled)", "launch": "CUDA graph",
                   "parallelism": f"tp{world}"},
        "kernel_us": {"w8a16": t_kern * 1e6, "all_gather_rows": t_gath * 1e6},
        "roofline": roof, "clocks": clk.summary(),
        "gpu_launches": LMHEAD_SETS * K_steps * (2 if world > 1 else 1), "e2e": e2e, "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g_step, g_kern, g_gath
    if comm is not None:
        comm.close()
    dist.destroy_process_group()


def run_allreduce(args, world, rank, local, dev, gloo):
    """Config 4's all-reduce sweep: bf16 messages of 1 KB .. 256 MB through TPComm.all_reduce (one-shot LL up to the
    LL capacity, two-shot above) and through NCCL (torch.distributed, the library baseline) on the same ranks. Each
    size: R calls captured in a CUDA graph, in place, CUDA events, max over ranks; bus GB/s = 2 (n-1)/n x bytes / t."""
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build
    from vllm_turing_b200.comm import TPComm

    _build.load()
    sizes = [1 << k for k in range(10, 29, 2)]   # 1 KB .. 256 MB
    comm = TPComm(gloo, dev)
    stream = torch.cuda.current_stream()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    rows = []
    for nbytes in sizes:
        n = nbytes // 2
        x = torch.randn(n, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16).to(dev)
        reps = 50 if nbytes <= (1 << 20) else (10 if nbytes <= (16 << 20) else 3)
        res = {}
        for impl in ("ours", "nccl"):
            if impl == "nccl" and world == 1:
                continue

            def once():
                if impl == "ours":
                    comm.all_reduce(x, out=x)
                else:
                    dist.all_reduce(x)

            for _ in range(3):
                once()
            torch.cuda.synchronize()
            dist.barrier(group=gloo)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(reps):
                    once()
            g.replay()
            torch.cuda.synchronize()
            dist.barrier(group=gloo)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            torch.cuda.synchronize()
            dist.barrier(group=gloo)
            t = max_over_ranks(a.elapsed_time(b) / reps) / 1e3
            res[impl] = t
            del g
        comm.check()
        bus = lambda t: (2.0 * (world - 1) / world * nbytes / t / 1e9) if world > 1 else 0.0   # noqa: E731
        rows.append({"bytes": nbytes, "us": res["ours"] * 1e6, "bus_gbs": bus(res["ours"]),
                     "nccl_us": res["nccl"] * 1e6 if "nccl" in res else None,
                     "nccl_bus_gbs": bus(res["nccl"]) if "nccl" in res else None})
        del x
    top = rows[-1]
    nvl, nvl_kind = nvlink_peak()
    line = {
        "metric": METRIC, "value": top["bus_gbs"], "unit": "GB/s", "n_gpus": world, "steps": 1, "warmup": 3,
        "ms_per_step": top["us"] / 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "mode": "allreduce",
        "config": {"workload": "TP all-reduce sweep 1 KB .. 256 MB, bf16, in place (BASELINE config 4)",
                   "tp": world, "launch": "CUDA graph of R calls per size", "parallelism": f"tp{world}"},
        "sweep": rows,
        "roofline": {"bound": "nvlink", "kernel": "ar_twoshot_kernel (256 MB)", "achieved": top["bus_gbs"],
                     "peak": nvl, "unit": "GB/s", "frac": top["bus_gbs"] / nvl, "traffic": None,
                     "peak_kind": nvl_kind, "frac_of_nominal_900": top["bus_gbs"] / 900.0},
        "gpu_launches": None, "e2e": None, "cpu_baseline": None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    comm.close()
    dist.destroy_process_group()


def run_gemv(args, world, rank, local, dev, gloo):
    """The decode-shape W8A8 GEMVs on one GPU: the dp4a GEMV (w8a8_gemv, the reference's kernel shape) and the tcgen05
    decode kernel (w8a8_mma) at M = 1, 5, 8 on config 1's two shapes, each over enough weight copies to exceed L2,
    captured in a CUDA graph; GB/s = algorithmic bytes N K + M K + 4 (M + N) + 2 M N per call / CUDA-event time."""
    import torch

    from vllm_turing_b200 import _build, w8a8
    from vllm_turing_b200.synthetic import make_layer_inputs

    _build.load()
    hbm, pk = peaks()
    stream = torch.cuda.current_stream()
    rows = []
    for (N, K) in ((HIDDEN, INTER), (2 * INTER, HIDDEN)):
        copies = max(2, int(4 * L2_BYTES // (N * K)) + 1)
        base = make_layer_inputs(8, N, K, seed=11, with_norm=False)
        ws_ = [base.w.to(dev) for _ in range(copies)]
        sw = base.sw.to(dev)
        for M in (1, 5, 8):
            a, sa = base.a[:M].contiguous().to(dev), base.sa[:M].contiguous().to(dev)
            out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            w8a8.workspace(dev, M, N)
            res = {}
            for name, fn in (("dp4a_gemv", w8a8.gemv), ("tcgen05_decode", w8a8.mma)):
                for w in ws_:
                    fn(out, a, w.t(), sa, sw, None)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for w in ws_:
                        fn(out, a, w.t(), sa, sw, None)
                g.replay()
                torch.cuda.synchronize()
                reps = 5
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    g.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                t = e0.elapsed_time(e1) / 1e3 / (reps * copies)
                alg = N * K + M * K + 4 * (M + N) + 2 * M * N
                res[name] = {"us": t * 1e6, "gbs": alg / t / 1e9, "frac": alg / t / 1e9 / hbm}
                del g
            rows.append({"N": N, "K": K, "M": M, **res})
        del ws_
    best = max(r["dp4a_gemv"]["gbs"] for r in rows)
    line = {
        "metric": "decode W8A8 GEMV achieved HBM GB/s", "value": best, "unit": "GB/s", "n_gpus": 1, "steps": 5,
        "warmup": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic", "mode": "gemv", "hbm_peak_gbs": hbm, "peak_kind": pk, "sweep": rows,
        "config": {"workload": "config 1 shapes (5120 <- 17408, 34816 <- 5120) at M = 1, 5, 8",
                   "l2": "inputs larger than L2 (weight copies cycled)", "launch": "CUDA graph"},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist_close()


def dist_close():
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()


def run_p2p(args, world, rank, local, dev, gloo):
    """NVLink peak for the rooflines: every rank copies B bytes into the next rank's region (a ring, so every GPU
    sends and receives at once), by SM stores (the way this package's kernels move data) and by the copy engines
    (cudaMemcpyAsync to the IPC-mapped peer address); GB/s per direction = B / t, CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build
    from vllm_turing_b200.comm import TPComm

    L = _build.load()
    assert world >= 2, "--mode p2p needs at least two ranks"
    B = 256 << 20
    comm = TPComm(gloo, dev, big_bytes=B * world)
    stream = torch.cuda.current_stream()
    peer = (rank + 1) % world
    res = {}
    with ClockSampler(local) as clk:
        for name, engine, ctas in (("sm_push", 0, 0), ("copy_engine", 1, 0), ("sm_push_1cta_per_sm", 0,
                                                                                  torch.cuda.get_device_properties(
                                                                                      dev).multi_processor_count)):
            reps = 10
            for _ in range(3):
                assert L.vt_comm_peer_copy(comm.handle, peer, B, engine, ctas, stream.cuda_stream) == 0
            torch.cuda.synchronize()
            dist.barrier(group=gloo)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                assert L.vt_comm_peer_copy(comm.handle, peer, B, engine, ctas, stream.cuda_stream) == 0
            b.record(stream)
            torch.cuda.synchronize()
            dist.barrier(group=gloo)
            t = torch.tensor([a.elapsed_time(b) / reps / 1e3], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[name] = B / t.item() / 1e9
    best = max(res.values())
    line = {
        "metric": "NVLink peer copy GB/s per direction (ring, every GPU sending and receiving)", "value": best,
        "unit": "GB/s", "n_gpus": world, "steps": 10, "warmup": 3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bytes", "data": "synthetic", "mode": "p2p", "bytes": B, "by_method": res,
        "nominal_gbs": 900.0, "frac_of_nominal": best / 900.0, "clocks": clk.summary(),
        "config": {"workload": f"{B >> 20} MiB from each rank to the next, 10 copies", "parallelism": f"tp{world}"},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    comm.close()
    dist.destroy_process_group()


QKV, HEADS_OUT = 14336, 6144   # the attention's input projection (q with its gate, k, v) and o_proj's K (24 x 256)


def run_stack(args, world, rank, local, dev, gloo):
    """a synthetic 64-layer W8A8 stack at N ranks through the public API, then the int8 LM head.
    Per layer (random-init weights of these shapes, each layer its own, so every step streams them from HBM):
      1. QKV, column-parallel: vllm_turing::scaled_mm_ 5120 -> 14336 / N, its output all-gathered along the last
         dimension (dmaag.all_gather_dim, the dmaag all-gather) -- the gathered output config 4 names;
      2. attention is out of scope: its stand-in output is this rank's first 6144 / N QKV columns, quantised per token
         (the scaled_int8_quant replacement);
      3. o_proj, row-parallel: TPComm.row_linear 6144 / N -> 5120 fused with the all-reduce, residual add, RMSNorm and
         int8 quant (decode: the one-kernel tail; prefill: the GEMM with the reduce-scatter in its epilogue + tail);
      4. gate_up 5120 -> 34816 / N + silu_mul_quant, down 17408 / N -> 5120 fused like o_proj; its int8 output is the
         next layer's input.
    Then the LM head (W8A16 on this rank's 151936 / N rows, the logits all-gathered): on all M rows at decode, on the
    last token at prefill (the sampled position). The step is captured once as a CUDA graph and replayed; value is the
    whole-job int8 TOPS of the layers (2 M (14336 + 6144 + 34816 + 17408) 5120 ops per layer)."""
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build, dmaag, lmhead, w8a8  # noqa: F401  (w8a8 registers scaled_mm_)
    from vllm_turing_b200.comm import TPComm
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant, scaled_int8_quant_cuda
    from vllm_turing_b200.synthetic import make_layer_inputs, quant_per_token
    from vllm_turing_b200.tailoverlap import silu_mul_quant

    _build.load()
    M = args.tokens
    NL = args.layers
    for full in (QKV, HEADS_OUT, 2 * INTER, INTER, VOCAB):
        assert full % world == 0, f"{full} does not split over {world} ranks"
    n_qkv, k_o, n_gu, k_dn, vs = QKV // world, HEADS_OUT // world, 2 * INTER // world, INTER // world, VOCAB // world
    prefill = M > 32
    m_head = 1 if prefill else M
    # a few generated weight sets; every layer gets its own device copy of one of them
    base = []
    for i in range(min(NL, 2)):
        qkv = make_layer_inputs(1, n_qkv, HIDDEN, seed=500 + i, rank=rank, with_norm=False)
        o = make_layer_inputs(1, HIDDEN, k_o, seed=600 + i, rank=rank)
        gu = make_layer_inputs(1, n_gu, HIDDEN, seed=700 + i, rank=rank, with_norm=False)
        dn = make_layer_inputs(1, HIDDEN, k_dn, seed=800 + i, rank=rank)
        base.append(dict(qkv_w=qkv.w.to(dev), qkv_sw=qkv.sw.to(dev).view(-1, 1), o_w=o.w.to(dev),
                         o_sw=o.sw.to(dev).view(-1, 1), gu_w=gu.w.to(dev), gu_sw=gu.sw.to(dev).view(-1, 1),
                         dn_w=dn.w.to(dev), dn_sw=dn.sw.to(dev).view(-1, 1)))
        if i == 0:
            norm_w = dn.norm_w.to(dev)
            g = torch.Generator().manual_seed(9)
            residual0 = torch.randn(M, HIDDEN, generator=g).to(torch.bfloat16).to(dev)
        del qkv, o, gu, dn
    layers = [{k: v.clone() for k, v in base[i % len(base)].items()} for i in range(NL)]
    del base
    gh = torch.Generator().manual_seed(10 + rank)
    head_w = torch.randint(-127, 128, (vs, HIDDEN), generator=gh, dtype=torch.int8).to(dev)
    head_s = (torch.rand(vs, generator=gh) * 1e-3 + 1e-4).to(dev)
    x0, xs0 = quant_per_token(torch.randn(M, HIDDEN, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16))
    x_q, x_s = x0.to(dev), xs0.view(M, 1).to(dev)
    residual = residual0.clone()
    qkv_out = torch.empty(M, n_qkv, dtype=torch.bfloat16, device=dev)
    out_gu = torch.empty(M, n_gu, dtype=torch.bfloat16, device=dev)
    h_q = torch.empty(M, k_dn, dtype=torch.int8, device=dev)
    h_s = torch.empty(M, 1, dtype=torch.float32, device=dev)
    logits = torch.empty(m_head, VOCAB, dtype=torch.bfloat16, device=dev)
    comm = TPComm(gloo, dev, big_bytes=max(2 * M * HIDDEN, 64 << 20),
                  ll_bytes=max(512 << 10, m_head * VOCAB * 2 // world))
    w8a8.workspace(dev, M, max(n_qkv, n_gu))
    lmhead.workspace(dev, HIDDEN)
    stream = torch.cuda.current_stream()

    def layer(s):
        torch.ops.vllm_turing.scaled_mm_(qkv_out, x_q, s["qkv_w"].t(), x_s, s["qkv_sw"], None)
        if world > 1:
            dmaag.all_gather_dim(comm, qkv_out, -1)   # column-parallel output, gathered (config 4)
        a_q, a_s = scaled_int8_quant_cuda(qkv_out[:, :k_o])   # the attention output's stand-in
        comm.row_linear(a_q, s["o_w"], a_s, s["o_sw"], residual=residual, norm_w=norm_w, eps=1e-6, q=x_q, scales=x_s)
        torch.ops.vllm_turing.scaled_mm_(out_gu, x_q, s["gu_w"].t(), x_s, s["gu_sw"], None)
        silu_mul_quant(out_gu, h_q, h_s)
        comm.row_linear(h_q, s["dn_w"], h_s, s["dn_sw"], residual=residual, norm_w=norm_w, eps=1e-6, q=x_q, scales=x_s)

    def head():
        lmhead.logits_gathered(residual[M - m_head:], head_w, head_s, comm=comm if world > 1 else None, out=logits)

    def step():
        for s in layers:
            layer(s)
        head()

    def barrier():
        torch.cuda.synchronize()
        dist.barrier(group=gloo)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def timed(fn, n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        barrier()
        return max_over_ranks(a.elapsed_time(b) / n) / 1e3

    K_steps, W = args.steps, max(args.warmup, 3)
    step()   # eager warm-up: kernel attributes, workspaces
    barrier()
    comm.check()
    # parity self-check (untimed) on layer 0's o_proj tail: the public call (TPComm.row_linear, whichever route it
    # takes) and the unfused chain from the same inputs, both against a torch float32 restatement
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant  # noqa: F811
    s0 = layers[0]
    a_q, a_s = scaled_int8_quant_cuda(qkv_out[:, :k_o].contiguous())
    partial = torch.empty(M, HIDDEN, dtype=torch.bfloat16, device=dev)
    torch.ops.vllm_turing.scaled_mm_(partial, a_q, s0["o_w"].t(), a_s, s0["o_sw"], None)
    fz = dict(residual=residual.clone(), residual0=residual.clone(), norm_w=norm_w, eps=1e-6,
              reduced=torch.empty(M, HIDDEN, dtype=torch.bfloat16, device=dev),
              q=torch.empty(M, HIDDEN, dtype=torch.int8, device=dev))
    comm.row_linear(a_q, s0["o_w"], a_s, s0["o_sw"], residual=fz["residual"], norm_w=norm_w, eps=1e-6, q=fz["q"],
                    scales=torch.empty(M, 1, dtype=torch.float32, device=dev), reduced=fz["reduced"])
    chk = dict(reduced=comm.all_reduce(partial.clone()), residual=residual.clone())
    chk["q"], _ = rms_norm_dynamic_per_token_quant(chk["reduced"], norm_w, 1e-6, chk["residual"])
    barrier()
    comm.check()
    parity = tail_parity(world, gloo, partial, fz, chk)
    del a_q, a_s, partial, fz, chk

    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        step()
    g_head = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_head):
        head()
    for _ in range(W):
        g_step.replay()
    barrier()
    comm.check()
    with ClockSampler(local) as clk:
        t_step = timed(g_step.replay, K_steps)
        t_head = timed(g_head.replay, max(K_steps, 10))
    comm.check()
    # the logits agree on every rank (each holds the gathered [m_head, 151936])
    lb = logits.view(torch.int16).to(torch.int32)
    l0 = lb.clone()
    if world > 1:
        dist.broadcast(l0, src=0)
    parity["logits_ranks_identical"] = bool(torch.equal(l0, lb))

    e2e = None
    if not args.no_e2e:
        h_x, h_xs = x0.pin_memory(), xs0.view(M, 1).pin_memory()
        h_l = torch.empty(m_head, VOCAB, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            x_q.copy_(h_x, non_blocking=True)
            x_s.copy_(h_xs, non_blocking=True)
            g_step.replay()
            h_l.copy_(logits, non_blocking=True)

        for _ in range(2):
            e2e_step()
        t_e2e = timed(e2e_step, K_steps)
        e2e = {"value": NL * 2.0 * M * HIDDEN * (QKV + HEADS_OUT + 2 * INTER + INTER) / (t_e2e - t_head) / 1e12
               if t_e2e > t_head else None, "unit": "TOPS (layers only)", "step_ms": t_e2e * 1e3,
               "h2d_bytes_per_step": int(h_x.numel() + h_xs.numel() * 4),
               "d2h_bytes_per_step": int(h_l.numel() * 2),
               "api": "the captured step (scaled_mm_, all_gather_dim, scaled_int8_quant, TPComm.row_linear, "
                      "silu_mul_quant, lmhead.logits_gathered); pinned host input copied in, logits read back"}
    ops_layer = 2.0 * M * HIDDEN * (QKV + HEADS_OUT + 2 * INTER + INTER)
    t_layers = t_step - t_head
    line = {
        "metric": "config-4 64-layer W8A8 TP stack: whole-job int8 TOPS of the layers, us per layer, LM head us",
        "value": NL * ops_layer / t_layers / 1e12, "unit": "TOPS", "n_gpus": world, "steps": K_steps, "warmup": W,
        "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic", "mode": "stack",
        "us_per_layer": t_layers / NL * 1e6, "lmhead_us": t_head * 1e6,
        "tokens_per_s": M / t_step,
        "config": {"workload": f"BASELINE config 4: {NL} layers of QKV 5120->14336 (column-parallel, all-gathered), "
                               f"o_proj 6144->5120 and down 17408->5120 (row-parallel, fused all-reduce + residual + "
                               f"RMSNorm + int8 quant), gate_up 5120->34816 + SiLU*up + quant; int8 LM head "
                               f"5120->151936 on {m_head} row(s), logits all-gathered; M={M}",
                   "tokens": M, "layers": NL, "tp": world, "head_rows": m_head,
                   "l2": f"inputs larger than L2: {NL} layers with their own weights",
                   "launch": "CUDA graph of the step, replayed K times", "parallelism": f"tp{world}"},
        "clocks": clk.summary(), "e2e": e2e, "cpu_baseline": None, "parity": parity,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g_step, g_head
    comm.close()
    dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build, w8a8
    from vllm_turing_b200.comm import TPComm
    from vllm_turing_b200.synthetic import make_layer_inputs, quant_per_token
    from vllm_turing_b200.tailoverlap import silu_mul_quant

    world, rank, local, dev, gloo = dist_setup(args)
    if args.mode == "prefill":
        return run_prefill(args, world, rank, local, dev, gloo)
    if args.mode == "allreduce":
        return run_allreduce(args, world, rank, local, dev, gloo)
    if args.mode == "lmhead":
        return run_lmhead(args, world, rank, local, dev, gloo)
    if args.mode == "p2p":
        return run_p2p(args, world, rank, local, dev, gloo)
    if args.mode == "gemv":
        return run_gemv(args, world, rank, local, dev, gloo)
    if args.mode == "stack":
        return run_stack(args, world, rank, local, dev, gloo)
    _build.load()
    M = args.tokens
    NL = args.layers
    assert INTER % world == 0 and (2 * INTER) % world == 0
    K_dn, N_gu = INTER // world, 2 * INTER // world
    bytes_gu_w = N_gu * HIDDEN
    bytes_dn_w = HIDDEN * K_dn
    base = []   # a few generated weight sets; every layer gets its own device copy of one of them
    for i in range(min(NL, 2)):
        gu = make_layer_inputs(M, N_gu, HIDDEN, seed=100 + i, rank=rank, with_norm=False)
        dn = make_layer_inputs(M, HIDDEN, K_dn, seed=i, rank=rank)
        gw, gsw = gu.w.to(dev), gu.sw.to(dev).view(-1, 1)
        st = dict(gu_w=gw, gu_sw=gsw, dn_w=dn.w.to(dev), dn_sw=dn.sw.to(dev).view(-1, 1))
        if args.mlp == "fused":   # weight layouts are made once, at load time
            st["gu_wi"], st["gu_si"] = w8a8.interleave_gate_up(gw, gsw)
        if args.blocked:
            st["gu_wb"] = w8a8.block_weight(gw)
        base.append(st)
        if i == 0:
            residual0, norm_w = dn.residual.to(dev), dn.norm_w.to(dev)
    keep = ("gu_wi", "gu_si") if args.mlp == "fused" else (("gu_wb", "gu_sw") if args.blocked else ("gu_w", "gu_sw"))
    layers = [{k: v.clone() for k, v in base[i % len(base)].items() if k in keep or k.startswith("dn_")}
              for i in range(NL)]
    del base
    # the stack's input: one hidden state every rank holds (seeded independently of the rank), quantised per token
    x0, xs0 = quant_per_token(torch.randn(M, HIDDEN, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16))
    xs0 = xs0.view(M, 1)
    x_q, x_s = x0.to(dev), xs0.to(dev)          # layer input, rewritten by every layer's down epilogue
    residual = residual0.clone()
    out_gu = torch.empty(M, N_gu, dtype=torch.bfloat16, device=dev)
    h_q = torch.empty(M, K_dn, dtype=torch.int8, device=dev)
    h_s = torch.empty(M, 1, dtype=torch.float32, device=dev)
    comm = TPComm(gloo, dev)
    w8a8.workspace(dev, M, N_gu)
    stream = torch.cuda.current_stream()

    # one decode MLP layer through the public API: vllm_turing::scaled_mm_ (the cutlass_scaled_mm replacement),
    # silu_mul_quant, and the fused row-parallel tail (down GEMM + all-reduce + residual + RMSNorm + int8 quant, whose
    # output is the next layer's input)
    def gate_up(s):
        if args.blocked:
            w8a8.mma_blocked(out_gu, x_q, s["gu_wb"], x_s, s["gu_sw"])
        else:
            torch.ops.vllm_turing.scaled_mm_(out_gu, x_q, s["gu_w"].t(), x_s, s["gu_sw"], None)

    def silu(s):
        silu_mul_quant(out_gu, h_q, h_s)

    def gate_up_silu(s):
        w8a8.gate_up_silu_quant(x_q, s["gu_wi"], x_s, s["gu_si"], q=h_q, scales=h_s)

    def down(s):
        comm.row_linear(h_q, s["dn_w"], h_s, s["dn_sw"], residual=residual, norm_w=norm_w, eps=1e-6, q=x_q, scales=x_s)

    def run(fns, sets):
        for s in sets:
            for fn in fns:
                fn(s)

    def barrier():
        torch.cuda.synchronize()
        dist.barrier(group=gloo)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    LAYER = (gate_up_silu, down) if args.mlp == "fused" else (gate_up, silu, down)
    K, W = args.steps, max(args.warmup, 1 if args.profile else 3)
    if args.profile:   # eager launches of two layers, for ncu launch lists and captures
        for i in range(W + K):
            run(LAYER, layers[:2])
        barrier()
        comm.check()
        if rank == 0:
            print(json.dumps({"profile": True, "steps": K}), flush=True)
        comm.close()
        dist.destroy_process_group()
        return

    # eager warm-up (sets every kernel's one-time attributes), then one CUDA graph per timed region: the NL-layer step,
    # and each kernel alone over the NL layers' buffers (the roofline's per-kernel durations)
    for _ in range(2):
        run(LAYER, layers)
    barrier()
    comm.check()

    # ---- parity self-check (untimed) on layer 0's down projection: the fused kernel and the unfused chain
    # (scaled_mm_ partial -> vt_all_reduce -> vt_rms_norm_quant) against a torch float32 restatement over every rank's
    # partial; the same calls in the same order on every rank ----
    from vllm_turing_b200.quantfuse import rms_norm_dynamic_per_token_quant
    s0 = layers[0]
    a_p, sa_p = h_q.clone(), h_s.clone()
    partial = torch.empty(M, HIDDEN, dtype=torch.bfloat16, device=dev)
    torch.ops.vllm_turing.scaled_mm_(partial, a_p, s0["dn_w"].t(), sa_p, s0["dn_sw"], None)
    res_before = residual.clone()
    fused = dict(residual=residual.clone(), reduced=torch.empty(M, HIDDEN, dtype=torch.bfloat16, device=dev),
                 q=torch.empty(M, HIDDEN, dtype=torch.int8, device=dev), residual0=res_before, norm_w=norm_w, eps=1e-6)
    comm.row_linear(a_p, s0["dn_w"], sa_p, s0["dn_sw"], residual=fused["residual"], norm_w=norm_w, eps=1e-6,
                    q=fused["q"], scales=torch.empty(M, 1, dtype=torch.float32, device=dev), reduced=fused["reduced"])
    chain = dict(reduced=comm.all_reduce(partial.clone()), residual=residual.clone())
    chain["q"], _ = rms_norm_dynamic_per_token_quant(chain["reduced"], norm_w, 1e-6, chain["residual"])
    barrier()
    comm.check()
    parity = tail_parity(world, gloo, partial, fused, chain)
    del a_p, sa_p, partial, fused, chain

    def capture(fns):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run(fns, layers)
        return g

    g_step = capture(LAYER)
    if args.mlp == "fused":
        g_k = {"gate_up_silu": capture((gate_up_silu,)), "down": capture((down,))}
    else:
        g_k = {"gate_up": capture((gate_up,)), "silu": capture((silu,)), "down": capture((down,))}
    barrier()

    def timed(fn, n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        barrier()
        return max_over_ranks(a.elapsed_time(b) / n) / 1e3

    # ---- timed region: K replays of the NL-layer step; clocks sampled from a warm-up of at least 1 s of the same load
    # through the end of the timed region ----
    x_q.copy_(x0)
    x_s.copy_(xs0)
    residual.copy_(residual0)
    with ClockSampler(local) as clk:
        t_w = time.perf_counter()
        i = 0
        while i < W or time.perf_counter() - t_w < 1.0:
            g_step.replay()
            i += 1
            if i % 8 == 0:
                torch.cuda.synchronize()
        barrier()
        comm.check()
        t_step = timed(g_step.replay, K)                           # seconds per step, max over ranks
    W = max(W, i)
    t_layer = t_step / NL
    comm.check()

    passes = max(1, min(K, 20))
    t_k = {k: timed(g.replay, passes) / NL for k, g in g_k.items()}
    comm.check()

    # the latency floor of the fused down kernel at N > 1: the one-shot all-reduce of its M x 5120 bf16 message alone
    # (NL calls in a graph, as the step), next to its weight stream's HBM floor
    t_ll = None
    if world > 1:
        msg = torch.zeros(M, HIDDEN, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            comm.all_reduce(msg, out=msg, algo=1)
        barrier()
        g_ll = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_ll):
            for _ in range(NL):
                comm.all_reduce(msg, out=msg, algo=1)
        t_ll = timed(g_ll.replay, passes) / NL
        comm.check()
        del g_ll

    # the same step launched eagerly (no graph): host-side launch cost included
    t_eager = timed(lambda: run(LAYER, layers), max(1, min(K, 10))) / NL
    comm.check()

    # ---- end to end with host buffers: each step copies the stack's inputs (layer 0's quantised hidden state and its
    # scales, the residual) from pinned host memory, replays the captured public-API calls (as vLLM's decode replays its
    # captured forward) and reads the outputs (next hidden state, scales, residual) back ----
    e2e = None
    if not args.no_e2e:
        h_x, h_xs, h_res = x0.pin_memory(), xs0.pin_memory(), residual0.cpu().pin_memory()
        o_x, o_xs, o_res = (torch.empty_like(h_x).pin_memory(), torch.empty_like(h_xs).pin_memory(),
                            torch.empty_like(h_res).pin_memory())
        h2d = h_x.numel() + h_xs.numel() * 4 + h_res.numel() * 2
        d2h = o_x.numel() + o_xs.numel() * 4 + o_res.numel() * 2

        def e2e_step():
            x_q.copy_(h_x, non_blocking=True)
            x_s.copy_(h_xs, non_blocking=True)
            residual.copy_(h_res, non_blocking=True)
            g_step.replay()
            o_x.copy_(x_q, non_blocking=True)
            o_xs.copy_(x_s, non_blocking=True)
            o_res.copy_(residual, non_blocking=True)

        for _ in range(W):
            e2e_step()
        t_e2e = timed(e2e_step, K)
        comm.check()
        e2e = {"value": layer_ops(M, world) * NL / t_e2e / 1e12, "unit": "TOPS", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "us_per_layer": t_e2e / NL * 1e6,
               "api": ("w8a8.gate_up_silu_quant" if args.mlp == "fused" else "vllm_turing::scaled_mm_ + silu_mul_quant")
                   + " + TPComm.row_linear per layer, captured in a CUDA graph; pinned host inputs copied in and "
                     "outputs read back every step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, n, thr = time_oracle_layer(M, cpu_cores())
        cpu = {"value": layer_ops(M, 1) / dt / 1e12, "unit": "TOPS", "cores": thr, "kind": "port",
               "sample": f"{n} full TP1 layers (M={M}: gate_up + silu_mul_quant + down + RMSNorm + quant) through the "
                         f"C oracle, OpenMP"}

    # algorithmic HBM bytes per launch (one layer) of each kernel
    alg = {"gate_up": bytes_gu_w + M * HIDDEN + 4 * M + 4 * N_gu + 2 * M * N_gu,
           "gate_up_silu": bytes_gu_w + M * HIDDEN + 4 * M + 4 * N_gu + M * K_dn + 4 * M,
           "silu": 2 * M * N_gu + M * K_dn + 4 * M,
           "down": bytes_dn_w + M * K_dn + 4 * M + 4 * HIDDEN + M * HIDDEN * (2 + 2 + 1) + 4 * M + 2 * HIDDEN}
    names = {"gate_up": "tc_gemm_kernel (gate_up, tcgen05 decode)", "silu": "silu_mul_quant_kernel",
             "gate_up_silu": "gate_up_silu_kernel (gate_up + SiLU*up + int8 quant, tcgen05 decode)",
             "down": ("tp_row_linear_tc_kernel" if os.environ.get("VLLM_TURING_DECODE_TAIL") == "rows" else
                      "tp_row_linear_tt_kernel") + " (down + all-reduce + RMSNorm + quant)"}
    dom = max(t_k, key=t_k.get)
    hbm, peak_kind = peaks()
    achieved = alg[dom] / t_k[dom] / 1e9
    traffic = read_traffic().get(f"{dom}_tp{world}_m{M}")

    # bus GB/s of the layer's all-reduce (nccl-tests convention, 2 (n - 1) / n x message bytes / time): the one-shot
    # all-reduce of the down projection's [M, 5120] bf16 message, timed alone in a captured graph of NL calls; the
    # same bytes over the whole layer's time beside it
    S = 2 * M * HIDDEN
    bus = (2.0 * (world - 1) / world * S / t_ll / 1e9) if t_ll else 0.0
    bus_layer = (2.0 * (world - 1) / world * S / t_layer / 1e9) if world > 1 else 0.0
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": layer_ops(M, world) / t_layer / 1e12, "unit": "TOPS", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "us_per_layer": t_layer * 1e6, "bus_gbs": bus, "bus_gbs_over_layer": bus_layer,
        "config": {"workload": f"decode W8A8 MLP stack of {NL} layers, M={M}: gate_up 5120->34816 column-parallel "
                               f"with SiLU*up + int8 quant ({'one kernel' if args.mlp == 'fused' else 'two ops'}), "
                               f"down 17408->5120 row-parallel fused with TP all-reduce + RMSNorm + int8 quant "
                               f"(BASELINE config 1 per layer at N=1, config 2 split at N>1)",
                   "tokens": M, "layers": NL, "tp": world, "K_down_local": K_dn, "N_gate_up_local": N_gu,
                   "l2": f"inputs larger than L2: {NL} layers with their own weights, "
                         f"{NL * (bytes_gu_w + bytes_dn_w) / 2**20:.0f} MiB of weights per step",
                   "launch": "CUDA graph of the step, replayed K times", "parallelism": f"tp{world}"},
        "kernel_us": {k: v * 1e6 for k, v in t_k.items()},
        "eager_us_per_layer": t_eager * 1e6,
        "roofline": {"bound": "hbm", "kernel": names[dom], "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic, "bytes_per_launch": alg[dom],
                     "peak_kind": peak_kind},
        # the fused down kernel against its own floor: max(weight stream at the HBM peak, the one-shot all-reduce of
        # its message measured alone); frac = floor / its measured time
        "down_roofline": {"hbm_floor_us": alg["down"] / (hbm * 1e9) * 1e6,
                          "oneshot_us": t_ll * 1e6 if t_ll is not None else None,
                          "floor_us": max(alg["down"] / (hbm * 1e9), t_ll or 0.0) * 1e6,
                          "measured_us": t_k["down"] * 1e6,
                          "frac": max(alg["down"] / (hbm * 1e9), t_ll or 0.0) / t_k["down"],
                          "hbm_gbs": alg["down"] / t_k["down"] / 1e9},
        "clocks": clocks, "gpu_launches": len(LAYER) * NL * K, "e2e": e2e, "cpu_baseline": cpu, "parity": parity,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g_step, g_k
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

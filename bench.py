#!/usr/bin/env python3
"""Benchmark of the tensor-parallel W8A8 linear layer on B200 (one process per GPU).

Workload (BASELINE.json config 1 at N = 1, the same layer tensor-parallel at N > 1, config 2's split): one "layer" =
  gate_up : column-parallel W8A8 GEMV, M tokens, [5120 -> 34816 / N]  (w8a8_gemv_ws)
  down    : row-parallel W8A8 GEMV, [17408 / N -> 5120] fused with the TP all-reduce, residual add, RMSNorm and per-token
            int8 re-quantisation (vt_tp_row_linear; at N = 1 the "fused epilogue without collective")
One step = a 64-layer decode stack of such layers (the depth of config 4), every layer with its own weight buffers, so
each step streams 64 x 267 MB / N of weights from HBM (inputs far larger than L2). M = 5 tokens (1 + 4 MTP drafts) by
default. Strong scaling: the layer's total work is fixed, N ranks split it. Inputs: seeded synthetic tensors of the
config's shapes and distributions (no checkpoint offline; the per-layer buffers are copies of a few generated sets).

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
    ap.add_argument("--tokens", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="short run for ncu: no clocks, e2e or CPU baseline")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:   # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


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
    """The same layer (TP1) on the host cores via the C oracle; returns (seconds per layer, steps, threads)."""
    import numpy as np

    from oracle import oracle as O
    from vllm_turing_b200.synthetic import make_layer_inputs
    O.set_threads(threads)
    gu = make_layer_inputs(M, 2 * INTER, HIDDEN, seed=1, rank=0, with_norm=False)
    dn = make_layer_inputs(M, HIDDEN, INTER, seed=0, rank=0)
    a_gu, w_gu, sa_gu, sw_gu = gu.a.numpy(), gu.w.numpy(), gu.sa.numpy(), gu.sw.numpy()
    args = ([dn.a.numpy()], [dn.w.numpy()], [dn.sa.numpy()], [dn.sw.numpy()])
    res, nw = O.to_bits(dn.residual), O.to_bits(dn.norm_w)

    def step():
        O.scaled_mm(a_gu, w_gu, sa_gu, sw_gu, None, 1)
        O.row_linear_tp(*args, res, nw, 1e-6, 1)

    step()
    n, t0 = 0, time.perf_counter()
    while n < max_steps and (n < 2 or time.perf_counter() - t0 < budget_s):
        step()
        n += 1
    dt = (time.perf_counter() - t0) / n
    del np
    return dt, n, threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M = args.tokens
    threads = cpu_cores()
    steps = max(1, min(args.steps, 20))
    dt, n, threads = time_oracle_layer(M, threads, budget_s=60.0, max_steps=steps)
    tops = layer_ops(M, 1) / dt / 1e12
    sample = f"{n} full layers (M={M}, gate_up 5120->34816 + down 17408->5120 + all-reduce + RMSNorm + quant), TP1"
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


# ---- GPU ------------------------------------------------------------------------------------------------------------
def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist

    from vllm_turing_b200 import _build, w8a8
    from vllm_turing_b200.comm import TPComm
    from vllm_turing_b200.synthetic import make_layer_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29655")
    from datetime import timedelta
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    else:
        dist.init_process_group("gloo", rank=0, world_size=1)
        gloo = dist.group.WORLD
    L = _build.load()
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
        base.append(dict(gu_a=gu.a.to(dev), gu_w=gu.w.to(dev), gu_sa=gu.sa.to(dev), gu_sw=gu.sw.to(dev),
                         dn_a=dn.a.to(dev), dn_w=dn.w.to(dev), dn_sa=dn.sa.to(dev), dn_sw=dn.sw.to(dev)))
        if i == 0:
            residual0, norm_w = dn.residual.to(dev), dn.norm_w.to(dev)
    sets = []
    for i in range(NL):
        b = base[i % len(base)]
        sets.append({k: (v.clone() if k in ("gu_w", "dn_w") else v) for k, v in b.items()})
    R = NL
    comm = TPComm(gloo, dev)
    out_gu = torch.empty(M, N_gu, dtype=torch.bfloat16, device=dev)
    residual = residual0.clone()
    q = torch.empty(M, HIDDEN, dtype=torch.int8, device=dev)
    scales = torch.empty(M, 1, dtype=torch.float32, device=dev)
    w8a8.workspace(dev, M, N_gu)
    stream = torch.cuda.current_stream()

    def gate_up(s):
        w8a8.gemv(out_gu, s["gu_a"], s["gu_w"].t(), s["gu_sa"], s["gu_sw"], None)

    def down(s):
        comm.row_linear(s["dn_a"], s["dn_w"], s["dn_sa"], s["dn_sw"], residual=residual, norm_w=norm_w, eps=1e-6,
                        q=q, scales=scales)

    def step(i):
        for s in sets:
            gate_up(s)
            down(s)

    def barrier():
        torch.cuda.synchronize()
        dist.barrier(group=gloo)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    K, W = args.steps, max(args.warmup, 1 if args.profile else 3)
    if args.profile:
        sets = sets[:2]
        for i in range(W + K):
            step(i)
        barrier()
        comm.check()
        if rank == 0:
            print(json.dumps({"profile": True, "steps": K}), flush=True)
        comm.close()
        dist.destroy_process_group()
        return

    # ---- timed region: K steps of the NL-layer stack; clocks sampled from warm-up (at least 1 s of the same load)
    # through the end of the timed region ----
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t_w = time.perf_counter()
        i = 0
        while i < W or time.perf_counter() - t_w < 1.0:
            step(i)
            i += 1
            if i % 8 == 0:
                torch.cuda.synchronize()
        barrier()
        comm.check()
        e0.record(stream)
        for i in range(K):
            step(i)
        e1.record(stream)
        barrier()
    W = max(W, i)
    t_step = max_over_ranks(e0.elapsed_time(e1) / K) / 1e3          # seconds per step, max over ranks
    t_layer = t_step / NL
    comm.check()

    # ---- per-kernel durations for the roofline: each kernel alone over the NL layers' buffers, K passes, CUDA events on
    # the launching stream ----
    def time_kernel(fn, passes):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for _ in range(passes):
            for s in sets:
                fn(s)
        b.record(stream)
        barrier()
        return max_over_ranks(a.elapsed_time(b) / (passes * NL)) / 1e3

    passes = max(1, min(K, 20))
    t_gu = time_kernel(gate_up, passes)
    t_dn = time_kernel(down, passes)
    comm.check()
    gu_bytes = bytes_gu_w + M * HIDDEN + 2 * M * N_gu + 4 * (M + N_gu)
    dn_bytes = bytes_dn_w + M * K_dn + 4 * (M + HIDDEN) + M * HIDDEN * (2 + 2 + 1) + 4 * M + 2 * HIDDEN
    hbm, peak_kind = peaks()
    dom = ("w8a8_gemv (gate_up)", t_gu, gu_bytes) if t_gu >= t_dn else ("tp_row_linear (down+AR+norm+quant)", t_dn,
                                                                           dn_bytes)
    achieved = dom[2] / dom[1] / 1e9

    # ---- end to end through the public API with host buffers: every step copies the stack's inputs (the first
    # layer's activations and scales, the residual) from pinned host memory and reads its outputs back ----
    e2e = None
    if not args.no_e2e:
        s0 = sets[0]
        h_in = {k: s0[k].cpu().pin_memory() for k in ("gu_a", "gu_sa", "dn_a", "dn_sa")}
        h_res = residual0.cpu().pin_memory()
        h_q = torch.empty(M, HIDDEN, dtype=torch.int8).pin_memory()
        h_s = torch.empty(M, 1, dtype=torch.float32).pin_memory()
        h_r = torch.empty_like(h_res).pin_memory()
        d_in = {k: torch.empty_like(v, device=dev) for k, v in h_in.items()}
        h2d = sum(v.numel() * v.element_size() for v in h_in.values()) + h_res.numel() * 2
        d2h = h_q.numel() + h_s.numel() * 4 + h_r.numel() * 2
        first = dict(sets[0])
        first.update(d_in)

        def e2e_step(i):
            for k, v in h_in.items():
                d_in[k].copy_(v, non_blocking=True)
            residual.copy_(h_res, non_blocking=True)
            for j, s in enumerate(sets):
                s = first if j == 0 else s
                gate_up(s)
                down(s)
            h_q.copy_(q, non_blocking=True)
            h_s.copy_(scales, non_blocking=True)
            h_r.copy_(residual, non_blocking=True)

        for i in range(args.warmup):
            e2e_step(i)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        for i in range(K):
            e2e_step(i)
        b.record(stream)
        barrier()
        t_e2e = max_over_ranks(a.elapsed_time(b) / K) / 1e3
        comm.check()
        e2e = {"value": layer_ops(M, world) * NL / t_e2e / 1e12, "unit": "TOPS", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "us_per_layer": t_e2e / NL * 1e6,
               "api": "w8a8.gemv + TPComm.row_linear over the stack, pinned host inputs / outputs copied every step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, n, thr = time_oracle_layer(M, cpu_cores())
        cpu = {"value": layer_ops(M, 1) / dt / 1e12, "unit": "TOPS", "cores": thr, "kind": "port",
               "sample": f"{n} full TP1 layers (M={M}) through the C oracle, OpenMP"}

    S = 2 * M * HIDDEN
    bus = (2.0 * (world - 1) / world * S / t_layer / 1e9) if world > 1 else 0.0
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": layer_ops(M, world) / t_layer / 1e12, "unit": "TOPS", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "us_per_layer": t_layer * 1e6, "bus_gbs": bus,
        "config": {"workload": f"decode W8A8 MLP stack of {NL} layers, M={M}: gate_up 5120->34816 column-parallel + "
                               f"down 17408->5120 row-parallel fused with TP all-reduce + RMSNorm + int8 quant "
                               f"(BASELINE config 1 per layer at N=1, config 2 split at N>1)",
                   "tokens": M, "layers": NL, "tp": world, "K_down_local": K_dn, "N_gate_up_local": N_gu,
                   "l2": f"inputs larger than L2: {NL} layers with their own weights, "
                         f"{NL * (bytes_gu_w + bytes_dn_w) / 2**20:.0f} MiB of weights per step",
                   "parallelism": f"tp{world}"},
        "kernel_us": {"w8a8_gemv_gate_up": t_gu * 1e6, "tp_row_linear_down": t_dn * 1e6},
        "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": None, "bytes_per_launch": dom[2],
                     "peak_kind": peak_kind},
        "clocks": clocks, "gpu_launches": 2 * NL * K, "e2e": e2e, "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Multi-rank collectives and the fused row-linear on 2..8 GPUs, one process per GPU (the reference's test pattern:
torch.multiprocessing.spawn, a gloo group for set-up, tests/test_hostar.py:13-20), against the CPU oracle:
  - one-shot and two-shot all-reduce bit-exact to the rank-ordered float32 sum (tests/bench_devll.py:28-36 for 2 ranks)
    at decode / odd / prefill sizes, fp16 and bf16, identical on every rank;
  - all-gather (LL and bulk, contiguous slots and row-strided along the last dimension) exact;
  - AR8 (int8 + fp16 scale per 128 values, all-gathered, rank-ordered sum) bit-exact to the oracle;
  - the int8 LM head's vocabulary-parallel logits at config 4's TP8 shard (151936 / 8 rows x 5120) gathered in place
    on every rank, within the W8A16 tolerance of the oracle;
  - the fused GEMV + all-reduce + residual + RMSNorm + quant at BASELINE config 0 (M=16, K_local=8704, N=5120) and
    config 2 (M in {1, 5}, K = 17408 / world): reduced sum bit-exact, residual bit-exact, int8 within 1 LSB;
  - the prefill row-linear on both routes (the fused tail, and the GEMM -> two-shot -> norm chain), the same bar;
  - 64 back-to-back calls without host syncs, and a captured CUDA graph of mixed calls replayed with fresh inputs
    (tests/test_hostar.py:33-54).
Skipped with fewer than 2 GPUs."""
import ctypes
import os
import socket
import traceback

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _parts(n, world, seed, dtype):
    return [(torch.randn(n, generator=torch.Generator().manual_seed(seed * 100 + r)) * 4).to(dtype)
            for r in range(world)]


def _ref_abi_two_ranks(L, rank, dev, check):
    """The reference's two-rank entry points with a real peer (vllm_turing/hostar.py:152-188, cear.py:52-87,
    dmaag.py:60-119 set them up the same way): har_all_reduce over IPC-shared device LL regions (push mode),
    ce_all_reduce over IPC-shared flag + receive buffers, dag_all_gather through a shared host segment."""
    import numpy as np
    import torch.distributed as dist
    from multiprocessing import shared_memory

    from oracle import oracle as O

    s = torch.cuda.current_stream().cuda_stream

    def shared_region(nbytes):
        p, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        assert L.ce_alloc(nbytes, ctypes.byref(p), h) == 0
        hs = [None, None]
        dist.all_gather_object(hs, h.raw)
        qp = ctypes.c_void_p()
        assert L.ce_open(ctypes.create_string_buffer(hs[1 - rank], 64), ctypes.byref(qp)) == 0
        return p.value, qp.value

    # har: LL words pushed into the peer's region, the peer's polled in the own one
    slot_words = 65536   # data words per slot: the largest message below is 24 x 5120 values = 61440 words
    local, remote = shared_region(2 * slot_words * 8)
    counters = torch.zeros(L.har_blocks(slot_words), dtype=torch.int32, device=dev)
    # a message beyond the slot is refused before any launch (host_ar.cu:115-117 returns -1 the same way)
    check(L.har_all_reduce(None, None, slot_words + 1, 1, remote, local, counters.data_ptr(), slot_words, s) == -1,
          "har_all_reduce accepted a message larger than its slot")
    for i, n in enumerate((5 * 5120, 24 * 5120, 2 * 777, 5 * 5120)):
        xs = [(torch.randn(n, generator=torch.Generator().manual_seed(60 + 2 * i + r)) * 3).to(torch.bfloat16)
              for r in range(2)]
        out = torch.empty(n, dtype=torch.bfloat16, device=dev)
        xd = xs[rank].to(dev)
        check(L.har_all_reduce(xd.data_ptr(), out.data_ptr(), n // 2, 1, remote, local, counters.data_ptr(),
                               slot_words, s) == 0, "har_all_reduce launch")
        torch.cuda.synchronize()
        want = O.all_reduce([O.to_bits(x) for x in xs], 1)
        check(np.array_equal(O.to_bits(out.cpu()), want), f"har_all_reduce n={n}")
    # ce: two-shot over the IPC buffers, host-side call numbers
    cap = 8 << 20
    my, peer = shared_region(256 + 2 * cap)
    for seq, n in enumerate((2048 * 5120 // 4, 16 * 999, 5120 * 64), start=1):
        xs = [(torch.randn(n, generator=torch.Generator().manual_seed(80 + 2 * seq + r)) * 2).half() for r in range(2)]
        out = torch.empty(n, dtype=torch.float16, device=dev)
        xd = xs[rank].to(dev)
        check(L.ce_all_reduce(xd.data_ptr(), out.data_ptr(), n, rank, my, peer, cap, seq, 8, s) == 0, "ce launch")
        torch.cuda.synchronize()
        check(np.array_equal(O.to_bits(out.cpu()), O.all_reduce([O.to_bits(x) for x in xs], 0)),
              f"ce_all_reduce n={n}")
    # dag: per rank [2 parity buffers of CAP bytes][2 x 4096 bytes of flags] in one shared host segment
    CAP, FB, P = 4 << 20, 4096, 8
    region = 2 * CAP + 2 * FB
    name = [None]
    shm = shared_memory.SharedMemory(create=True, size=2 * region) if rank == 0 else None
    if rank == 0:
        name[0] = shm.name
    dist.broadcast_object_list(name, src=0)
    if rank != 0:
        shm = shared_memory.SharedMemory(name=name[0])
    try:
        base = ctypes.addressof(ctypes.c_char.from_buffer(shm.buf))
        if rank == 0:
            ctypes.memset(base, 0, 2 * region)
        dist.barrier()
        dbase = L.dag_register(base, 2 * region)
        check(bool(dbase), "dag_register")
        for seq, m in enumerate((3 << 20, 5 * 1024 + 16, CAP), start=1):
            b = seq & 1
            payload = [torch.randint(0, 256, (m,), generator=torch.Generator().manual_seed(90 + 2 * seq + r),
                                     dtype=torch.uint8) for r in range(2)]
            g = torch.zeros(2 * m, dtype=torch.uint8, device=dev)
            g[rank * m:(rank + 1) * m] = payload[rank].to(dev)
            stage = lambda r: base + r * region + b * CAP   # noqa: E731
            flags = lambda r: dbase + r * region + 2 * CAP + b * FB   # noqa: E731
            check(L.dag_all_gather(g.data_ptr(), m, rank, stage(rank), stage(1 - rank), flags(rank),
                                   flags(1 - rank), seq, P, s, None, None, None, None, None) == 0, "dag launch")
            torch.cuda.synchronize()
            check(torch.equal(g.cpu(), torch.cat(payload)), f"dag_all_gather m={m}")
        dist.barrier()
        L.har_unregister(base)
    finally:
        dist.barrier()
        shm.close()
        if rank == 0:
            shm.unlink()
    check(L.vt_status(1) == 0, "a wait of the two-rank transports timed out")


def _worker(rank, world, port, q):
    import numpy as np
    import torch.distributed as dist
    from datetime import timedelta

    from oracle import oracle as O
    from vllm_turing_b200.comm import TPComm
    from vllm_turing_b200.synthetic import make_layer_inputs

    fails = []
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        comm = TPComm(dist.group.WORLD, dev)

        def check(cond, what):
            if not cond:
                fails.append(f"rank {rank}: {what}")

        # ---- all-reduce ----
        for dtype, code in ((torch.bfloat16, 1), (torch.float16, 0)):
            for i, (n, algo) in enumerate(((5120, 1), (5 * 5120, 1), (24 * 5120, 1), (4100, 1), (5 * 5120, 2),
                                           (1000 * 8, 2), (2048 * 5120, 2), (8192 * 5120, 0))):
                parts = _parts(n, world, 10 + i, dtype)
                y = comm.all_reduce(parts[rank].to(dev), algo=algo)
                torch.cuda.synchronize()
                want = O.all_reduce([O.to_bits(p) for p in parts], code)
                check(np.array_equal(O.to_bits(y.cpu()), want), f"all_reduce n={n} algo={algo} {dtype}")
        # in place
        parts = _parts(5 * 5120, world, 99, torch.bfloat16)
        x = parts[rank].to(dev)
        comm.all_reduce(x, out=x, algo=2)
        torch.cuda.synchronize()
        check(np.array_equal(O.to_bits(x.cpu()), O.all_reduce([O.to_bits(p) for p in parts], 1)), "in-place")

        # ---- all-gather ----
        for m in (5 * 1024, 48 * 1024, 3 * 1024 * 1024 + 16):
            g = torch.zeros(world * m, dtype=torch.uint8, device=dev)
            g[rank * m:(rank + 1) * m] = (rank * 37 + torch.arange(m, device=dev) % 251).to(torch.uint8)
            comm.all_gather(g, m)
            torch.cuda.synchronize()
            for r in range(world):
                exp = (r * 37 + torch.arange(m) % 251).to(torch.uint8)
                check(torch.equal(g[r * m:(r + 1) * m].cpu(), exp), f"all_gather m={m} slot {r}")

        # ---- AR8 (the optional lossy all-reduce): bit-exact to the oracle's rank-ordered sum, same on every rank ----
        for n in (8192 * 5120 // 8, 1024 * 40):
            xs8 = [(torch.randn(n, generator=torch.Generator().manual_seed(900 + r)) * 2).half() for r in range(world)]
            y = comm.all_reduce_ar8(xs8[rank].to(dev))
            torch.cuda.synchronize()
            want = O.ar8_dequant_sum([O.ar8_quant(O.to_bits(x)) for x in xs8])
            check(np.array_equal(O.to_bits(y.cpu()), want), f"ar8 all-reduce n={n}")

        # ---- row-strided all-gather, and the int8 LM head's vocabulary-parallel logits gathered in place ----
        from vllm_turing_b200 import dmaag, lmhead
        for shape in ((5, 24), (3, 2, 40)):
            xs_ = [(torch.randn(*shape, generator=torch.Generator().manual_seed(7 + r)) * 2).to(torch.bfloat16)
                   for r in range(world)]
            got = dmaag.all_gather_dim(comm, xs_[rank].to(dev), -1)
            torch.cuda.synchronize()
            check(got is not None and torch.equal(got.cpu(), torch.cat(xs_, -1)), f"all_gather_dim {shape}")
        Vs, Kh = 151936 // 8, 5120                       # one TP8 rank's share of the vocabulary (config 4's head)
        for M in (1, 5):
            xh = torch.randn(M, Kh, generator=torch.Generator().manual_seed(300 + M)).to(torch.bfloat16)
            heads = []
            for r in range(world):
                gw = torch.Generator().manual_seed(400 + r)
                heads.append((torch.randint(-128, 128, (Vs, Kh), generator=gw, dtype=torch.int8),
                              torch.rand(Vs, generator=gw) * 1e-3))
            logits = lmhead.logits_gathered(xh.to(dev), heads[rank][0].to(dev), heads[rank][1].to(dev), comm=comm)
            torch.cuda.synchronize()
            lb = O.to_bits(logits.cpu())
            for r in range(world):
                if r in (rank, (rank + 1) % world):   # own columns and one peer's: the CPU oracle is slow at this size
                    want, _, mag = O.w8a16(O.to_bits(xh), heads[r][0].numpy(), heads[r][1].numpy(), None, 1,
                                           want_acc=True)
                    err = O.w8a16_close(lb[:, r * Vs:(r + 1) * Vs], want, mag, heads[r][1].numpy(), 1)
                    check(err <= 1.0, f"lm head logits M={M} block {r}: error {err:.2f} of tolerance")
            lbits = logits.cpu().view(torch.int16).to(torch.int32)   # gloo has no 16-bit integer type
            l0 = lbits.clone()
            dist.broadcast(l0, src=0)
            check(torch.equal(l0, lbits), f"lm head logits differ from rank 0 (M={M})")

        # ---- fused row-linear ----
        for (M, N, K) in ((16, 5120, 8704), (5, 5120, 17408 // world), (1, 5120, 17408 // world),
                          (32, 5120, 17408 // world), (24, 5120, 8704)):
            lis = [make_layer_inputs(M, N, K, seed=M, rank=r) for r in range(world)]
            me = lis[rank]
            res = me.residual.to(dev)
            red = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            qd, sd = comm.row_linear(me.a.to(dev), me.w.to(dev), me.sa.to(dev), me.sw.to(dev), residual=res,
                                     norm_w=me.norm_w.to(dev), eps=1e-6, reduced=red)
            torch.cuda.synchronize()
            ro, qo, so, redo = O.row_linear_tp([li.a.numpy() for li in lis], [li.w.numpy() for li in lis],
                                               [li.sa.numpy() for li in lis], [li.sw.numpy() for li in lis],
                                               O.to_bits(me.residual), O.to_bits(me.norm_w), 1e-6, 1)
            check(np.array_equal(O.to_bits(red.cpu()), redo), f"fused reduced M={M} K={K}")
            check(np.array_equal(O.to_bits(res.cpu()), ro), f"fused residual M={M} K={K}")
            d = np.abs(qd.cpu().numpy().astype(np.int32) - qo.astype(np.int32))
            check(d.max() <= 1, f"fused q M={M} K={K} off by {d.max()}")
            # identical on every rank
            q0 = qd.clone().cpu()
            dist.broadcast(q0, src=0)
            check(torch.equal(q0, qd.cpu()), f"fused q differs from rank 0 (M={M})")

        # ---- fused prefill row-linear (M > 32): the GEMM epilogue scatters tiles to their owner ranks, the owners
        # reduce in rank order and every rank pulls the reduced rows and runs the residual + RMSNorm + quant ----
        # both routes of the prefill row-linear: the fused tail and the three-kernel chain (the default route at
        # comm.PREFILL_CHAIN_WORLD ranks or more), against one oracle result per shape
        for (M, N, K) in ((256 * world, 5120, 512), (128 * world, 2048, 1040)):
            lis = [make_layer_inputs(M, N, K, seed=40 + M + N, rank=r) for r in range(world)]
            me = lis[rank]
            a_d, w_d, sa_d, sw_d, nw_d = me.a.to(dev), me.w.to(dev), me.sa.to(dev), me.sw.to(dev), me.norm_w.to(dev)
            ro, qo, so, redo = O.row_linear_tp_big([li.a.numpy() for li in lis], [li.w.numpy() for li in lis],
                                                   [li.sa.numpy() for li in lis], [li.sw.numpy() for li in lis],
                                                   O.to_bits(me.residual), O.to_bits(me.norm_w), 1e-6, 1)
            for route in ("fused", "chain"):
                res = me.residual.to(dev)
                red = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                qd, sd = comm.row_linear(a_d, w_d, sa_d, sw_d, residual=res, norm_w=nw_d, eps=1e-6, reduced=red,
                                         route=route)
                # ten more calls back to back on fresh residual copies: identical results, no host sync between them
                more = []
                for _ in range(10):
                    r2 = me.residual.to(dev)
                    more.append((r2,) + tuple(comm.row_linear(a_d, w_d, sa_d, sw_d, residual=r2, norm_w=nw_d,
                                                              eps=1e-6, route=route)))
                torch.cuda.synchronize()
                check(np.array_equal(O.to_bits(red.cpu()), redo), f"prefill {route} reduced M={M} N={N}")
                check(np.array_equal(O.to_bits(res.cpu()), ro), f"prefill {route} residual M={M} N={N}")
                d = np.abs(qd.cpu().numpy().astype(np.int32) - qo.astype(np.int32))
                check(d.max() <= 1, f"prefill {route} q M={M} off by {d.max()}")
                for i, (r2, q2, s2) in enumerate(more):
                    check(torch.equal(r2, res) and torch.equal(q2, qd) and torch.equal(s2, sd),
                          f"prefill {route} call {i + 1} differs from call 0 (M={M})")
                q0 = qd.clone().cpu()
                dist.broadcast(q0, src=0)
                check(torch.equal(q0, qd.cpu()), f"prefill {route} q differs from rank 0 (M={M})")

        # ---- fused row-linear captured in a CUDA graph (three chained calls), replayed with fresh inputs ----
        M, N, K = 5, 5120, 17408 // world
        ws = [make_layer_inputs(M, N, K, seed=70 + j, rank=rank) for j in range(3)]
        dw = [(w.w.to(dev), w.sw.to(dev)) for w in ws]
        a_in, sa_in = ws[0].a.to(dev), ws[0].sa.to(dev)
        res_g = ws[0].residual.to(dev)
        nw_g = ws[0].norm_w.to(dev)
        qs = [torch.empty(M, N, dtype=torch.int8, device=dev) for _ in range(3)]
        ss = [torch.empty(M, 1, dtype=torch.float32, device=dev) for _ in range(3)]

        def chain():
            for j in range(3):   # each call's int8 output feeds nothing: every call reads the same a, sa
                comm.row_linear(a_in, dw[j][0], sa_in, dw[j][1], residual=res_g, norm_w=nw_g, eps=1e-6,
                                q=qs[j], scales=ss[j])
        chain()
        torch.cuda.synchronize()
        dist.barrier()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            chain()
        allw = [[make_layer_inputs(M, N, K, seed=70 + j, rank=r) for r in range(world)] for j in range(3)]
        for it in range(3):
            lis = [make_layer_inputs(M, N, K, seed=200 + it, rank=r) for r in range(world)]
            a_in.copy_(lis[rank].a.to(dev))
            sa_in.copy_(lis[rank].sa.to(dev))
            res_g.copy_(lis[rank].residual.to(dev))
            r_host = O.to_bits(lis[rank].residual)
            gr.replay()
            torch.cuda.synchronize()
            for j in range(3):
                r_host, qo, so, _ = O.row_linear_tp([li.a.numpy() for li in lis], [x.w.numpy() for x in allw[j]],
                                                    [li.sa.numpy() for li in lis], [x.sw.numpy() for x in allw[j]],
                                                    r_host, O.to_bits(ws[0].norm_w), 1e-6, 1)
                d = np.abs(qs[j].cpu().numpy().astype(np.int32) - qo.astype(np.int32))
                check(d.max() <= 1, f"graph replay {it} fused call {j}: q off by {d.max()}")
            check(np.array_equal(O.to_bits(res_g.cpu()), r_host), f"graph replay {it}: residual")
        del gr

        # ---- stress: back-to-back mixed calls without host syncs ----
        xs = [_parts(n, world, 500 + i, torch.bfloat16) for i, n in enumerate((5120, 15360, 5120, 30720) * 16)]
        ys = [comm.all_reduce(p[rank].to(dev)) for p in xs]
        torch.cuda.synchronize()
        bad = sum(not np.array_equal(O.to_bits(y.cpu()), O.all_reduce([O.to_bits(t) for t in p], 1))
                  for y, p in zip(ys, xs))
        check(bad == 0, f"stress: {bad} of {len(xs)} wrong")

        # ---- CUDA graph of mixed calls, replayed with fresh inputs ----
        sizes = (5120, 15360, 5120, 30720, 2048 * 5120) * 3
        ins = [torch.empty(n, dtype=torch.bfloat16, device=dev) for n in sizes]
        outs = [torch.empty_like(t) for t in ins]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for t, o in zip(ins, outs):
                comm.all_reduce(t, out=o)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for t, o in zip(ins, outs):
                comm.all_reduce(t, out=o)
        for it in range(6):
            parts = [_parts(n, world, 1000 + 31 * it + j, torch.bfloat16) for j, n in enumerate(sizes)]
            for t, p in zip(ins, parts):
                t.copy_(p[rank])
            g.replay()
            torch.cuda.synchronize()
            for j, (o, p) in enumerate(zip(outs, parts)):
                if not np.array_equal(O.to_bits(o.cpu()), O.all_reduce([O.to_bits(x) for x in p], 1)):
                    check(False, f"graph replay {it} call {j}")
                    break
        del g
        st = comm.status(clear=True)
        check(st == 0, f"device status {st:#x}")
        if world == 2:
            _ref_abi_two_ranks(comm.L, rank, dev, check)
        comm.close()
        dist.destroy_process_group()
    except Exception:   # noqa: BLE001
        fails.append(f"rank {rank}: {traceback.format_exc()}")
    q.put((rank, fails))


def _run(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, f = q.get(timeout=600)
            res[r] = f
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    fails = [x for r in sorted(res) for x in res[r]]
    assert len(res) == world, f"only {len(res)} of {world} ranks reported"
    assert not fails, "\n".join(fails)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_ranks(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run(world)

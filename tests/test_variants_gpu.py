"""The kernel variants chosen by environment switches that are read once per process, each checked in a child
process against the oracle (int32 accumulators and the fused layer's reduced sum and residual bit-exact, int8 within
1 LSB):
  - the fused row-linear's dp4a GEMV phase (VLLM_TURING_FUSED_GEMV=1);
  - the tcgen05 decode kernel's K blocks per pipeline stage (VLLM_TURING_TC_KBS = 1 or 2; 4 is the default);
  - the row-CTA epilogue of the fused row-linear instead of the tile owners (VLLM_TURING_DECODE_TAIL=rows), alone and
    with several CTAs per token row and the mailbox combine that tensor parallelism above two ranks uses there
    (VLLM_TURING_ROW_CTAS);
  - launches without programmatic dependent launch (VLLM_TURING_PDL=0), and the weight prefetch into L2 ahead of the
    launch wait (VLLM_TURING_L2_PREFETCH_KB, off by default);
  - the prefill GEMM on 128 x 256 tiles instead of 256 x 256 (VLLM_TURING_PREFILL_WIDE=0), its last round as whole
    256 x 256 tiles instead of 128-row halves (VLLM_TURING_PREFILL_SPLIT=0), and the fused prefill
    tail's reduce-scatter stores staged through shared memory at one rank too (VLLM_TURING_PF_STAGE=2);
  - the prefill row-linear's three-kernel chain (GEMM, all-reduce, norm + quant), the default route from four ranks
    up, taken at one rank (VLLM_TURING_PREFILL_CHAIN_WORLD=1)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def child():
    """Runs in the child process: decode GEMMs through vt_gemm_s32 and the fused layer at world size 1."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from tests.helpers import assert_bits_equal, q_off, rand_int8
    from vllm_turing_b200 import _build
    from vllm_turing_b200.comm import TPComm
    from vllm_turing_b200.synthetic import make_layer_inputs

    L = _build.load()
    s = torch.cuda.current_stream().cuda_stream
    for M, N, K in ((5, 34816, 5120), (16, 5120, 17408), (32, 1000, 5136), (1, 136, 128),   # decode orientation
                    (33, 256, 128), (300, 1000, 5136), (2048, 5120, 2176)):                 # prefill orientation
        a, w = rand_int8((M, K), M + 1), rand_int8((N, K), N + 2)
        ac, wc = a.cuda(), w.cuda()   # kept alive until the kernel has run
        acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
        assert L.vt_gemm_s32(ac.data_ptr(), wc.data_ptr(), acc.data_ptr(), M, N, K, s) == 0
        torch.cuda.synchronize()
        assert np.array_equal(acc.cpu().numpy(), O.gemm_s32(a.numpy(), w.numpy())), (M, N, K)
    assert L.vt_status(1) == 0
    assert L.vt_workspace_nonzero(8 << 20) == 0

    from vllm_turing_b200 import w8a8
    from vllm_turing_b200.tailoverlap import silu_mul_quant
    for M, I, K in ((5, 4352, 5120), (24, 1088, 2176)):   # the fused gate/up + SiLU + quant kernel
        a, w = rand_int8((M, K), 3 * M), rand_int8((2 * I, K), 5 * I)
        ac, wc = a.cuda(), w.cuda()
        sa = (torch.rand(M, 1, generator=torch.Generator().manual_seed(M)) * 2e-2).cuda()
        sw = (torch.rand(2 * I, 1, generator=torch.Generator().manual_seed(I)) * 2e-4).cuda()
        wi, si = w8a8.interleave_gate_up(wc, sw)
        q, sc = w8a8.gate_up_silu_quant(ac, wi, sa, si)
        out = torch.empty(M, 2 * I, dtype=torch.bfloat16, device="cuda")
        w8a8.mma(out, ac, wc.t(), sa, sw, None)
        q0, s0 = silu_mul_quant(out)
        torch.cuda.synchronize()
        assert torch.equal(q, q0) and torch.equal(sc.view(-1), s0.view(-1)), (M, I, K)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=os.environ.get("VT_TEST_PORT", "29631"))
    dist.init_process_group("gloo", rank=0, world_size=1)
    torch.cuda.set_device(0)
    comm = TPComm(dist.group.WORLD, torch.device("cuda", 0))
    for M, N, K in ((5, 5120, 17408), (16, 5120, 8704), (1, 1024, 512)):
        li = make_layer_inputs(M, N, K, seed=M + K, rank=0)
        res = li.residual.cuda()
        red = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        q, sc = comm.row_linear(li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), residual=res,
                                norm_w=li.norm_w.cuda(), eps=li.eps, reduced=red)
        torch.cuda.synchronize()
        comm.check()
        ro, qo, so, redo = O.row_linear_tp([li.a.numpy()], [li.w.numpy()], [li.sa.numpy()], [li.sw.numpy()],
                                           O.to_bits(li.residual), O.to_bits(li.norm_w), li.eps, 1)
        assert_bits_equal(red, redo, f"reduced M={M}")
        assert_bits_equal(res, ro, f"residual M={M}")
        assert q_off(q.cpu().numpy(), qo) <= 1
    for M, N, K in ((384, 5120, 2176),):   # the prefill tail (its GEMM's tiles follow VLLM_TURING_PREFILL_WIDE)
        li = make_layer_inputs(M, N, K, seed=M + K, rank=0)
        res = li.residual.cuda()
        red = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        q, sc = comm.row_linear(li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), residual=res,
                                norm_w=li.norm_w.cuda(), eps=li.eps, reduced=red)
        torch.cuda.synchronize()
        comm.check()
        ro, qo, so, redo = O.row_linear_tp_big([li.a.numpy()], [li.w.numpy()], [li.sa.numpy()], [li.sw.numpy()],
                                               O.to_bits(li.residual), O.to_bits(li.norm_w), li.eps, 1)
        assert_bits_equal(red, redo, f"prefill reduced M={M}")
        assert_bits_equal(res, ro, f"prefill residual M={M}")
        assert q_off(q.cpu().numpy(), qo) <= 1
    comm.close()
    dist.destroy_process_group()
    print("CHILD OK")


@pytest.mark.parametrize("env", [{"VLLM_TURING_FUSED_GEMV": "1"}, {"VLLM_TURING_TC_KBS": "1"},
                                 {"VLLM_TURING_TC_KBS": "2"}, {"VLLM_TURING_DECODE_TAIL": "rows"},
                                 {"VLLM_TURING_DECODE_TAIL": "rows", "VLLM_TURING_ROW_CTAS": "4"},
                                 {"VLLM_TURING_FUSED_GEMV": "1", "VLLM_TURING_ROW_CTAS": "3"},
                                 {"VLLM_TURING_PDL": "0"}, {"VLLM_TURING_L2_PREFETCH_KB": "256"},
                                 {"VLLM_TURING_PREFILL_WIDE": "0"}, {"VLLM_TURING_PF_STAGE": "2"},
                                 {"VLLM_TURING_PF_STAGE": "2", "VLLM_TURING_PREFILL_WIDE": "0"},
                                 {"VLLM_TURING_PREFILL_SPLIT": "0"}, {"VLLM_TURING_PREFILL_CHAIN_WORLD": "1"}],
                         ids=["fused_gemv", "kbs1", "kbs2", "rows_tail", "rows_tail_ctas4", "gemv_row_ctas3", "no_pdl",
                              "l2_prefetch",
                              "prefill_128x256", "pf_staged", "pf_staged_128x256", "prefill_no_split",
                              "prefill_chain"])
def test_variant_in_child(env):
    e = dict(os.environ, **env)
    r = subprocess.run([sys.executable, "-c", "import tests.test_variants_gpu as t; t.child()"], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "CHILD OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])

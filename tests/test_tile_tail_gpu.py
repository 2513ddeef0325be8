"""The fused decode tail's tile owners (csrc/tp_fused.cu) take each token row's absmax in ONE mailbox round: every
128-feature tile publishes, with its sum of squares, the |residual|, |norm weight| pair of its largest product and a
flag when a second product of the tile lies within 2^-19 of it; the normalised values of those candidates give the
exact absmax, and only a flagged candidate (a near-tie) sends the call through a second round.

Child processes run the same inputs with the one-round path (the default) and with every row forced through the
second round (VLLM_TURING_TT_ROUNDS=2): the reduced sum, the residual, q and the scales must be bit-identical between
the two, and match the oracle (reduced and residual bit-exact, int8 within 1 LSB). Inputs: random rows, and rows with
planted exact ties -- two features with the same large residual and the same norm weight, inside one tile (flagged:
the fallback) and in two tiles (two unflagged candidates)."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = {"random": [], "tie_in_tile": [(1, 10, 20)], "tie_across_tiles": [(0, 10, 300), (3, 700, 5000)]}


def _inputs(case):
    from vllm_turing_b200.synthetic import make_layer_inputs
    M, N, K = 5, 5120, 17408
    li = make_layer_inputs(M, N, K, seed=21, rank=0)
    for m, f1, f2 in CASES[case]:
        # h = bf16(reduced + 4096) is 4096 for |reduced| < 16 (bf16 spacing 32 there): equal products |h w| at f1, f2
        li.residual[m, f1] = 4096.0
        li.residual[m, f2] = 4096.0
        li.norm_w[f1] = 1.25
        li.norm_w[f2] = 1.25
    return li


def child(outdir):
    import torch
    import torch.distributed as dist

    from vllm_turing_b200.comm import TPComm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=os.environ.get("VT_TEST_PORT", "29641"))
    dist.init_process_group("gloo", rank=0, world_size=1)
    torch.cuda.set_device(0)
    comm = TPComm(dist.group.WORLD, torch.device("cuda", 0))
    for case in CASES:
        li = _inputs(case)
        res = li.residual.cuda()
        red = torch.empty_like(res)
        q, sc = comm.row_linear(li.a.cuda(), li.w.cuda(), li.sa.cuda(), li.sw.cuda(), residual=res,
                                norm_w=li.norm_w.cuda(), eps=li.eps, reduced=red)
        torch.cuda.synchronize()
        comm.check()
        np.savez(os.path.join(outdir, f"{case}.npz"), q=q.cpu().numpy(), scales=sc.cpu().numpy().reshape(-1),
                 residual=res.cpu().view(torch.int16).numpy(), reduced=red.cpu().view(torch.int16).numpy())
    comm.close()
    dist.destroy_process_group()
    print("CHILD OK")


def _run(outdir, extra_env, port):
    env = dict(os.environ, VT_TEST_PORT=str(port), **extra_env)
    r = subprocess.run([sys.executable, "-c", f"import tests.test_tile_tail_gpu as t; t.child({outdir!r})"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "CHILD OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])


def test_one_round_absmax_equals_two_rounds(tmp_path):
    from oracle import oracle as O
    one, two = tmp_path / "one", tmp_path / "two"
    one.mkdir()
    two.mkdir()
    _run(str(one), {}, 29641)
    _run(str(two), {"VLLM_TURING_TT_ROUNDS": "2"}, 29642)
    for case in CASES:
        a, b = np.load(one / f"{case}.npz"), np.load(two / f"{case}.npz")
        for k in ("q", "scales", "residual", "reduced"):
            assert np.array_equal(a[k], b[k]), f"{case}: {k} differs between one and two mailbox rounds"
        li = _inputs(case)
        ro, qo, so, redo = O.row_linear_tp([li.a.numpy()], [li.w.numpy()], [li.sa.numpy()], [li.sw.numpy()],
                                           O.to_bits(li.residual), O.to_bits(li.norm_w), li.eps, 1)
        assert np.array_equal(a["reduced"].view(np.uint16), redo), case
        assert np.array_equal(a["residual"].view(np.uint16), ro), case
        d = np.abs(a["q"].astype(np.int32) - qo.astype(np.int32))
        assert d.max() <= 1 and (d != 0).mean() < 1e-2, case
        assert np.max(np.abs(a["scales"] - so.reshape(-1)) / so.reshape(-1)) < 1e-2, case
        for m, f1, f2 in CASES[case]:   # the planted ties are the row's absmax: both quantise to +-127
            assert abs(int(a["q"][m, f1])) == 127 and abs(int(a["q"][m, f2])) == 127, (case, m)

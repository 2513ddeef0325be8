"""Host-side protocol of comm.TPComm on CPU ranks (gloo, world size 2 and 4), with a fake of the C library standing in
for the device calls: IPC handles are exchanged so every rank maps every peer in rank order, all ranks agree on
success, a failure on one rank (ce_alloc / ce_open) makes every rank raise instead of hanging, a device-side timeout
reported in the status word surfaces as CommError, a rank that never joins ends the others' set-up with an error
within the group's timeout, and close() unmaps peers before owners free. No GPU is used."""
import ctypes
import os
import socket
import traceback

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class FakeLib:
    """Records calls; region r lives at fake address 0x1000000 * (r + 1)."""

    def __init__(self, rank, fail_alloc=False, fail_open=False, status=0):
        self.rank, self.fail_alloc, self.fail_open, self.status = rank, fail_alloc, fail_open, status
        self.calls = []
        self.created = None

    def vt_tp_preload(self):
        return 0

    def vt_comm_region_bytes(self, world, ll, big, scratch):
        return 4096 * world if 1 <= world <= 8 else 0

    def ce_alloc(self, size, pp, handle):
        self.calls.append("alloc")
        if self.fail_alloc:
            return 1
        pp._obj.value = 0x1000000 * (self.rank + 1)
        ctypes.memmove(handle, f"rank{self.rank}".encode().ljust(64, b"\0"), 64)
        return 0

    def ce_open(self, handle, pp):
        self.calls.append("open")
        if self.fail_open:
            return 1
        r = int(bytes(handle.raw[4:6]).split(b"\0")[0])
        pp._obj.value = 0x1000000 * (r + 1) + 0x10   # mapped peer address (differs from the owner's)
        return 0

    def vt_comm_create(self, rank, world, arr, ll, big, scratch):
        self.created = [arr[i] for i in range(world)]
        return 0xABC

    def vt_comm_status(self, h, clear):
        s, self.status = self.status, (0 if clear else self.status)
        return s

    def vt_comm_destroy(self, h):
        self.calls.append("destroy")
        return 0

    def ce_close(self, p):
        self.calls.append("close")
        return 0

    def ce_free(self, p):
        self.calls.append("free")
        return 0


def _worker(rank, world, port, scenario, q):
    import torch.distributed as dist
    from datetime import timedelta

    from vllm_turing_b200.comm import CommError, TPComm
    out = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        if scenario == "never_joins" and rank == world - 1:
            q.put(out)
            return
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        lib = FakeLib(rank, fail_alloc=(scenario == "alloc_fails" and rank == 1),
                      fail_open=(scenario == "open_fails" and rank == 0),
                      status=(0x02000001 if scenario == "timeout_status" and rank == 0 else 0))
        try:
            c = TPComm(dist.group.WORLD, "cpu", lib=lib)
        except CommError as e:
            out["error"] = str(e)
            q.put(out)
            return
        out["bases"] = lib.created
        try:
            c.check()
            out["check"] = "ok"
        except CommError as e:
            out["check"] = str(e)
        c.close()
        out["calls"] = lib.calls
        dist.destroy_process_group()
    except Exception:   # noqa: BLE001
        out["exc"] = traceback.format_exc()
    q.put(out)


def _run(world, scenario, timeout=60):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        o = q.get(timeout=timeout)
        res[o["rank"]] = o
    for p in ps:
        p.join(timeout=20)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_handles_exchanged_in_rank_order(world):
    res = _run(world, "ok")
    for r in range(world):
        o = res[r]
        assert "exc" not in o, o.get("exc")
        bases = o["bases"]
        assert bases[r] == 0x1000000 * (r + 1)                        # own region: the allocation itself
        for p in range(world):
            if p != r:
                assert bases[p] == 0x1000000 * (p + 1) + 0x10          # peers: mapped through their handles
        assert o["check"] == "ok"
        calls = o["calls"]
        assert calls.index("destroy") < calls.index("free")
        assert all(calls.index("close") < calls.index("free") for _ in [0] if "close" in calls)


@pytest.mark.parametrize("scenario", ["alloc_fails", "open_fails"])
def test_one_rank_failing_fails_all(scenario):
    res = _run(2, scenario)
    for r in range(2):
        assert "exc" not in res[r], res[r].get("exc")
        assert "set-up failed" in res[r].get("error", ""), res[r]


def test_device_timeout_surfaces_as_error():
    res = _run(2, "timeout_status")
    assert "timed out" in res[0]["check"]
    assert res[1]["check"] == "ok"


def test_rank_that_never_joins_ends_setup_with_error():
    """The last rank never joins: the others' process-group set-up fails within the short timeout (no hang)."""
    res = _run(2, "never_joins", timeout=120)
    assert "exc" in res[0] or "error" in res[0]

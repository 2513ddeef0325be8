"""The all-gather primitive (the reference's DmaAllGather API, vllm_turing/dmaag.py:205-267) on NVLink P2P.

The reference gathers two ranks' payloads through pinned host memory with copy engines (no peer access on its
hosts). B200 nodes have NVSwitch, so the same contract -- `gathered` holds world slots of m bytes, the caller has
written this rank's slot on the current stream, the call fills the peers' slots on the current stream -- runs as one
kernel over the communicator (csrc/tp_comm.cu: LL words for small payloads, pushed bulk slices with per-CTA flags for
large ones), for any rank count and inside CUDA graphs. Used for column-parallel outputs and lm-head logits.
VLLM_TURING_DAG=0 disables; VLLM_TURING_DAG_MIN_KB sets the smallest payload taken (default 0).
"""
import logging
import os

import torch

logger = logging.getLogger("vllm.turing")
ENABLED = os.environ.get("VLLM_TURING_DAG", "1") != "0"
MIN_BYTES = int(os.environ.get("VLLM_TURING_DAG_MIN_KB", "0")) << 10


class DmaAllGather:
    """all_gather(gathered, m) over an existing communicator (comm.TPComm) or a new one on `cpu_group`."""

    def __init__(self, cpu_group=None, device=None, comm=None):
        if comm is None:
            from .comm import TPComm
            comm = TPComm(cpu_group, device)
        self.comm = comm
        self.rank, self.world = comm.rank, comm.world

    def usable(self, m):
        return ENABLED and m >= MIN_BYTES and m % 8 == 0

    def all_gather(self, gathered, m):
        """gathered: device uint8 [world * m]; this rank's payload already in slot `rank`."""
        return self.comm.all_gather(gathered, m)

    def all_gather_tensor(self, x):
        """[*, D] tensor -> [world, *, D] gathered copy (convenience for column-parallel outputs / logits)."""
        m = x.numel() * x.element_size()
        g = torch.empty(self.world * m, dtype=torch.uint8, device=x.device)
        g[self.rank * m:(self.rank + 1) * m].copy_(x.contiguous().view(-1).view(torch.uint8))
        self.all_gather(g, m)
        return g.view(x.dtype).view(self.world, *x.shape)


def install():
    """Nothing to patch: the all-gather is created by the layers that use it (as in the reference, dmaag.py:1-7)."""
    return None

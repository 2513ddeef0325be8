"""The all-gather primitive (the reference's DmaAllGather API, vllm_turing/dmaag.py:57-119) on NVLink P2P.

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


def all_gather_dim(comm, x, dim=-1):
    """vLLM's all_gather(input_, dim) contract on the communicator: the ranks' tensors concatenated along `dim`.
    Along the last dimension (vocabulary-parallel logits, column-parallel outputs) the result is written in its final
    layout by the row-strided gather (this rank's columns copied in, the peers' filled over NVLink); along the first
    dimension the slots are contiguous; otherwise, or when the payload exceeds the one-shot capacity, the gather
    runs on contiguous slots and the result is rearranged like vLLM's (movedim). Returns None if not applicable."""
    if not (x.is_contiguous() and x.dim() >= 1 and x.numel() > 0):
        return None
    world, rank = comm.world, comm.rank
    nd = x.dim()
    dim = dim + nd if dim < 0 else dim
    esz = x.element_size()
    m = x.numel() * esz
    if dim == nd - 1 and nd >= 1:
        S = x.shape[-1]
        rows = x.numel() // S
        if (S * esz) % 8 == 0 and m <= comm.ll_capacity:
            out = torch.empty(*x.shape[:-1], world * S, dtype=x.dtype, device=x.device)
            out[..., rank * S:(rank + 1) * S].copy_(x)
            comm.all_gather_rows(out, rows, S * esz, world * S * esz)
            return out
    if m % 16 != 0 and not (m % 8 == 0 and m <= comm.ll_capacity):
        return None
    g = torch.empty(world * m, dtype=torch.uint8, device=x.device)
    g[rank * m:(rank + 1) * m].copy_(x.view(-1).view(torch.uint8))
    comm.all_gather(g, m)
    out = g.view(x.dtype).view(world, *x.shape)
    if dim == 0:
        return out.reshape(world * x.shape[0], *x.shape[1:])
    out = out.movedim(0, dim)
    return out.reshape(*x.shape[:dim], world * x.shape[dim], *x.shape[dim + 1:])


def install():
    """Nothing to install here: vLLM's CudaCommunicator.all_gather / gather are routed to all_gather_dim by the
    communicator patch (hostar.install), and layers may create a DmaAllGather themselves (the reference's
    dmaag.py:1-7 usage)."""
    return None

"""The tensor-parallel all-reduce of vLLM's CudaCommunicator on the B200 P2P kernels (csrc/tp_comm.cu).

The reference hooks CudaCommunicator.__init__ / all_reduce (vllm_turing/hostar.py:191-282) to route two-rank messages
to its LL kernel (<= 128 KiB), its copy-engine all-reduce (>= 8 MiB eager) or its host-memory kernel, else to vLLM's
custom all-reduce / NCCL. On B200 every TP size 2..8 with full NVLink peer access gets one communicator (comm.TPComm)
whose kernels serve every size: one-shot LL up to VLLM_TURING_LL_KB, two-shot reduce-scatter + all-gather above it,
both CUDA-graph capturable (device-resident call counter). Other messages (odd sizes, other dtypes) and failed set-ups
keep vLLM's path. Switches: VLLM_TURING_HAR=0 disables the module; VLLM_TURING_LL=0 disables the one-shot path;
VLLM_TURING_CE_AR=0 disables the two-shot path; VLLM_TURING_AR8=1 sends large fp16 messages through the lossy int8
all-reduce (comm.all_reduce_ar8). all_gather / gather (vocabulary-parallel logits, column-parallel
outputs) go to the communicator's P2P all-gather (dmaag.all_gather_dim; VLLM_TURING_DAG=0 keeps vLLM's).
"""
import logging
import os

import torch

logger = logging.getLogger("vllm.turing")
ENABLED = os.environ.get("VLLM_TURING_HAR", "1") != "0"
LL_ENABLED = os.environ.get("VLLM_TURING_LL", "1") != "0"
CE_ENABLED = os.environ.get("VLLM_TURING_CE_AR", "1") != "0"
# lossy int8 all-reduce for large messages (the reference's VLLM_TURING_AR8=1, hostar.py:40-44; off by default). On
# NVLink it moves fewer bytes than the two-shot only at two ranks: (w - 1) (1 + 1/64) n vs 2 (w - 1) / w * 2n bytes.
AR8 = os.environ.get("VLLM_TURING_AR8", "0") == "1"


def peer_ok(n=None):
    n = torch.cuda.device_count() if n is None else n
    return n > 1 and all(torch.cuda.can_device_access_peer(i, j) for i in range(n) for j in range(n) if i != j)


def choose_algo(comm, t):
    """0: not ours (vLLM's path), 1: one-shot, 2: two-shot, 3: AR8 (lossy, opt-in)."""
    if comm is None or not comm.should_use(t):
        return 0
    nbytes = t.numel() * t.element_size()
    if LL_ENABLED and nbytes <= comm.ll_bytes:
        return 1
    if AR8 and comm.ar8_ok(t):   # above the one-shot size, as the reference (ar8_ok: numel * 2 > SLOT_BYTES)
        return 3
    if CE_ENABLED:
        return 2
    return 0


def install():
    if not ENABLED:
        return
    from vllm.platforms import current_platform
    cap = current_platform.get_device_capability()
    if cap is None or cap.to_int() != 100:
        return
    from vllm.distributed.device_communicators.cuda_communicator import CudaCommunicator
    if getattr(CudaCommunicator, "_vllm_turing_har", False):
        return
    orig_init, orig_ar = CudaCommunicator.__init__, CudaCommunicator.all_reduce

    def __init__(self, *args, **kwargs):
        orig_init(self, *args, **kwargs)
        self.turing_comm = None
        try:
            name = getattr(self, "unique_name", "") or ""
            if (2 <= self.world_size <= 8 and name.startswith("tp") and self.device.type == "cuda"
                    and peer_ok()):
                from .comm import TPComm
                self.turing_comm = TPComm(self.cpu_group, self.device)
                logger.info("vllm_turing_b200: P2P all-reduce for %s (%d ranks; one-shot <= %d KB, two-shot above)",
                            name, self.world_size, self.turing_comm.ll_bytes >> 10)
        except Exception as e:   # noqa: BLE001
            logger.warning("vllm_turing_b200: P2P all-reduce unavailable (%s), vLLM's all-reduce is used", e)
            self.turing_comm = None

    def all_reduce(self, input_):
        comm = getattr(self, "turing_comm", None)
        algo = choose_algo(comm, input_)
        if algo == 3:
            return comm.all_reduce_ar8(input_)
        if algo:
            return comm.all_reduce(input_, algo=algo)
        return orig_ar(self, input_)

    from . import dmaag
    orig_ag, orig_gather = CudaCommunicator.all_gather, CudaCommunicator.gather

    def all_gather(self, input_, dim=-1):
        comm = getattr(self, "turing_comm", None)
        if comm is not None and dmaag.ENABLED and input_.is_cuda and \
                input_.numel() * input_.element_size() >= dmaag.MIN_BYTES:
            out = dmaag.all_gather_dim(comm, input_, dim)
            if out is not None:
                return out
        return orig_ag(self, input_, dim)

    def gather(self, input_, dst=0, dim=-1):
        # every rank takes part in the same all-gather (the communicator's calls are collective); only dst keeps it
        comm = getattr(self, "turing_comm", None)
        if comm is not None and dmaag.ENABLED and input_.is_cuda and \
                input_.numel() * input_.element_size() >= dmaag.MIN_BYTES:
            out = dmaag.all_gather_dim(comm, input_, dim)
            if out is not None:
                return out if self.rank_in_group == dst else None
        return orig_gather(self, input_, dst, dim)

    CudaCommunicator.__init__ = __init__
    CudaCommunicator.all_reduce = all_reduce
    CudaCommunicator.all_gather = all_gather
    CudaCommunicator.gather = gather
    CudaCommunicator._vllm_turing_har = True

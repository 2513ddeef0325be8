"""vLLM's custom all-reduce through its staging buffer inside CUDA graphs (the reference's customar.py:20-39).

Messages that the P2P communicator declines (hostar.choose_algo) still reach vLLM's CustomAllreduce. Inside CUDA
graphs it reads the captured tensors directly and exchanges their legacy IPC handles after capture, which memory from
PyTorch's expandable segments (cuMemMap) does not have. As in the reference, the graph path is switched to vLLM's
copy-into-staging-buffer path (registered=False), whose buffer is a plain cudaMalloc shared at init, so the custom
all-reduce works with expandable segments. VLLM_TURING_CUSTOM_AR_COPY=0 disables.
"""
import logging
import os

import torch

logger = logging.getLogger("vllm.turing")
ENABLED = os.environ.get("VLLM_TURING_CUSTOM_AR_COPY", "1") != "0"


def install():
    if not ENABLED:
        return
    try:
        from vllm.distributed.device_communicators import custom_all_reduce as car
    except ImportError:
        return
    C = car.CustomAllreduce
    if getattr(C, "_vllm_turing_copy", False):
        return

    def custom_all_reduce(self, input):
        if self.disabled or not self.should_custom_ar(input):
            return None
        if self._IS_CAPTURING and not torch.cuda.is_current_stream_capturing():
            return torch.empty_like(input)   # warm-up run inside the capture context: allocation pattern only
        return self.all_reduce(input, registered=False)

    C.custom_all_reduce, C._vllm_turing_copy = custom_all_reduce, True
    logger.info("vllm_turing_b200: vLLM custom all-reduce through its staging buffer in CUDA graphs")

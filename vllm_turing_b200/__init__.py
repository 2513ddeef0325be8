"""B200 (sm_100a) tensor-parallel W8A8 linear for vLLM, loaded as a `vllm.general_plugins` entry point.

The drop-in replacement for vllm-turing's hot path (vllm_turing/__init__.py:38-72 registers it there):
  - w8a8: INT8 W8A8 GEMM behind vLLM's cutlass_scaled_mm -- tcgen05 kind::i8 tensor-core kernels with TMEM
    accumulators (a stream-K decode kernel for M <= 32, 128 x 256 tiles above); the TMA-streamed dp4a GEMV on request;
    the fused gate/up + SiLU*up + quant kernel (gate_up_silu_quant)
  - hostar: the tensor-parallel all-reduce of CudaCommunicator replaced by P2P kernels over NVLink (one-shot LL for
    decode messages, two-shot reduce-scatter + all-gather for prefill)
  - quantfuse: per-token int8 activation quantisation (the formula inductor fuses into the producer)
  - fused: row-parallel linear + all-reduce + residual add + RMSNorm + per-token int8 quantisation in one kernel
  - dmaag: the all-gather primitive (each rank pre-writes its slot, the kernel fills the peers' slots), also behind
    CudaCommunicator.all_gather / gather
  - lmhead: the int8 LM head (W8A16: int8 rows converted to 16-bit in tensor memory, tcgen05 kind::f16) and the
    vocabulary-parallel logits gathered in place
  - customar / tailoverlap: the reference's vLLM-side switches on this path
VLLM_TURING_DISABLE=1 turns everything off. Every module honours the reference's VLLM_TURING_<NAME> switches.
"""
import logging
import os

logger = logging.getLogger("vllm.turing")   # under "vllm": uses vLLM's log handler
_registered = False


def register():
    """vLLM plugin entry point (pyproject: [project.entry-points."vllm.general_plugins"] turing = ...)."""
    global _registered
    if _registered or os.environ.get("VLLM_TURING_DISABLE") == "1":
        return
    _registered = True
    from . import customar, dmaag, hostar, lmhead, quantfuse, tailoverlap, w8a8

    tailoverlap.install()
    quantfuse.install()
    customar.install()
    w8a8.install()
    hostar.install()
    dmaag.install()
    lmhead.install()
    logger.info("vllm_turing_b200: W8A8 GEMV for M <= %d, tensor-core kernels above; P2P all-reduce %s",
                w8a8.MAX_M, "on" if hostar.ENABLED else "off")

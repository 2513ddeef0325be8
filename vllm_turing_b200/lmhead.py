"""INT8 LM head (the reference's vllm_turing/lmhead.py:1-141) on the B200 W8A16 kernel (csrc/w8a16_tc.cu).

After loading, vLLM's ParallelLMHead weight (16-bit) is replaced by int8 rows with an fp32 scale per row (half the
memory); logits come from one tcgen05 kernel for up to 64 rows (the int8 rows are converted to the activations' 16-bit
type in tensor memory and multiplied on the tensor cores with fp32 sums), in 64-row passes up to GEMV_MAX_M rows, and
from the reference's chunked dequantisation above (prompt logprobs, warm-up). With tensor parallelism the vocabulary
shards are gathered along the last dimension by the P2P all-gather (csrc/tp_comm.cu, `vt_all_gather_rows`): each
rank's kernel writes its columns of the [M, V] logits in place, the gather fills the peers' columns.

Switches (the reference's names): VLLM_TURING_LMHEAD=0 disables; VLLM_TURING_LMHEAD_MMA=0 limits a pass to 16 rows
(the reference's GEMV-only mode).
"""
import logging
import os

import torch

from . import _build

logger = logging.getLogger("vllm.turing")
GEMV_MAX_M = 256   # rows through the kernel in passes; more dequantise chunks instead (lmhead.py:106-110)
MMA = os.environ.get("VLLM_TURING_LMHEAD_MMA", "1") != "0"
PASS_M = 64 if MMA else 16
_ws = {}


def lib():
    return _build.load()


def _code(dt):
    if dt == torch.float16:
        return 0
    if dt == torch.bfloat16:
        return 1
    raise TypeError(f"vllm_turing_b200: W8A16 needs fp16 / bf16 activations, got {dt}")


def workspace(device, K):
    """The per-device zeroed workspace of vt_w8a16_mm for up to 64 rows of K (allocated on first use, which must come
    before any graph capture; the kernels leave its split-K slots zeroed)."""
    d = torch.device(device)
    idx = d.index if d.index is not None else torch.cuda.current_device()
    ws = _ws.get((idx, K))
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("vllm_turing_b200: W8A16 workspace must be allocated before graph capture")
        ws = torch.zeros(int(lib().vt_w8a16_ws_bytes(64, K)), dtype=torch.uint8, device=torch.device("cuda", idx))
        _ws[(idx, K)] = ws
    return ws


@torch.no_grad()
def quantize_rows(w: torch.Tensor, chunk: int = 16384):
    """[N, K] float -> int8 [N, K] and fp32 per-row scales [N]: scale = max(amax, 1e-12) / 127, q = round(w / scale)
    clamped to [-128, 127] (the reference's formula, lmhead.py:52-61)."""
    q = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    s = torch.empty(w.shape[0], dtype=torch.float32, device=w.device)
    for i in range(0, w.shape[0], chunk):
        wf = w[i:i + chunk].float()
        sc = wf.abs().amax(dim=1).clamp(min=1e-12) / 127.0
        q[i:i + chunk] = torch.round(wf / sc[:, None]).clamp(-128, 127).to(torch.int8)
        s[i:i + chunk] = sc
    return q, s


def mm_into(out, x, w, s, bias=None, ldo=None):
    """out[:, :N] (row stride ldo, default N) = x . (w * s)^T + bias for M <= 64 rows, one kernel."""
    M, K = x.shape
    N = w.shape[0]
    ldo = N if ldo is None else int(ldo)
    ws = workspace(x.device, K)
    rc = lib().vt_w8a16_mm(x.data_ptr(), w.data_ptr(), s.data_ptr(), bias.data_ptr() if bias is not None else None,
                           out.data_ptr(), M, N, K, ldo, _code(x.dtype), ws.data_ptr(), ws.numel(),
                           torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"vt_w8a16_mm failed: {rc}")
    return out


def kernel_ok(x, w):
    M, K = x.shape
    return (x.is_cuda and x.dtype in (torch.float16, torch.bfloat16) and x.is_contiguous() and w.is_contiguous()
            and w.dtype == torch.int8 and K % 16 == 0 and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0)


_frag = torch.library.Library("vllm_turing", "FRAGMENT")
_frag.define("w8a16_mm(Tensor x, Tensor w, Tensor s, Tensor? bias) -> Tensor")


@torch.library.impl(_frag, "w8a16_mm", "CUDA")
def _w8a16_mm(x, w, s, bias):
    """vllm_turing::w8a16_mm (lmhead.py:83-111): logits [M, N] of x [M, K] against the int8 head."""
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    if 1 <= M <= GEMV_MAX_M and kernel_ok(x, w):
        for r0 in range(0, M, PASS_M):
            r1 = min(M, r0 + PASS_M)
            mm_into(out[r0:r1], x[r0:r1], w, s, bias)
        return out
    if M == 0:
        return out
    c = 4096   # larger M: dequantise 4096 rows of the head at a time (the reference's path, lmhead.py:104-110)
    for j in range(0, N, c):
        wd = (w[j:j + c].float() * s[j:j + c, None]).to(x.dtype)
        out[:, j:j + c] = x @ wd.t()
    if bias is not None:
        out += bias
    return out


@torch.library.register_fake("vllm_turing::w8a16_mm")
def _w8a16_mm_fake(x, w, s, bias):
    return x.new_empty(x.shape[0], w.shape[0])


def shard_logits(x, w, s, bias=None):
    """This rank's logits [M, Vs] through the op (any M)."""
    return torch.ops.vllm_turing.w8a16_mm(x, w, s, bias)


def logits_gathered(x, w, s, bias=None, comm=None, out=None):
    """Vocabulary-parallel logits gathered on every rank: out [M, world * Vs] (Vs = this rank's rows of the head).
    The kernel writes this rank's columns in place (row stride world * Vs); the row-strided P2P all-gather fills
    the others. M <= 64 and M * Vs * 2 bytes within the communicator's one-shot capacity; otherwise the shard is
    computed on its own and gathered through contiguous slots."""
    M, K = x.shape
    Vs = w.shape[0]
    world = comm.world if comm is not None else 1
    rank = comm.rank if comm is not None else 0
    if out is None:
        out = torch.empty(M, world * Vs, dtype=x.dtype, device=x.device)
    elif (tuple(out.shape) != (M, world * Vs) or out.dtype != x.dtype or not out.is_contiguous()
          or out.device != x.device):
        # the kernel and the row-strided gather write through out's pointer with row stride world * Vs
        raise ValueError(f"logits_gathered: out must be a contiguous {x.dtype} [{M}, {world * Vs}] tensor on "
                         f"{x.device}, got {out.dtype} {tuple(out.shape)} contiguous={out.is_contiguous()}")
    esz = x.element_size()
    if M <= 64 and kernel_ok(x, w) and (world == 1 or M * Vs * esz <= comm.ll_capacity) and (Vs * esz) % 8 == 0:
        mm_into(out[:, rank * Vs:], x, w, s, bias, ldo=world * Vs)
        if world > 1:
            comm.all_gather_rows(out, M, Vs * esz, world * Vs * esz)
        return out
    shard = shard_logits(x, w, s, bias)
    if world == 1:
        out.copy_(shard)
        return out
    m = shard.numel() * esz
    g = torch.empty(world * m, dtype=torch.uint8, device=x.device)
    g[rank * m:(rank + 1) * m].copy_(shard.view(-1).view(torch.uint8))
    comm.all_gather(g, m)
    out.copy_(g.view(x.dtype).view(world, M, Vs).permute(1, 0, 2).reshape(M, world * Vs))
    return out


def install():
    """Patch vLLM's unquantized LM head (the reference's install, lmhead.py:118-141) on B200 (capability 10.0)."""
    from vllm.platforms import current_platform
    cap = current_platform.get_device_capability()
    if cap is None or cap.to_int() != 100 or os.environ.get("VLLM_TURING_LMHEAD", "1") == "0":
        return
    from vllm.model_executor.layers import vocab_parallel_embedding as vpe
    Meth = vpe.UnquantizedEmbeddingMethod
    if getattr(Meth, "_vllm_turing_lmhead", False):
        return
    orig_pw, orig_apply = Meth.process_weights_after_loading, Meth.apply

    def process_weights_after_loading(self, layer):
        orig_pw(self, layer)
        if isinstance(layer, vpe.ParallelLMHead) and not hasattr(layer, "turing_w8") and layer.weight.dim() == 2 \
                and layer.weight.is_cuda and layer.weight.shape[1] % 16 == 0:
            w = layer.weight.data
            layer.turing_w8, layer.turing_s = quantize_rows(w)
            K = w.shape[1]
            layer.weight.data = torch.empty(0, K, dtype=w.dtype, device=w.device)   # free the 16-bit head
            del w
            torch.cuda.empty_cache()
            logger.info("vllm_turing_b200: int8 LM head, %d x %d per rank", layer.turing_w8.shape[0], K)

    def apply(self, layer, x, bias=None):
        if hasattr(layer, "turing_w8"):
            shp = x.shape
            y = torch.ops.vllm_turing.w8a16_mm(x.reshape(-1, shp[-1]).contiguous(), layer.turing_w8, layer.turing_s,
                                               bias)
            return y.view(*shp[:-1], y.shape[-1])
        return orig_apply(self, layer, x, bias)

    Meth.process_weights_after_loading = process_weights_after_loading
    Meth.apply = apply
    Meth._vllm_turing_lmhead = True

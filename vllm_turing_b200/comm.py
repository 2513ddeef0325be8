"""The tensor-parallel P2P communicator: one IPC-shared device region per rank, mapped by every peer.

Set-up follows the reference's DevLLAllReduce / CeAllReduce (vllm_turing/hostar.py:152-175, cear.py:52-71): each rank
allocates a zeroed region with a CUDA IPC handle (ce_alloc), the 64-byte handles are exchanged over a CPU (gloo) group
with all_gather_object, every rank opens its peers' handles (ce_open) and the ranks agree on success before use. The
collectives (csrc/tp_comm.cu) and the fused row-linear (csrc/tp_fused.cu) then load and store peers' regions directly
over NVLink; all ranks must issue the same calls in the same order (cear.py:79), stream-ordered on each rank.

Sizes (the reference's switches where they exist): VLLM_TURING_LL_KB one-shot / fused message limit (default 512 KiB),
VLLM_TURING_CE_AR_MB two-shot bytes per launch (default 64 MiB; larger messages run in pieces).
"""
import ctypes
import os

import torch
import torch.distributed as dist

from . import _build

LL_BYTES = int(os.environ.get("VLLM_TURING_LL_KB", "512")) << 10
BIG_BYTES = int(float(os.environ.get("VLLM_TURING_CE_AR_MB", "64")) * (1 << 20))
# Prefill row-linear (M > 32) at this many ranks or more runs as the three-kernel chain (this rank's GEMM, the two-shot
# all-reduce in place, the residual + RMSNorm + quant kernel) instead of the fused prefill tail. Measured on B200 at
# M = 8192, N = 5120, K = 17408 / TP: at 2 ranks the fused tail takes 447 us against ~537 us for the chain; at 4 ranks
# the chain's kernels take 479 us (184 + 240 + 55) against the fused tail's 518 us.
PREFILL_CHAIN_WORLD = int(os.environ.get("VLLM_TURING_PREFILL_CHAIN_WORLD", "4"))


class CommError(RuntimeError):
    pass


def _code(dt):
    if dt == torch.float16:
        return 0
    if dt == torch.bfloat16:
        return 1
    raise TypeError(f"vllm_turing_b200: unsupported dtype {dt}")


class TPComm:
    """group: a CPU (gloo) process group of the tensor-parallel ranks (one process per GPU); device: this rank's GPU.
    `lib` may be injected (tests use a host-only fake to exercise the set-up protocol without a GPU)."""

    def __init__(self, group, device, ll_bytes=LL_BYTES, big_bytes=BIG_BYTES, scratch_ints=None, lib=None):
        self.L = lib if lib is not None else _build.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device)
        self.ll_bytes, self.big_bytes = int(ll_bytes), int(big_bytes)
        # split-K scratch of the fused row-linear: the GEMV's int32 [M, N] partials, or the tcgen05 kernel's slots
        # (SMs x 128 x ceil(M / 2) x 16 bytes: 4.9 MB at M = 32 on 148 SMs)
        self.scratch_ints = int(scratch_ints if scratch_ints is not None else max(self.ll_bytes // 2, 2 << 20))
        self.handle = None
        self._opened = []
        self._local = None
        L = self.L
        with torch.cuda.device(self.device) if self.device.type == "cuda" else _nullctx():
            if L.vt_tp_preload() != 0:
                raise CommError("vllm_turing_b200: kernel preload failed")
            size = L.vt_comm_region_bytes(self.world, self.ll_bytes, self.big_bytes, self.scratch_ints)
            if not size:
                raise CommError(f"vllm_turing_b200: unsupported world size {self.world}")
            self.region_bytes = size
            p, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            rc = L.ce_alloc(size, ctypes.byref(p), h)
            ok = rc == 0
            self._local = p.value if ok else None
            handles = [None] * self.world
            dist.all_gather_object(handles, h.raw if ok else None, group=group)
            bases = [None] * self.world
            bases[self.rank] = self._local
            for r in range(self.world):
                if r == self.rank or not ok:
                    continue
                if handles[r] is None:
                    ok = False
                    continue
                q = ctypes.c_void_p()
                if L.ce_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(q)) != 0:
                    ok = False
                    continue
                bases[r] = q.value
                self._opened.append(q.value)
            oks = [None] * self.world
            dist.all_gather_object(oks, ok, group=group)
            if not all(oks):
                self._release()
                raise CommError(f"vllm_turing_b200: communicator set-up failed on ranks "
                                f"{[r for r, o in enumerate(oks) if not o]} (ce_alloc rc={rc})")
            arr = (ctypes.c_void_p * self.world)(*bases)
            self.handle = L.vt_comm_create(self.rank, self.world, arr, self.ll_bytes, self.big_bytes,
                                           self.scratch_ints)
            if not self.handle:
                self._release()
                raise CommError("vllm_turing_b200: vt_comm_create failed")
        dist.barrier(group=group)

    # ---- bookkeeping -------------------------------------------------------------------------------------------------
    def _release(self):
        for q in self._opened:
            self.L.ce_close(q)
        self._opened = []
        if self._local:
            self.L.ce_free(self._local)
            self._local = None

    def close(self):
        """Collective: every rank closes (peers' mappings must go before the owners free their regions)."""
        if self.handle is None:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.L.vt_comm_destroy(self.handle)
        self.handle = None
        for q in self._opened:
            self.L.ce_close(q)
        self._opened = []
        dist.barrier(group=self.group)
        if self._local:
            self.L.ce_free(self._local)
            self._local = None

    def status(self, clear=False):
        """0, or the first device-side timeout code on this rank (synchronises)."""
        return int(self.L.vt_comm_status(self.handle, int(clear)))

    def check(self):
        st = self.status(clear=True)
        if st:
            raise CommError(f"vllm_turing_b200: collective timed out on rank {self.rank} (status {st:#010x}); "
                            "a peer did not make the same call in time")

    def seq(self):
        return int(self.L.vt_comm_seq(self.handle))

    @property
    def ll_capacity(self):
        return int(self.L.vt_comm_ll_bytes(self.handle))

    # ---- collectives -------------------------------------------------------------------------------------------------
    def should_use(self, t):
        n = t.numel()
        return (t.is_cuda and t.dtype in (torch.float16, torch.bfloat16) and t.is_contiguous() and n > 0
                and n % 8 == 0 and t.data_ptr() % 16 == 0)

    def all_reduce(self, t, out=None, algo=0):
        """Sum over ranks (float32 in rank order, one rounding) -> out (new tensor if None); in-place allowed."""
        if out is None:
            out = torch.empty_like(t)
        rc = self.L.vt_all_reduce(self.handle, t.data_ptr(), out.data_ptr(), t.numel(), _code(t.dtype), int(algo),
                                  torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise CommError(f"vt_all_reduce failed: {rc}")
        return out

    def all_gather(self, gathered, m):
        """gathered: uint8 [world * m] with this rank's payload in slot `rank` already; fills the peers' slots."""
        if not gathered.is_cuda:
            raise CommError("vllm_turing_b200: all_gather needs a device buffer")
        rc = self.L.vt_all_gather(self.handle, gathered.data_ptr(), int(m), torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise CommError(f"vt_all_gather failed: {rc}")
        return gathered

    def ar8_ok(self, t):
        """AR8 applies to fp16 messages of n % 1024 == 0 elements (each packed block n + n / 64 bytes, a multiple of
        16, so the gather takes whole 16-byte words)."""
        return t.is_cuda and t.dtype == torch.float16 and t.is_contiguous() and t.numel() % 1024 == 0 and \
            t.data_ptr() % 16 == 0

    def all_reduce_ar8(self, t, out=None):
        """The reference's optional lossy all-reduce (AR8, vllm_turing/hostar.py:40-96, csrc/host_ar.cu:133-201) for
        any rank count: int8 + an fp16 scale per 128 values, all-gathered over the P2P kernels, every rank summing the
        dequantised blocks of all ranks in rank order (identical results on every rank). The packed blocks live in a
        persistent per-communicator buffer, grown outside graph capture only."""
        n = t.numel()
        m = n + n // 64
        need = self.world * m
        buf = getattr(self, "_ar8_buf", None)
        if buf is None or buf.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise CommError("vllm_turing_b200: AR8 scratch must grow before graph capture")
            buf = self._ar8_buf = torch.empty(need, dtype=torch.uint8, device=t.device)
        if out is None:
            out = torch.empty_like(t)
        st = torch.cuda.current_stream().cuda_stream
        rc = self.L.ar8_quant(t.data_ptr(), buf.data_ptr() + self.rank * m, n, st)
        if rc != 0:
            raise CommError(f"ar8_quant failed: {rc}")
        self.all_gather(buf, m)
        rc = self.L.vt_ar8_dequant_sum(buf.data_ptr(), out.data_ptr(), n, self.world, st)
        if rc != 0:
            raise CommError(f"vt_ar8_dequant_sum failed: {rc}")
        return out

    def all_gather_rows(self, gathered, rows, row_bytes, ld_bytes):
        """gathered: [rows, ld_bytes] device buffer holding world column blocks of row_bytes per row, this rank's
        block pre-written; fills the peers' blocks (one-shot LL; rows * row_bytes within ll_capacity)."""
        if not gathered.is_cuda:
            raise CommError("vllm_turing_b200: all_gather_rows needs a device buffer")
        rc = self.L.vt_all_gather_rows(self.handle, gathered.data_ptr(), int(rows), int(row_bytes), int(ld_bytes),
                                       torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise CommError(f"vt_all_gather_rows failed: {rc}")
        return gathered

    def row_linear(self, a, w, sa, sw, residual=None, norm_w=None, eps=1e-6, q=None, scales=None, reduced=None,
                   route="auto"):
        """The fused row-parallel tail. With residual: residual += all_reduce(a.w^T * sa * sw) in place and returns
        (q, scales) of RMSNorm(residual) * norm_w; without: returns the all-reduced [M, N] (reduced).
        route, for prefill (M > 32): "auto" takes the three-kernel chain at PREFILL_CHAIN_WORLD ranks or more and the
        fused prefill tail below; "fused" / "chain" force one (the chain needs the prefill GEMM's shapes, else the
        fused tail runs)."""
        M, K = a.shape
        N = w.shape[0]
        dt = residual.dtype if residual is not None else (reduced.dtype if reduced is not None else torch.bfloat16)
        if residual is not None:
            q = q if q is not None else torch.empty(M, N, dtype=torch.int8, device=a.device)
            scales = scales if scales is not None else torch.empty(M, 1, dtype=torch.float32, device=a.device)
        elif reduced is None:
            reduced = torch.empty(M, N, dtype=dt, device=a.device)
        if route not in ("auto", "fused", "chain"):
            raise ValueError(f"row_linear: unknown route {route!r}")
        if M > 32 and (route == "chain" or (route == "auto" and self.world >= PREFILL_CHAIN_WORLD)):
            from . import w8a8
            part = reduced if reduced is not None else torch.empty(M, N, dtype=dt, device=a.device)
            if w8a8.big_ok(part, a, w.t(), sa, sw, None):
                return self._row_linear_chain(part, a, w, sa, sw, residual, norm_w, eps, q, scales)
        rc = self.L.vt_tp_row_linear(self.handle, a.data_ptr(), w.data_ptr(), sa.data_ptr(), sw.data_ptr(),
                                     residual.data_ptr() if residual is not None else None,
                                     norm_w.data_ptr() if norm_w is not None else None, float(eps),
                                     q.data_ptr() if q is not None else None,
                                     scales.data_ptr() if scales is not None else None,
                                     reduced.data_ptr() if reduced is not None else None, M, N, K, _code(dt),
                                     torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise CommError(f"vt_tp_row_linear failed: {rc}")
        return (q, scales) if residual is not None else reduced

    def _row_linear_chain(self, part, a, w, sa, sw, residual, norm_w, eps, q, scales):
        """The prefill row-linear as three launches: the int8 GEMM into part (bf16 / fp16 partial of this rank's K
        slice), the all-reduce of part in place (float32 sum in rank order, one rounding: the fused tail's reduced
        values), then residual += part and the RMSNorm + per-token int8 quant."""
        from . import w8a8
        from .quantfuse import rms_norm_dynamic_per_token_quant
        w8a8.big(part, a, w.t(), sa, sw)
        self.all_reduce(part, out=part)
        if residual is None:
            return part
        rms_norm_dynamic_per_token_quant(part, norm_w, eps, residual, q=q, s=scales)
        return q, scales


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False

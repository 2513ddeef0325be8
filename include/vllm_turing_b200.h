/*
 * vllm_turing_b200.h -- C ABI of libvllm_turing_b200.so, the B200 (sm_100a) tensor-parallel W8A8 linear hot path.
 *
 * Plain pointers and sizes only (no torch types), loaded with ctypes by the Python package exactly as the reference
 * loads its csrc/ libraries (vllm_turing/_build.py:33-55). Every entry returns 0 on success, a negative VT_E* code on
 * rejected arguments, or a positive cudaError_t of the launch, unless stated otherwise. Every launch goes on `stream`
 * (a cudaStream_t; NULL = legacy default stream). Pointers are device pointers unless stated otherwise.
 *
 * dtype: 0 = float16, 1 = bfloat16 (the reference's code, vllm_turing/csrc/w8a8_gemv.cu:346).
 * Matrices are row-major: activations a [M, K] int8, weights w [N, K] int8 (vLLM hands the GEMM the transposed [K, N]
 * view of this tensor, stride (1, K); vllm_turing/csrc/w8a8_gemv.cu:5), outputs [M, N].
 */
#ifndef VLLM_TURING_B200_H
#define VLLM_TURING_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VT_EARG (-1)     /* unsupported shape, alignment or argument */
#define VT_ECAPTURE (-2) /* a library workspace would have to grow while the stream is capturing */
#define VT_ENOMEM (-3)   /* workspace allocation failed */

/* ---- W8A8 GEMM: out = (a . w^T) * sa[m] * sw[n] (+ bias[n]), int32 accumulation -------------------------------- */

/* Decode GEMV, M 1..16, K % 16 == 0, a / w 16-byte aligned; sa_rows / sw_rows = 0 for per-tensor scales.
 * Replaces vllm_turing/csrc/w8a8_gemv.cu:347-361 (same signature and return convention). */
int w8a8_gemv(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M, int N,
              int K, int sa_rows, int sw_rows, int dtype, void *stream);

/* w8a8_gemv with a caller-owned workspace of w8a8_gemv_ws_bytes(M, N) bytes, zeroed before first use (kernels leave
 * it zeroed; calls sharing it must be stream-ordered). No counterpart in the reference (its GEMV needs no scratch). */
size_t w8a8_gemv_ws_bytes(int M, int N);
int w8a8_gemv_ws(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M,
                 int N, int K, int sa_rows, int sw_rows, int dtype, void *workspace, size_t ws_bytes, void *stream);

/* w8a8_gemv for callers that cannot allocate device memory when they run it (inside a memory profiler or a custom
 * allocator, or after handing all device memory to a pool): same arguments and results, but the split-K scratch is a
 * fixed array compiled into the library (about 1 MiB per GPU that loads it, held until exit), so the call allocates
 * nothing. Limits: M * N <= 262144 and N <= 262144, else VT_EARG. The first call on a device resolves the array's
 * address and, with lazy module loading (CUDA_MODULE_LOADING=LAZY, the default), may load the library's module and
 * with it the array: make it before any stream capture and before the window in which nothing may be allocated.
 * Calls sharing a device must not overlap on the GPU (they share the array). A device-side timeout inside the call
 * is reported through vt_noalloc_status, not through the return code. No counterpart in the reference (its GEMV
 * needs no scratch). */
int w8a8_gemv_noalloc(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out,
                      int M, int N, int K, int sa_rows, int sw_rows, int dtype, void *stream);
/* Status word of w8a8_gemv_noalloc on the current device: 0, or the first timeout code its kernels reported (see
 * vt_status for the codes); clear != 0 resets it. Synchronises the device; allocates nothing. New entry. */
unsigned vt_noalloc_status(int clear);

/* int32 accumulators acc[M, N] = a . w^T (bit-exact parity checks), M 1..16. New entry. */
int vt_gemv_s32(const void *a, const void *w, void *acc, int M, int N, int K, void *stream);

/* Small-M tensor-core GEMM, M 1..32 (the default decode path): tcgen05 kind::i8 with the weights as the MMA's A
 * operand and stream-K over the SMs; split-K scratch from the library's per-device workspace (grown outside stream
 * capture only). Replaces vllm_turing/csrc/w8a8_gemv.cu:330-344 (w8a8_mma: same signature and return convention). */
int w8a8_mma(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M, int N,
             int K, int sa_rows, int sw_rows, int dtype, void *stream);
/* w8a8_mma with a caller-owned workspace of w8a8_mma_ws_bytes(M, N) bytes (256-byte aligned, zeroed before first
 * use; the kernel leaves it zeroed; calls sharing it must be stream-ordered). No counterpart in the reference (its
 * MMA kernel needs no scratch). */
size_t w8a8_mma_ws_bytes(int M, int N);
int w8a8_mma_ws(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M,
                int N, int K, int sa_rows, int sw_rows, int dtype, void *workspace, size_t ws_bytes, void *stream);

/* w8a8_mma_ws with the weight in the tile-blocked layout [N / 128][K / 128][128][128] int8 (each 128 x 128 block of
 * the row-major weight contiguous, a tile's blocks in K order; made once at load time): every TMA box the decode
 * stream reads is one contiguous 16 KB block. N % 128 == 0, K % 128 == 0. Same results as w8a8_mma_ws. No
 * counterpart in the reference (its GEMV reads the row-major weight). */
int w8a8_mma_blocked_ws(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out,
                        int M, int N, int K, int sa_rows, int sw_rows, int dtype, void *workspace, size_t ws_bytes,
                        void *stream);

/* Prefill GEMM (tcgen05 kind::i8, 128 x 256 tiles): A [M, K], W [N, K] int8, sa [M], sw [N] float32, out [M, N],
 * dequant order sa[m] * (sw[n] * acc). Returns 0 ok, 1 cannot implement (shape / alignment), 3 launch failed.
 * Replaces vllm_turing/csrc/w8a8_big.cu:66-73 (w8a8_big: same signature and return convention). */
int w8a8_big(const void *A, const void *W, const void *sa, const void *sw, void *out, int M, int N, int K, int dtype,
             void *stream);

/* int32 accumulators acc[M, N] = a . w^T on the tensor cores, any M (decode orientation for M <= 32). New entry. */
int vt_gemm_s32(const void *a, const void *w, void *acc, int M, int N, int K, void *stream);

/* The decode MLP's first half in one kernel: q [M, I] int8 and scales [M] float32 = per-token int8 quantisation of
 * SiLU(gate) * up, [gate | up] the W8A8 linear a [M, K] . w^T with w [2I, K] int8 and sw [2I] float32 in the
 * interleaved row order (128-row tile t = gate rows 64t..64t+63, then up rows 64t..64t+63; made once at load time),
 * sa [M] (sa_rows = 1) or [1]. Bit-identical to w8a8_mma / scaled_mm_ with the plain weight followed by
 * silu_mul_quant. 1 <= M <= 32, I % 64 == 0, K % 16 == 0; a 256-byte aligned workspace of
 * vt_gate_up_silu_quant_ws_bytes(M, I) bytes, zeroed once before first use; calls sharing it must be stream-ordered.
 * dtype (0 fp16 / 1 bf16): the type of the gate / up / product values. Replaces the pair scaled_mm_ (w8a8.py:108-117)
 * + silu_mul_quant (silu_quant.cu:71-77, tailoverlap.py:148-151). */
size_t vt_gate_up_silu_quant_ws_bytes(int M, int I);
int vt_gate_up_silu_quant(const void *a, const void *w, const void *sa, const void *sw, void *q, void *scales, int M,
                          int I, int K, int sa_rows, int dtype, void *workspace, size_t ws_bytes, void *stream);

/* ---- LM head: W8A16 (int8 weight rows + fp32 row scales, 16-bit activations) ------------------------------------ */

/* out [M, N] = x [M, K] . (w [N, K] int8 * s [N])^T + bias [N], fp32 sums, one rounding to dtype (0 fp16 / 1 bf16).
 * tcgen05 kind::f16 with the weights converted to 16-bit in tensor memory, stream-K over the SMs. M 1..16, K % 16 == 0,
 * x and w 16-byte aligned; -1 on bad arguments, else a cudaError. Replaces w8a16_gemv (w8a16_gemv.cu:114-123). */
int w8a16_gemv(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K,
               int dtype, void *stream);
/* rows (int32 [N] indices into w, or NULL): the output covers those weight rows only (CUDA-core kernel; the caller
 * guarantees the indices are in range). Replaces w8a16_gemv_rows (w8a16_gemv.cu:125-145). */
int w8a16_gemv_rows(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K,
                    int dtype, const void *rows, void *stream);
/* fp16 activations, M 1..64, N even; cfg (the reference's tiling choice) is ignored. Same kernel as w8a16_gemv.
 * Replaces w8a16_mma (w8a16_mma.cu:160-175). */
int w8a16_mma(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K, int cfg,
              void *stream);
/* The same for M 1..64 in either dtype, output row stride ldo >= N (write one rank's columns of a [M, world * N]
 * logits buffer), caller-owned workspace of vt_w8a16_ws_bytes(M, K) bytes (256-byte aligned, zeroed once; the kernel
 * leaves it zeroed; calls sharing it must be stream-ordered). New entries. */
size_t vt_w8a16_ws_bytes(int M, int K);
int vt_w8a16_mm(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K, int ldo,
                int dtype, void *workspace, size_t ws_bytes, void *stream);

/* Non-zero 32-bit words in the first `bytes` of the current device's library workspace scratch (kernels leave it
 * zeroed; a test hook). Synchronises the device; -1 on error. New entry. */
long long vt_workspace_nonzero(long long bytes);

/* Status word of the library workspace of the current device: 0, or the first device-side timeout code
 * (0x01xxxxxx pipeline, 0x02xxxxxx peer, 0x03xxxxxx cooperating CTA). Synchronises the device. */
unsigned vt_status(int clear);

/* ---- row-wise epilogues --------------------------------------------------------------------------------------- */

/* Per-token dynamic symmetric int8 quantisation x [M, N] -> q [M, N], scales [M] (float32).
 * Replaces vLLM's scaled_int8_quant as the reference patches it (vllm_turing/quantfuse.py:18-39). */
int vt_scaled_int8_quant(const void *x, void *q, void *scales, int M, int N, int dtype, void *stream);

/* residual := x + residual; q, scales := quant(RMSNorm(residual) * weight); normed (optional) := RMSNorm(...) * w.
 * Replaces vLLM's rms_norm_dynamic_per_token_quant(h, w1, eps, int8, None, res) as called at
 * vllm_turing/tailoverlap.py:200-201. N % 4 == 0, N <= 49152. */
int vt_rms_norm_quant(const void *x, void *residual, const void *weight, float eps, void *q, void *scales,
                      void *normed, int M, int N, int dtype, void *stream);

/* SiLU(gate) * up + per-token int8 quantisation, gate_up (M, 2I) fp16 -> q (M, I), scales (M).
 * Replaces vllm_turing/csrc/silu_quant.cu:71-77 (same signature; returns 1 bad args, 2 launch error). */
int silu_mul_quant(const void *gu, void *q, void *scales, int M, int I, void *stream);
/* The same for fp16 (dtype 0) or bf16 (dtype 1). New entry. */
int vt_silu_mul_quant(const void *gu, void *q, void *scales, int M, int I, int dtype, void *stream);

/* ---- IPC helpers (replace vllm_turing/csrc/ce_ar.cu:77-101, same names and semantics) ------------------------ */

/* A zeroed device buffer of `bytes` and its 64-byte CUDA IPC handle (written to host memory `handle64`).
 * 0 ok; 1 cudaMalloc, 2 memset, 3 sync, 4 handle failed. (ce_ar.cu:79-86) */
int ce_alloc(size_t bytes, void **ptr, void *handle64);
/* Maps a peer's buffer from its 64-byte handle. 0 ok, 1 failed. (ce_ar.cu:88-92) */
int ce_open(const void *handle64, void **ptr);
/* Unmaps a buffer opened with ce_open / frees one from ce_alloc. 0 ok, 1 failed. New entries. */
int ce_close(void *ptr);
int ce_free(void *ptr);
/* Single-process use: peer access from the current device to `peer`. 0 ok, 1 failed. (ce_ar.cu:95-99) */
int ce_enable_peer(int peer);

/* ---- the reference's two-rank transports, same names / signatures / return codes, B200 kernels ----------------
 * Waits are bounded (VLLM_TURING_AR_TIMEOUT_MS); a wait that runs out reports into vt_status. */

/* Loads the kernels below and creates the library workspace (call once per device, before any capture). 0 ok.
 * Replaces vllm_turing/csrc/host_ar.cu:86-92. */
int har_preload(void);
/* Blocks of the LL all-reduce for nwords data words: the number of zeroed int32 call counters the caller keeps.
 * Replaces vllm_turing/csrc/host_ar.cu:94-96 (the block size differs; callers size their counters with it). */
int har_blocks(int nwords);
/* cudaHostRegister (mapped, portable) of a host range; its device pointer or NULL. Replaces host_ar.cu:99-108. */
void *har_register(void *ptr, size_t size);
/* cudaHostUnregister; returns the cudaError. Replaces host_ar.cu:110-112. */
int har_unregister(void *ptr);
/* Two-rank LL all-reduce: out[nwords 32-bit words] = in + the peer's in (dtype 0 fp16 / 1 bf16, float32 sum rounded
 * once). my_ll: where this rank's LL words go (the peer's region, or a mapped host segment); peer_ll: where the peer's
 * arrive; each 2 * slot_words 8-byte words (two parity slots of {data word, call number}); counters: har_blocks(
 * slot_words) zeroed ints of this rank. -1 if nwords > slot_words, else the launch's cudaError. CUDA-graph capturable.
 * Replaces host_ar.cu:115-131. */
int har_all_reduce(const void *in, void *out, int nwords, int dtype, void *my_ll, const void *peer_ll, void *counters,
                   int slot_words, void *stream);
/* 0: ce_all_reduce can run (it needs no driver entry points here). Replaces vllm_turing/csrc/ce_ar.cu:101. */
int ce_driver_ok(void);
/* Two-rank fp16 all-reduce over IPC-shared buffers my / peer (256 bytes of flags, then R1 and R2 of cap bytes, from
 * ce_alloc / ce_open): out[n] = x + the peer's x, n % 16 == 0, 16-byte aligned; seq = 1, 2, ... in the same order on
 * both ranks; blocks is accepted and unused. One SM kernel (two-shot over NVLink stores, a flag pair per slice).
 * Returns 0, 2 bad arguments, 3 cap too small, 7 launch failed. Replaces ce_ar.cu:103-146 (copy engines and stream
 * waits there). */
int ce_all_reduce(const void *x, void *out, long n, int rank, void *my, void *peer, long cap, unsigned seq, int blocks,
                  void *stream);
/* cudaHostRegister of the staging segment; the device pointer of its start or NULL. Replaces vllm_turing/csrc/dma_ag.cu:26-41. */
void *dag_register(void *host, size_t bytes);
/* Two-rank all-gather through registered host staging: gathered (2 m bytes, this rank's half pre-written on main_);
 * my_stage / peer_stage host pointers of m bytes; my_flag_dev / peer_flag_dev device pointers of P int32 piece flags;
 * seq the call number (flags compared with >=). One kernel on main_; d2h_, h2d_ and the events are accepted and
 * unused. 0 ok, 1 failure. Replaces dma_ag.cu:41-74. */
int dag_all_gather(void *gathered, long long m, int rank, void *my_stage, const void *peer_stage, int *my_flag_dev,
                   const int *peer_flag_dev, int seq, int P, void *main_, void *d2h_, void *h2d_, void *ev0, void *ev1,
                   void *ev2);

/* ---- tensor-parallel communicator (N = 1..8 ranks, one process per GPU, NVLink P2P) ---------------------------
 * Replaces the reference's two-rank transports (DevLLAllReduce over har_all_reduce, vllm_turing/hostar.py:152-188 /
 * host_ar.cu:114-131; CeAllReduce over ce_all_reduce, cear.py:52-87 / ce_ar.cu:103-146; DmaAllGather over
 * dag_all_gather, dmaag.py:107-119 / dma_ag.cu:45-74). All ranks must make the same calls in the same order; calls
 * on one communicator must be stream-ordered on each rank. Call counting is device-resident (CUDA-graph safe). */

/* Bounds of the device-side waits of launches made from now on, in milliseconds (<= 0 keeps a bound): pipe_ms for
 * waits inside one CTA, peer_ms for waits on other CTAs or GPUs; initially VLLM_TURING_PIPE_TIMEOUT_MS (2000) and
 * VLLM_TURING_AR_TIMEOUT_MS (10000). A wait that runs out records its code in the status word and the kernel returns.
 * Returns 0. New entry. */
int vt_set_wait_bounds(double pipe_ms, double peer_ms);

/* Bytes of the per-rank region: ll_data = largest one-shot / fused message (bytes), big_data = largest two-shot
 * message per launch (bytes; larger ones run in pieces), scratch_ints = split-K scratch of the fused row-linear in
 * int32 words (>= M * N for the GEMV phase, >= SMs * 128 * ceil(M / 2) * 4 for the tcgen05 phase). */
size_t vt_comm_region_bytes(int world, size_t ll_data, size_t big_data, size_t scratch_ints);
/* bases[world]: each rank's region (own from ce_alloc, peers' from ce_open), same sizes. NULL on bad arguments. */
void *vt_comm_create(int rank, int world, void *const *bases, size_t ll_data, size_t big_data, size_t scratch_ints);
int vt_comm_destroy(void *comm);
long long vt_comm_ll_bytes(void *comm);
long long vt_comm_big_bytes(void *comm);
/* 0 or the first timeout code a collective reported on this rank; synchronises the device. */
unsigned vt_comm_status(void *comm, int clear);
/* Number of completed calls on this communicator (device counter); synchronises the device. */
unsigned vt_comm_seq(void *comm);

/* AR8, the optional lossy all-reduce (VLLM_TURING_AR8=1): x fp16 [n] -> packed [n int8 | n / 128 fp16 scales], one
 * scale per 128 values (amax / 127 rounded to fp16), q = clamp(rint(x / scale), -127, 127); n % 128 == 0, x 16-byte and
 * packed 8-byte aligned. Replaces ar8_quant (host_ar.cu:182-188). */
int ar8_quant(const void *x, void *packed, int n, void *stream);
/* out fp16 [n] = the rank-ordered float32 sum of the dequantised packed blocks of two ranks (gathered = 2 blocks of
 * n + n / 64 bytes); n % 128 == 0 as there (vectorised when n % 512 == 0). Replaces ar8_dequant_sum
 * (host_ar.cu:190-201). */
int ar8_dequant_sum(const void *gathered, void *out, int n, void *stream);
/* The same for 1..8 ranks. New entry. */
int vt_ar8_dequant_sum(const void *gathered, void *out, long long n, int world, void *stream);

/* out[n] = sum over ranks of in[n], float32 accumulation in rank order, one rounding (the arithmetic of
 * host_ar.cu:90-101). algo 0 auto, 1 one-shot LL (n % 4 == 0, up to ll_data), 2 two-shot (n % 8 == 0).
 * in may equal out; 16-byte aligned. One rank: no kernel (a device-to-device copy when in != out). Replaces
 * har_all_reduce (host_ar.cu:114-131) and ce_all_reduce (ce_ar.cu:103-146) for any rank count. */
int vt_all_reduce(void *comm, const void *in, void *out, long long n, int dtype, int algo, void *stream);

/* NVLink bandwidth probe: copies `bytes` (% 16 == 0, at most the two-shot chunk capacity) from this rank's region to
 * rank `peer`'s region, by SM stores (engine 0; ctas CTAs, 0 = 4 per SM) or the copy engines (engine 1). Not a
 * collective and not ordered with the communicator's calls: bracket it with barriers. New entry (measurement only). */
int vt_comm_peer_copy(void *comm, int peer, long long bytes, int engine, int ctas, void *stream);

/* gathered [world * m bytes] with this rank's payload pre-written at [rank * m, (rank + 1) * m); fills the peers'
 * slots. m % 8 == 0 (LL) or m % 16 == 0 (bulk). Replaces dag_all_gather (dma_ag.cu:45-74) for N ranks over P2P. */
int vt_all_gather(void *comm, void *gathered, long long m, void *stream);
/* gathered [rows, ld_bytes]: world column blocks of row_bytes per row, this rank's block (offset rank * row_bytes)
 * pre-written; fills the peers' blocks (vLLM's all_gather along the last dimension, e.g. vocabulary-parallel logits,
 * with no transpose). row_bytes, ld_bytes % 8 == 0, rows * row_bytes within the communicator's one-shot LL capacity
 * (vt_comm_ll_bytes). New entry. */
int vt_all_gather_rows(void *comm, void *gathered, long long rows, long long row_bytes, long long ld_bytes,
                       void *stream);

/* The fused row-parallel layer tail, one kernel: this rank's W8A8 GEMM partial (tcgen05; the dp4a GEMV for M <= 16
 * with VLLM_TURING_FUSED_GEMV=1) -> all-reduce over the communicator -> residual add (in place) -> RMSNorm * norm_w
 * -> per-token int8 q / scales. residual = NULL: plain row-linear + all-reduce into `reduced`. 1 <= M <= 32,
 * N % 4 == 0, K % 16 == 0, M * N * 2 <= ll_data, M * N <= scratch_ints. Replaces the reference's
 * decode tail: scaled_mm_ (w8a8.py:108-117) -> tensor_model_parallel_all_reduce (hostar.py:260-278) ->
 * rms_norm_dynamic_per_token_quant (tailoverlap.py:200). */
int vt_tp_row_linear(void *comm, const void *a, const void *w, const void *sa, const void *sw, void *residual,
                     const void *norm_w, float eps, void *q, void *scales, void *reduced, int M, int N, int K,
                     int dtype, void *stream);
/* The fused row-parallel layer tail for prefill shapes (vt_tp_row_linear forwards M > 32 here): the tcgen05 GEMM's
 * epilogue writes each finished 128 x 256 tile into the receive buffer of the rank that owns its rows (rank o owns rows
 * [o M / world, (o + 1) M / world)) and flags it; a second kernel sums each owned row over the ranks in rank order,
 * publishes it, pulls the peers' reduced rows over NVLink and runs residual add + RMSNorm + int8 quant on every row.
 * Same arguments and results as vt_tp_row_linear (partials dequantised in the prefill GEMM's order sa[m] * (sw[n] *
 * acc)); M % (128 * world) == 0, N % 8 == 0 with N / 8 / v a multiple of 32 in [64, 256] for some v <= 8,
 * K % 16 == 0, residual / norm_w / reduced 16-byte and q 8-byte aligned; rows beyond the communicator's two-shot
 * buffers run as several calls. Replaces the reference's prefill tail: scaled_mm_ (w8a8.py:108-117, w8a8_big) ->
 * all-reduce (cear.py:75-87) -> rms_norm_dynamic_per_token_quant (tailoverlap.py:200), chunk-overlapped across two
 * streams in the reference (tailoverlap.py:165-204). */
int vt_tp_row_linear_prefill(void *comm, const void *a, const void *w, const void *sa, const void *sw,
                             void *residual, const void *norm_w, float eps, void *q, void *scales, void *reduced,
                             int M, int N, int K, int dtype, void *stream);
/* Loads the fused kernels now (a lazily loaded module may synchronise behind a kernel spinning on a peer). */
int vt_tp_preload(void);
int vt_tp_prefill_preload(void);

#ifdef __cplusplus
}
#endif

#endif /* VLLM_TURING_B200_H */

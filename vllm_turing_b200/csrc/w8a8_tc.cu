// W8A8 INT8 GEMM on the 5th-generation tensor cores of B200 (sm_100a): tcgen05.mma kind::i8, int32 accumulators in
// tensor memory (TMEM), operands staged by TMA (the core is tc_core.cuh).
//
//   D[rows, cols] = A[rows, K] . B[cols, K]^T   (both K-major int8), then out = dequant(D) in bf16 / fp16.
//
//   prefill (w8a8_big):  A = activations, B = weights (256-row tiles of N); 256 x 256 tiles per CTA, two 128-row A
//                        halves sharing the B tile (tc_phase_wide; 128 x 256 tiles with VLLM_TURING_PREFILL_WIDE=0);
//                        MMA 128 x 256 x 32.
//                        Dequant order of the reference's CUTLASS epilogue, sa[m] * (sw[n] * acc)
//                        (vllm_turing/csrc/w8a8_big.cu:26-35).
//   decode (w8a8_mma):   A = weights (128-row tiles of N), B = activations (16 or 32 token rows); MMA 128 x 16|32 x 32
//                        ("swap AB", so a few tokens do not pad a 128-row tile), stream-K over the SMs so every SM
//                        streams the same share of the weights (the HBM-bound regime); dequant
//                        (acc * sa[m]) * sw[n] + b (vllm_turing/csrc/w8a8_gemv.cu:288).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "host_util.h"
#include "tc_core.cuh"
#include "tma_host.h"

namespace vt {

template <typename T, int BN, bool SWAP, int KBS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   TcArgs P) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    TcOutEpi<T, BN> fin{};
    tc_phase<T, BN, SWAP, KBS>(&tmap_a, &tmap_b, P, smem_raw, fin);
}

template <typename T, int BN, bool SWAP, int KBS>
static int launch_tc(const CUtensorMap &ma, const CUtensorMap &mb, TcArgs P, cudaStream_t s) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    const int stages = tc_stages<BN, KBS>(dev, 64, SWAP ? decode_smem_budget() : 0);
    if (stages < 2) return VT_EARG;
    P.stages = stages;
    const int smem = tc_smem_bytes<BN, KBS>(stages);
    static bool attr[VT_MAX_DEV] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(tc_gemm_kernel<T, BN, SWAP, KBS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    int g = num_sms(dev);
    if (g > P.units) g = P.units;
    return launch_k(tc_gemm_kernel<T, BN, SWAP, KBS>, dim3(g), dim3(TC_THREADS), smem, s, true, ma, mb, P);
}

// Prefill GEMM on 256 x 256 tiles (tc_phase_wide): two 128-row A halves share each 256-row B tile.
template <typename T>
__global__ void __launch_bounds__(TCW_THREADS, 1)
    tc_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        TcArgs P) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    TcOutEpi<T, TCW_BN> fin{};
    tc_phase_wide<T>(&tmap_a, &tmap_b, P, smem_raw, fin);
}

template <typename T>
static int launch_tc_wide(const CUtensorMap &ma, const CUtensorMap &mb, TcArgs P, cudaStream_t s) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    const int stages = tc_wide_stages(dev);
    if (stages < 2) return VT_EARG;
    P.stages = stages;
    const int smem = tc_wide_smem_bytes(stages);
    static bool attr[VT_MAX_DEV] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(tc_gemm_wide_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    const int g = tc_wide_grid(num_sms(dev), P);
    return launch_k(tc_gemm_wide_kernel<T>, dim3(g), dim3(TCW_THREADS), smem, s, true, ma, mb, P);
}

// Prefill orientation: a [M, K] activations, w [N, K] weights, whole tiles per CTA: 256 x 256 (default) or 128 x 256
// (VLLM_TURING_PREFILL_WIDE=0).
template <typename T>
static int big_gemm(const void *a, const void *w, const float *sa, const float *sw, void *out, int M, int N, int K,
                    int s32, unsigned *status, cudaStream_t s) {
    CUtensorMap ma, mb;
    if (!tc_make_map(&ma, a, M, K, TC_BM) || !tc_make_map(&mb, w, N, K, 256)) return VT_EARG;
    const bool wide = prefill_wide();
    TcArgs P{};
    P.n_tiles_a = wide ? (M + 2 * TC_BM - 1) / (2 * TC_BM) : (M + TC_BM - 1) / TC_BM;
    P.n_tiles_b = (N + 255) / 256;
    P.nkb = (K + TC_BK - 1) / TC_BK;
    P.units = P.n_tiles_a * P.n_tiles_b;
    P.stream_k = 0;
    // a group's A tiles + all of B stay in L2 across a wave (2048 activation rows per group either way)
    const int gm = wide ? 8 : 16;
    P.group_m = P.n_tiles_a < gm ? P.n_tiles_a : gm;
    P.split_tail = wide ? prefill_split_tail() : 0;
    P.sa = sa;
    P.sw = sw;
    P.sa_rows = 1;
    P.sw_rows = 1;
    P.out = out;
    P.M = M;
    P.N = N;
    P.s32_out = s32;
    P.timeout_ns = pipe_timeout_ns();
    P.status = status;
    if (wide) return launch_tc_wide<T>(ma, mb, P, s);
    return launch_tc<T, 256, false, 1>(ma, mb, P, s);
}

template <typename T, int BN>
static int small_kbs(const CUtensorMap &ma, const CUtensorMap &mb, const TcArgs &P, cudaStream_t s) {
    switch (decode_kbs()) {
        case 1: return launch_tc<T, BN, true, 1>(ma, mb, P, s);
        case 2: return launch_tc<T, BN, true, 2>(ma, mb, P, s);
        default: return launch_tc<T, BN, true, 4>(ma, mb, P, s);
    }
}

// Decode orientation: weights as operand A, M <= 32 token rows as operand B, stream-K over the SMs. scratch holds
// decode_ws(M) zeroed bytes (the split-K slots); the kernel leaves them zeroed.
template <typename T>
static int small_gemm(const void *a, const void *w, const float *sa, const float *sw, const void *bias, void *out,
                      int M, int N, int K, int sa_rows, int sw_rows, int s32, void *scratch, unsigned *status,
                      cudaStream_t s, bool blocked = false) {
    const int BN = M <= 16 ? 16 : 32;
    CUtensorMap ma, mb;
    if (blocked) {   // [N / 128][K / 128][128][128]: rows of 128 bytes, one 16 KB box per block
        if ((N % TC_BM) || (K % TC_BK) || !tc_make_map(&ma, w, (N / TC_BM) * (K / TC_BK) * TC_BM, TC_BK, TC_BM))
            return VT_EARG;
    } else if (!tc_make_map(&ma, w, N, K, TC_BM)) {
        return VT_EARG;
    }
    if (!tc_make_map(&mb, a, M, K, BN)) return VT_EARG;
    TcArgs P{};
    tc_decode_args(P, M, N, K);
    P.blocked_a = blocked ? 1 : 0;
    P.sa = sa;
    P.sw = sw;
    P.bias = bias;
    P.sa_rows = sa_rows;
    P.sw_rows = sw_rows;
    P.out = out;
    P.slots = (uint4 *)scratch;
    P.s32_out = s32;
    P.timeout_ns = pipe_timeout_ns();
    P.status = status;
    if (BN == 16) return small_kbs<T, 16>(ma, mb, P, s);
    return small_kbs<T, 32>(ma, mb, P, s);
}

// split-K slot bytes for M token rows on this device (the grid is at most one CTA per SM)
static size_t decode_ws(int M) { return tc_decode_slot_bytes(M, num_sms(cur_device())); }

static bool tc_args_ok(const void *a, const void *w, int M, int N, int K) {
    return M >= 1 && N >= 1 && K >= 16 && (K & 15) == 0 && ((uintptr_t)a & 15) == 0 && ((uintptr_t)w & 15) == 0;
}

template <typename T>
static int mma_dequant(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out,
                       int M, int N, int K, int sa_rows, int sw_rows, void *scratch, unsigned *status,
                       cudaStream_t s, bool blocked = false) {
    return small_gemm<T>(a, w, (const float *)sa, (const float *)sw, bias, out, M, N, K, sa_rows, sw_rows, 0, scratch,
                         status, s, blocked);
}

}  // namespace vt

using namespace vt;

extern "C" {

// The reference's small-M tensor-core entry (vllm_turing/csrc/w8a8_gemv.cu:330-344: M 1..32, same signature and
// return convention): here tcgen05 kind::i8 with the weights as the MMA's A operand, stream-K across the SMs. The
// split-K scratch comes from the library's per-device workspace (grown outside stream capture only).
int w8a8_mma(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M, int N,
             int K, int sa_rows, int sw_rows, int dtype, void *stream) {
    if (!tc_args_ok(a, w, M, N, K) || M > 32) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    if (int rc = ws_acquire(decode_ws(M), s, &scratch, &status)) return rc;
    if (dtype == 0)
        return mma_dequant<__half>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
    return mma_dequant<__nv_bfloat16>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
}

// Bytes of zeroed workspace w8a8_mma_ws needs for these shapes (256-byte status header included).
size_t w8a8_mma_ws_bytes(int M, int N) { return (void)N, 256 + decode_ws(M); }

// w8a8_mma with a caller-owned workspace of w8a8_mma_ws_bytes(M, N) bytes, zeroed once before its first use (the
// kernel leaves it zeroed); calls sharing a workspace must be stream-ordered. The first 256 bytes hold the status word.
int w8a8_mma_ws(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M,
                int N, int K, int sa_rows, int sw_rows, int dtype, void *workspace, size_t ws_bytes, void *stream) {
    if (!tc_args_ok(a, w, M, N, K) || M > 32 || !workspace || ws_bytes < w8a8_mma_ws_bytes(M, N) ||
        ((uintptr_t)workspace & 255))
        return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned *status = (unsigned *)workspace;
    void *scratch = (char *)workspace + 256;
    if (dtype == 0)
        return mma_dequant<__half>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
    return mma_dequant<__nv_bfloat16>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
}

// w8a8_mma_ws with the weight in the tile-blocked layout [N / 128][K / 128][128][128] (int8; every 128 x 128 block of
// the row-major weight stored contiguously, blocks of a 128-row tile in K order): each TMA box of the stream is one
// contiguous 16 KB block. N % 128 == 0, K % 128 == 0. Same results as w8a8_mma_ws on the row-major weight.
int w8a8_mma_blocked_ws(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out,
                        int M, int N, int K, int sa_rows, int sw_rows, int dtype, void *workspace, size_t ws_bytes,
                        void *stream) {
    if (!tc_args_ok(a, w, M, N, K) || M > 32 || (N % 128) || (K % 128) || !workspace ||
        ws_bytes < w8a8_mma_ws_bytes(M, N) || ((uintptr_t)workspace & 255))
        return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned *status = (unsigned *)workspace;
    void *scratch = (char *)workspace + 256;
    if (dtype == 0)
        return mma_dequant<__half>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s, true);
    return mma_dequant<__nv_bfloat16>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s, true);
}

// The reference's prefill entry (vllm_turing/csrc/w8a8_big.cu:66-73: A [M, K], W [N, K] int8, sa [M], sw [N]
// float32, out [M, N]; dtype 0 fp16 / 1 bf16): returns 0 ok, 1 cannot implement (shape / alignment / no driver
// tensor-map entry), 3 launch failed.
int w8a8_big(const void *A, const void *W, const void *sa, const void *sw, void *out, int M, int N, int K, int dtype,
             void *stream) {
    if (!tc_args_ok(A, W, M, N, K) || (N & 15)) return 1;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    if (ws_acquire(0, s, &scratch, &status)) return 1;
    int rc = dtype == 0 ? big_gemm<__half>(A, W, (const float *)sa, (const float *)sw, out, M, N, K, 0, status, s)
                        : big_gemm<__nv_bfloat16>(A, W, (const float *)sa, (const float *)sw, out, M, N, K, 0, status,
                                                  s);
    if (rc == VT_EARG) return 1;
    return rc ? 3 : 0;
}

// int32 accumulators acc[M, N] = a . w^T on the tensor cores (any M; bit-exact parity checks): the decode orientation
// for M <= 32, the prefill orientation above.
int vt_gemm_s32(const void *a, const void *w, void *acc, int M, int N, int K, void *stream) {
    if (!tc_args_ok(a, w, M, N, K)) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    if (M <= 32) {
        if (int rc = ws_acquire(decode_ws(M), s, &scratch, &status)) return rc;
        return small_gemm<__nv_bfloat16>(a, w, nullptr, nullptr, nullptr, acc, M, N, K, 1, 1, 1, scratch, status, s);
    }
    if (int rc = ws_acquire(0, s, &scratch, &status)) return rc;
    return big_gemm<__nv_bfloat16>(a, w, nullptr, nullptr, acc, M, N, K, 1, status, s);
}

}  // extern "C"

// The decode MLP's first half in one kernel on B200 (sm_100a): the column-parallel gate/up W8A8 GEMM, SiLU(gate) * up
// and the per-token int8 quantisation of the product -- what the reference runs as scaled_mm_ (w8a8.py:108-117, the
// GEMV / MMA kernels) followed by silu_mul_quant (csrc/silu_quant.cu:1-77, tailoverlap.py:148-151), here without the
// [M, 2I] bf16 round trip through HBM and without the second launch.
//
//   gate[m, j] = bf16((acc_g * sa[m]) * sw_g[j]),  up[m, j] = bf16((acc_u * sa[m]) * sw_u[j])   (the GEMM epilogue)
//   p[m, j]    = bf16(bf16(gate / (1 + exp(-gate))) * up)                                      (silu_quant.cu:11-14, 39)
//   q[m, j]    = quant(p[m, :]) per token row, scales[m] = absmax / 127                        (quantfuse.py:18-24)
//
// The weight is used in an interleaved row order, made once when the weights are loaded: 128-row tile t holds the
// gate rows of features 64t .. 64t+63 followed by the up rows of the same features (vllm_turing_b200.w8a8
// .interleave_gate_up). The GEMM is the tcgen05 decode core (tc_core.cuh) with a finisher that, per finished tile, has
// the up half of its epilogue threads hand their bf16 values to the gate half through shared memory; the gate half
// forms p, parks it in a bf16 scratch and keeps a running max |p| per token row. Then each CTA publishes its row
// maxima as 8-byte words tagged with the call's epoch (value and tag in one store, after a fence for its products)
// and leaves, freeing its SM for the next kernel in the stream: under programmatic dependent launch the down
// projection's CTAs take those SMs and start streaming weights while the slowest tiles here finish. Sixteen CTAs
// stay: they read every CTA's words -- a bounded wait; the grid is one CTA per SM, all resident -- take the maximum
// (order-independent) and quantise an even share of p. CTA 0 advances the epoch once it has seen every CTA's word
// (every CTA has read the old epoch by then), so an earlier call's words are never taken for this call's. Only the
// split-K slots must be zero between calls, and the GEMM leaves them so.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "host_util.h"
#include "tc_core.cuh"
#include "tma_host.h"

namespace vt {

constexpr int SILU_MAX_M = 32;

// Workspace of one call: [status 256 B][split-K slots (zero between calls)][sync 256 B][max words][p: bf16 M x I].
// The max words are tagged with the call's epoch, so nothing but the slots needs to return to zero.
struct SiluSync {
    unsigned epoch;   // calls completed on this workspace (advanced by CTA 0 once every CTA has read it)
};

template <typename T>
struct SiluArgs {
    SiluSync *sync;
    unsigned long long *words;   // [grid][M] {float bits of this CTA's max |p| of row m, epoch + 1}
    T *p;                        // [M, I] scratch: written by the tile's finisher, read back by the same thread
    int8_t *q;                   // [M, I]
    float *scales;               // [M]
    int I;
};

// Tile finisher: thread = tile row `row` (0..63 gate of feature 64 ta + row, 64..127 up of feature 64 ta + row - 64).
// Keeps, per gate thread, the running max |p| of each token row over the tiles it finished (lmax).
template <typename T, int BN>
struct TcSiluEpi {
    static constexpr int kSmemFloats = 64 + 64 * BN;   // token scales, then the up values [BN][64]
    struct Prep {
        float swn;
    };
    SiluArgs<T> S;
    float *sa_sm, *ubuf;
    unsigned *s_tag;   // shared: this call's tag (epoch + 1), read after pdl_wait, before the GEMM's tail
    float lmax[BN];
    __device__ __forceinline__ void on_start(const TcArgs &P, float *sm) {
        sa_sm = sm;
        ubuf = sm + 64;
        const int t = threadIdx.x - TC_EPI_LEAD;
        if (t < P.M) sm[t] = P.sa[P.sa_rows ? t : 0];
        if (t == 0) *s_tag = *reinterpret_cast<volatile unsigned *>(&S.sync->epoch) + 1u;
#pragma unroll
        for (int m = 0; m < BN; ++m) lmax[m] = 0.0f;
    }
    __device__ __forceinline__ void post_start() {}
    __device__ __forceinline__ Prep prep(const TcArgs &P, int n) const { return Prep{n < P.N ? P.sw[n] : 0.0f}; }
    __device__ __forceinline__ void operator()(const TcArgs &P, int n, bool nok, const int (&acc)[BN],
                                               const Prep &pr) {
        const int row = n & (TC_BM - 1), M = P.M;
        if (row >= 64) {   // up half: bf16 values to the gate half
#pragma unroll
            for (int m = 0; m < BN; ++m)
                if (m < M) ubuf[m * 64 + row - 64] = nok ? rnd<T>(dequant1(acc[m], sa_sm[m], pr.swn)) : 0.0f;
        }
        named_sync(TC_EPI_BAR, 128);
        if (row < 64 && nok) {
            const int j = (n >> 7) * 64 + row;   // feature index in [0, I)
#pragma unroll
            for (int m = 0; m < BN; ++m) {
                if (m >= M) break;
                const float g = rnd<T>(dequant1(acc[m], sa_sm[m], pr.swn));
                const float sg = rnd<T>(__fdiv_rn(g, 1.0f + expf(-g)));
                const float p = rnd<T>(__fmul_rn(sg, ubuf[m * 64 + row]));
                S.p[(size_t)m * S.I + j] = f2t<T>(p);
                lmax[m] = fmaxf(lmax[m], fabsf(p));
            }
        }
        named_sync(TC_EPI_BAR, 128);   // the up values are read: the next tile may overwrite them
    }
};

constexpr int SILU_QUANT_CTAS = 16;   // CTAs that stay for the quantisation; the rest leave their SMs at once

template <typename T, int BN, int KBS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gate_up_silu_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                        TcArgs P, SiluArgs<T> S) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ float s_part[2][SILU_MAX_M];   // the two gate warps' maxima
    __shared__ unsigned s_gmax[SILU_MAX_M];   // the grid's maxima (float bits)
    __shared__ float s_inv[SILU_MAX_M];
    __shared__ unsigned s_tag;
    TcSiluEpi<T, BN> fin{S, nullptr, nullptr, &s_tag, {}};
    tc_phase<T, BN, true, KBS>(&tmap_w, &tmap_a, P, smem_raw, fin);   // ends with __syncthreads

    const int M = P.M, I = S.I, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // 1. this CTA's max |p| per token row, published as one tagged word each after its products are visible
    if (threadIdx.x < SILU_MAX_M) s_gmax[threadIdx.x] = 0u;
    if (warp >= 4) {   // epilogue warps 4, 5 hold tile rows 0..63 (the gate half)
#pragma unroll
        for (int m = 0; m < BN; ++m) {
            if (m >= M) break;
            float a = fin.lmax[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            if (lane == 0) s_part[warp - 4][m] = a;
        }
    }
    __syncthreads();
    const unsigned tag = s_tag;
    if (threadIdx.x < M) {
        const float a = fmaxf(s_part[0][threadIdx.x], s_part[1][threadIdx.x]);
        __threadfence();   // this CTA's products (stored before the barrier above) before its word
        st_volatile8(&S.words[(size_t)blockIdx.x * M + threadIdx.x],
                     ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(a));
    }
    // The other CTAs are done: their SMs go to the next kernel in the stream (the down projection's weight stream
    // starts there while the slowest tiles of this one finish).
    const int QC = (int)gridDim.x < SILU_QUANT_CTAS ? (int)gridDim.x : SILU_QUANT_CTAS;
    if ((int)blockIdx.x >= QC) return;
    // 2. every CTA's words: the grid's maxima (every tile is finished once all words carry this call's tag)
    const uint64_t deadline = globaltimer() + P.timeout_ns;
    const int nwords = (int)gridDim.x * M;
    for (int w = threadIdx.x; w < nwords; w += blockDim.x) {
        unsigned long long x = ld_volatile8(&S.words[w]);
        uint32_t it = 0;
        while ((unsigned)(x >> 32) != tag) {
            if ((++it & 63u) == 0 && globaltimer() > deadline) {
                report(P.status, ST_GROUP_TIMEOUT | 0x600000u | (unsigned)w);
                break;
            }
            x = ld_volatile8(&S.words[w]);
        }
        atomicMax(&s_gmax[w % M], (unsigned)(x & 0xffffffffu));   // |p| bits: order-independent
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x < M) {
        const float amax = __uint_as_float(s_gmax[threadIdx.x]);
        s_inv[threadIdx.x] = quant_inv(amax);
        if (blockIdx.x == 0) S.scales[threadIdx.x] = __fdiv_rn(amax, 127.0f);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) S.sync->epoch = tag;   // every CTA has read the old epoch
    __syncthreads();
    // 3. an even share of the [M, I] products per quantising CTA, 8 at a time (I % 64 == 0: never across a row)
    const int groups = M * (I >> 3);
    const int g0 = (int)((long long)groups * blockIdx.x / QC);
    const int g1 = (int)((long long)groups * (blockIdx.x + 1) / QC);
    const uint4 *pv = reinterpret_cast<const uint4 *>(S.p);
    uint2 *qv = reinterpret_cast<uint2 *>(S.q);
    for (int gi = g0 + threadIdx.x; gi < g1; gi += blockDim.x) {
        const float inv = s_inv[gi / (I >> 3)];
        const uint4 u = __ldcg(pv + gi);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        uint32_t b[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<T>(w[e]);
            const uint32_t two = (uint32_t)(uint8_t)quant1(f.x, inv) | ((uint32_t)(uint8_t)quant1(f.y, inv) << 8);
            b[e >> 1] |= two << (16 * (e & 1));
        }
        qv[gi] = make_uint2(b[0], b[1]);
    }
}

}  // namespace vt

namespace vt {

// [status 256][slots][sync 256][max words: SMs x M x 8][p: M x I x 2]
inline size_t silu_slots_bytes(int M) { return tc_decode_slot_bytes(M, num_sms(cur_device())); }
inline size_t silu_words_bytes(int M) { return ((size_t)num_sms(cur_device()) * M * 8 + 255) & ~(size_t)255; }
inline size_t silu_ws_bytes(int M, int I) {
    return 256 + ((silu_slots_bytes(M) + 255) & ~(size_t)255) + 256 + silu_words_bytes(M) +
           (((size_t)M * I * 2 + 255) & ~(size_t)255);
}

template <typename T, int BN, int KBS>
static int launch_silu_gemm(const CUtensorMap &mw, const CUtensorMap &ma, TcArgs P, SiluArgs<T> S, cudaStream_t s) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    constexpr int EF = TcSiluEpi<T, BN>::kSmemFloats;
    const int stages = tc_stages<BN, KBS>(dev, EF, decode_smem_budget());
    if (stages < 2) return VT_EARG;
    P.stages = stages;
    const int smem = tc_smem_bytes<BN, KBS>(stages, EF);
    static bool attr[VT_MAX_DEV] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(gate_up_silu_kernel<T, BN, KBS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    int g = num_sms(dev);
    if (g > P.units) g = P.units;
    return launch_k(gate_up_silu_kernel<T, BN, KBS>, dim3(g), dim3(TC_THREADS), smem, s, true, mw, ma, P, S);
}

template <typename T, int BN>
static int silu_kbs(const CUtensorMap &mw, const CUtensorMap &ma, const TcArgs &P, const SiluArgs<T> &S,
                    cudaStream_t s) {
    switch (decode_kbs()) {
        case 1: return launch_silu_gemm<T, BN, 1>(mw, ma, P, S, s);
        case 2: return launch_silu_gemm<T, BN, 2>(mw, ma, P, S, s);
        default: return launch_silu_gemm<T, BN, 4>(mw, ma, P, S, s);
    }
}

template <typename T>
static int gate_up_silu(const void *a, const void *w, const float *sa, const float *sw, void *q, void *scales, int M,
                        int I, int K, int sa_rows, void *workspace, cudaStream_t s) {
    const int N = 2 * I;
    const int BN = M <= 16 ? 16 : 32;
    CUtensorMap mw, ma;
    if (!tc_make_map(&mw, w, N, K, TC_BM) || !tc_make_map(&ma, a, M, K, BN)) return VT_EARG;
    char *ws = (char *)workspace;
    TcArgs P{};
    tc_decode_args(P, M, N, K);
    P.sa = sa;
    P.sw = sw;
    P.sa_rows = sa_rows;
    P.sw_rows = 1;
    P.status = (unsigned *)ws;
    P.slots = (uint4 *)(ws + 256);
    P.timeout_ns = pipe_timeout_ns();
    SiluArgs<T> S;
    S.sync = (SiluSync *)(ws + 256 + ((silu_slots_bytes(M) + 255) & ~(size_t)255));
    S.words = (unsigned long long *)((char *)S.sync + 256);
    S.p = (T *)((char *)S.words + silu_words_bytes(M));
    S.q = (int8_t *)q;
    S.scales = (float *)scales;
    S.I = I;
    if (BN == 16) return silu_kbs<T, 16>(mw, ma, P, S, s);
    return silu_kbs<T, 32>(mw, ma, P, S, s);
}

}  // namespace vt

using namespace vt;

extern "C" {

// Bytes of workspace vt_gate_up_silu_quant needs (256-byte status header included); zero it once before first use.
size_t vt_gate_up_silu_quant_ws_bytes(int M, int I) { return silu_ws_bytes(M, I); }

// q [M, I] int8, scales [M] float32 = per-token int8 quantisation of SiLU(gate) * up, where [gate | up] = the W8A8
// linear a [M, K] int8 . w^T with w the gate/up weight [2I, K] int8 in the interleaved row order (128-row tile t =
// gate rows 64t..64t+63, then up rows 64t..64t+63), sw [2I] float32 in the same order, sa [M] (sa_rows = 1) or [1]
// float32. Bit-identical to scaled_mm_ with the plain weight followed by silu_mul_quant. 1 <= M <= 32, I % 64 == 0,
// K % 16 == 0, 16-byte aligned a / w / workspace, q 8-byte aligned. dtype (0 fp16 / 1 bf16) is the dtype of the
// intermediate gate / up / product values. The workspace is zeroed once before first use; calls sharing it must be
// stream-ordered.
int vt_gate_up_silu_quant(const void *a, const void *w, const void *sa, const void *sw, void *q, void *scales, int M,
                          int I, int K, int sa_rows, int dtype, void *workspace, size_t ws_bytes, void *stream) {
    if (!a || !w || !sa || !sw || !q || !scales || !workspace || M < 1 || M > SILU_MAX_M || I < 64 || (I & 63) ||
        K < 16 || (K & 15) || ((uintptr_t)a & 15) || ((uintptr_t)w & 15) || ((uintptr_t)workspace & 255) ||
        ((uintptr_t)q & 7) || ws_bytes < silu_ws_bytes(M, I))
        return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == 0)
        return gate_up_silu<__half>(a, w, (const float *)sa, (const float *)sw, q, scales, M, I, K, sa_rows,
                                    workspace, s);
    return gate_up_silu<__nv_bfloat16>(a, w, (const float *)sa, (const float *)sw, q, scales, M, I, K, sa_rows,
                                       workspace, s);
}

}  // extern "C"

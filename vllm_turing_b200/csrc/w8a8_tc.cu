// W8A8 INT8 GEMM on the 5th-generation tensor cores of B200 (sm_100a): tcgen05.mma kind::i8, int32 accumulators in
// tensor memory (TMEM), operands staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast).
//
//   D[rows, cols] = A[rows, K] . B[cols, K]^T   (both K-major int8), then out = dequant(D) in bf16 / fp16.
//
// Two orientations of one kernel template:
//   prefill (w8a8_big):  A = activations (128-row tiles of M), B = weights (256-row tiles of N); MMA 128 x 256 x 32.
//                        Epilogue thread = token row m, columns = output features n. Dequant order of the reference's
//                        CUTLASS epilogue, sa[m] * (sw[n] * acc) (vllm_turing/csrc/w8a8_big.cu:26-35).
//   decode (w8a8_mma):   A = weights (128-row tiles of N), B = activations (16 or 32 token rows); MMA 128 x 16|32 x 32,
//                        "swap AB" so a few tokens do not pad a 128-row tile. K is split across CTAs so all SMs stream
//                        weights (the HBM-bound regime); partial int32 tiles meet in a zeroed scratch by atomicAdd
//                        (exact) and the CTA whose ticket completes a tile dequantises it ((acc * sa[m]) * sw[n] + b,
//                        vllm_turing/csrc/w8a8_gemv.cu:288).
//
// CTA = 6 warps, persistent over its work units: warp 0 issues TMA loads into a ring of shared-memory stages, warp 1
// allocates TMEM and one of its threads issues the MMAs (4 per 128-byte K block) and commits their completion to
// mbarriers, warps 2..5 drain TMEM (tcgen05.ld, 32 lanes each: warp w reads lanes 32 (w % 4) ..) and write the
// outputs. TMEM holds two accumulator buffers so the epilogue of one unit overlaps the MMAs of the next. Every wait is
// bounded (globaltimer); on a timeout the CTA records the status, stops waiting, still frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "host_util.h"
#include "tma_host.h"

namespace vt {

constexpr int TC_THREADS = 192;
constexpr int TC_BK = 128;   // bytes of K per stage (= one 128-byte swizzle row)
constexpr int TC_BM = 128;   // MMA M (rows of operand A per tile)

// ---- tcgen05 / TMA primitives (PTX ISA 8.6, sm_100a) ------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (TMEM) (+)= A (smem desc) . B (smem desc)^T, kind::i8, int32 accumulate
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 TMEM lanes x 32 consecutive 32-bit columns; thread i of the warp receives lane (base lane + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile written by TMA with 128-byte swizzle: rows of 128 bytes,
// 8-row swizzle atoms 1024 bytes apart (stride byte offset), sm100 descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;                      // leading byte offset: unused for swizzled K-major
    d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;                      // descriptor version (sm100)
    d |= (uint64_t)2u << 61;                      // SWIZZLE_128B
    return d;
}
// Instruction descriptor, kind::i8: int32 accumulator, signed A and B, both K-major, MMA M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- the kernel ------------------------------------------------------------------------------------------------------
struct TcArgs {
    int rows_a, rows_b, K;          // A: rows_a x K, B: rows_b x K
    int n_tiles_a, n_tiles_b;       // tiles along A rows (128) and B rows (BN)
    int ksplit;                     // K-block ranges per tile (decode); every range non-empty
    int kb_per;                     // K blocks per range
    int nkb;                        // K blocks of 128 bytes
    int units;                      // n_tiles_a * n_tiles_b * ksplit
    const float *sa, *sw;           // per token, per output feature
    const void *bias;
    int sa_rows, sw_rows;
    void *out;                      // [M, N] row-major
    int M, N;                       // tokens, output features
    int *scratch, *tickets;         // decode split-K: int32 [M, N] zeroed, tickets [n_tiles_a]
    int s32_out;                    // write int32 accumulators instead of dequant
    int stages;
    uint64_t timeout_ns;
    unsigned *status;
};

template <int BN> struct TcLayout {
    static constexpr int A_BYTES = TC_BM * TC_BK;
    static constexpr int B_BYTES = BN * TC_BK;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
};

// SWAP = false: prefill orientation (A = activations); true: decode orientation (A = weights).
template <typename T, int BN, bool SWAP>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   TcArgs P) {
    using Lay = TcLayout<BN>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int S = P.stages;
    unsigned char *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * Lay::STAGE);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;     // [2]
    uint64_t *tempty = tfull + 2;    // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    volatile int *flags = reinterpret_cast<volatile int *>(tmem_slot + 4);   // [0] abort, [1..] finisher per epi warp

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t deadline = globaltimer() + P.timeout_ns;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        flags[0] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Lay::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

    const int kb_per = P.kb_per;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int it = 0;
            for (int u = blockIdx.x; u < P.units; u += gridDim.x) {
                const int ks = u % P.ksplit, t = u / P.ksplit;
                const int ta = t % P.n_tiles_a, tb = t / P.n_tiles_a;
                const int kb0 = ks * kb_per, kb1 = min(P.nkb, kb0 + kb_per);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t r = (uint32_t)(it / S);
                    if (!flags[0] && !mbar_wait(&empty[s], (r & 1u) ^ 1u, deadline)) {
                        report(P.status, ST_PIPE_TIMEOUT | 0x10u);
                        flags[0] = 1;
                    }
                    if (flags[0]) continue;   // aborted: issue nothing more
                    mbar_arrive_expect_tx(&full[s], Lay::STAGE);
                    unsigned char *st = tiles + (size_t)s * Lay::STAGE;
                    tma_load_2d(st, &tmap_a, kb * TC_BK, ta * TC_BM, &full[s]);
                    tma_load_2d(st + Lay::A_BYTES, &tmap_b, kb * TC_BK, tb * BN, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(TC_BM, BN);
            int it = 0, ut = 0;
            for (int u = blockIdx.x; u < P.units; u += gridDim.x, ++ut) {
                const int ks = u % P.ksplit;
                const int kb0 = ks * kb_per, kb1 = min(P.nkb, kb0 + kb_per);
                const int buf = ut & 1;
                const uint32_t use = (uint32_t)(ut >> 1);
                if (!flags[0] && !mbar_wait(&tempty[buf], (use & 1u) ^ 1u, deadline)) {
                    report(P.status, ST_PIPE_TIMEOUT | 0x20u);
                    flags[0] = 1;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t r = (uint32_t)(it / S);
                    if (!flags[0] && !mbar_wait(&full[s], r & 1u, deadline)) {
                        report(P.status, ST_PIPE_TIMEOUT | 0x30u);
                        flags[0] = 1;
                    }
                    tc_fence_after();
                    if (flags[0]) continue;   // aborted: issue nothing more
                    const uint32_t sa_ = smem_u32(tiles + (size_t)s * Lay::STAGE);
                    const uint64_t adesc = sw128_desc(sa_), bdesc = sw128_desc(sa_ + Lay::A_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 32; ++k)   // 32 bytes of K per MMA: +2 in the 16-byte address field
                        umma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                if (!flags[0]) umma_commit(&tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..5 ----------------
        const int q = warp & 3;            // TMEM lane quarter this warp may access
        const int ew = warp - 2;           // 0..3
        int ut = 0;
        for (int u = blockIdx.x; u < P.units; u += gridDim.x, ++ut) {
            const int t = u / P.ksplit;
            const int ta = t % P.n_tiles_a, tb = t / P.n_tiles_a;
            const int buf = ut & 1;
            const uint32_t use = (uint32_t)(ut >> 1);
            if (!flags[0] && !mbar_wait(&tfull[buf], use & 1u, deadline)) {
                report(P.status, ST_PIPE_TIMEOUT | 0x40u);
                flags[0] = 1;
            }
            tc_fence_after();
            const int arow = ta * TC_BM + q * 32 + lane;          // row of operand A this thread holds
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
            if (!SWAP) {
                // thread = token row m, columns = output features n
                const int m = arow;
                const bool mok = m < P.M;
                const float sam = (mok && !P.s32_out) ? P.sa[P.sa_rows ? m : 0] : 0.f;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(taddr + (uint32_t)c, r);
                    tmem_ld_wait();
                    const int n0 = tb * BN + c;
                    if (!mok) continue;
                    if (P.s32_out) {
                        int *o = reinterpret_cast<int *>(P.out) + (size_t)m * P.N;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + j < P.N) o[n0 + j] = (int)r[j];
                        continue;
                    }
                    T *o = reinterpret_cast<T *>(P.out) + (size_t)m * P.N;
                    if (n0 + 32 <= P.N && (P.N & 7) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint32_t w4[4];
#pragma unroll
                            for (int h = 0; h < 4; ++h) {
                                const int n = n0 + j + 2 * h;
                                const float v0 = __fmul_rn(sam, __fmul_rn(P.sw[P.sw_rows ? n : 0], (float)(int)r[j + 2 * h]));
                                const float v1 =
                                    __fmul_rn(sam, __fmul_rn(P.sw[P.sw_rows ? n + 1 : 0], (float)(int)r[j + 2 * h + 1]));
                                w4[h] = pack2<T>(v0, v1);
                            }
                            *reinterpret_cast<uint4 *>(o + n0 + j) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                        }
                    } else {
                        for (int j = 0; j < 32; ++j) {
                            const int n = n0 + j;
                            if (n < P.N)
                                o[n] = f2t<T>(__fmul_rn(sam, __fmul_rn(P.sw[P.sw_rows ? n : 0], (float)(int)r[j])));
                        }
                    }
                }
            } else {
                // thread = output feature n, columns = tokens m (BN <= 32)
                const int n = arow;
                uint32_t r[32];
                if (BN == 16)
                    tmem_ld16(taddr, r);
                else
                    tmem_ld32(taddr, r);
                tmem_ld_wait();
                const bool nok = n < P.N;
                if (P.ksplit == 1) {
                    if (nok) {
                        // scales and bias only in dequant mode (they are NULL for int32 output)
                        const float swn = P.s32_out ? 0.f : P.sw[P.sw_rows ? n : 0];
                        const float bn = (!P.s32_out && P.bias) ? t2f<T>(reinterpret_cast<const T *>(P.bias)[n]) : 0.f;
                        #pragma unroll
                        for (int m = 0; m < BN; ++m) {
                            if (m >= P.M) continue;
                            if (P.s32_out) {
                                reinterpret_cast<int *>(P.out)[(size_t)m * P.N + n] = (int)r[m];
                            } else {
                                const float sam = P.sa[P.sa_rows ? m : 0];
                                const float v = P.bias ? dequant1b((int)r[m], sam, swn, bn) : dequant1((int)r[m], sam, swn);
                                reinterpret_cast<T *>(P.out)[(size_t)m * P.N + n] = f2t<T>(v);
                            }
                        }
                    }
                } else {
                    // split-K: add this K range's partial sums, then the completing CTA dequantises the tile
                    if (nok)
                        
#pragma unroll
                        for (int m = 0; m < BN; ++m) if (m < P.M) atomicAdd(&P.scratch[(size_t)m * P.N + n], (int)r[m]);
                    __threadfence();
                    __syncwarp();
                    // one ticket per (tile, epilogue warp): the 32 rows this warp covers
                    int last = 0;
                    if (lane == 0) {
                        const int old = atomicAdd(&P.tickets[ta * 4 + q], 1);
                        last = (old + 1 == P.ksplit);
                    }
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (last) {
                        __threadfence();
                        if (nok) {
                            const float swn = P.s32_out ? 0.f : P.sw[P.sw_rows ? n : 0];
                            const float bn =
                                (!P.s32_out && P.bias) ? t2f<T>(reinterpret_cast<const T *>(P.bias)[n]) : 0.f;
                            #pragma unroll
                        for (int m = 0; m < BN; ++m) {
                            if (m >= P.M) continue;
                                int *sp = &P.scratch[(size_t)m * P.N + n];
                                const int acc = __ldcg(sp);
                                *sp = 0;
                                if (P.s32_out) {
                                    reinterpret_cast<int *>(P.out)[(size_t)m * P.N + n] = acc;
                                } else {
                                    const float sam = P.sa[P.sa_rows ? m : 0];
                                    const float v = P.bias ? dequant1b(acc, sam, swn, bn) : dequant1(acc, sam, swn);
                                    reinterpret_cast<T *>(P.out)[(size_t)m * P.N + n] = f2t<T>(v);
                                }
                            }
                        }
                        if (lane == 0) P.tickets[ta * 4 + q] = 0;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            (void)ew;
        }
    }
    // all roles done: free TMEM (the allocating warp), after every TMEM read and MMA has completed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Lay::TMEM_COLS);
    }
}

// rows x K int8 operand, box = 128 bytes of K x box_rows rows, 128-byte swizzle (the UMMA K-major SW128 layout)
static bool make_map(CUtensorMap *m, const void *base, int rows, int K, int box_rows) {
    return make_map_i8(m, base, rows, K, TC_BK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int BN, bool SWAP>
static int launch_tc(const CUtensorMap &ma, const CUtensorMap &mb, TcArgs P, cudaStream_t s) {
    using Lay = TcLayout<BN>;
    const int dev = cur_device();
    const int budget = max_smem_optin(dev) - 2048;   // barriers + 1024-byte alignment slack
    int stages = budget / Lay::STAGE;
    if (stages > 8) stages = 8;
    if (stages < 2) return VT_EARG;
    P.stages = stages;
    const int smem = stages * Lay::STAGE + 1024 + 256;
    static bool attr[VT_MAX_DEV] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(tc_gemm_kernel<T, BN, SWAP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    int g = num_sms(dev);
    if (g > P.units) g = P.units;
    tc_gemm_kernel<T, BN, SWAP><<<g, TC_THREADS, smem, s>>>(ma, mb, P);
    return (int)cudaGetLastError();
}

// Prefill orientation: a [M, K] activations, w [N, K] weights.
template <typename T>
static int big_gemm(const void *a, const void *w, const float *sa, const float *sw, void *out, int M, int N, int K,
                    int s32, unsigned *status, cudaStream_t s) {
    CUtensorMap ma, mb;
    if (!make_map(&ma, a, M, K, TC_BM) || !make_map(&mb, w, N, K, 256)) return VT_EARG;
    TcArgs P{};
    P.rows_a = M;
    P.rows_b = N;
    P.K = K;
    P.n_tiles_a = (M + TC_BM - 1) / TC_BM;
    P.n_tiles_b = (N + 255) / 256;
    P.ksplit = 1;
    P.nkb = (K + TC_BK - 1) / TC_BK;
    P.kb_per = P.nkb;
    P.units = P.n_tiles_a * P.n_tiles_b;
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
    return launch_tc<T, 256, false>(ma, mb, P, s);
}

// Decode orientation: weights as operand A, M <= 32 token rows as operand B, split-K over the SMs.
template <typename T>
static int small_gemm(const void *a, const void *w, const float *sa, const float *sw, const void *bias, void *out,
                      int M, int N, int K, int sa_rows, int sw_rows, int s32, int *scratch, int *tickets,
                      unsigned *status, cudaStream_t s) {
    const int BN = M <= 16 ? 16 : 32;
    CUtensorMap ma, mb;
    if (!make_map(&ma, w, N, K, TC_BM) || !make_map(&mb, a, M, K, BN)) return VT_EARG;
    TcArgs P{};
    P.rows_a = N;
    P.rows_b = M;
    P.K = K;
    P.n_tiles_a = (N + TC_BM - 1) / TC_BM;
    P.n_tiles_b = 1;
    P.nkb = (K + TC_BK - 1) / TC_BK;
    const int sms = num_sms(cur_device());
    int ks = (sms + P.n_tiles_a - 1) / P.n_tiles_a;   // enough units to cover every SM
    if (ks > P.nkb) ks = P.nkb;
    if (ks < 1) ks = 1;
    P.kb_per = (P.nkb + ks - 1) / ks;
    P.ksplit = (P.nkb + P.kb_per - 1) / P.kb_per;   // no empty K range
    P.units = P.n_tiles_a * ks;
    P.sa = sa;
    P.sw = sw;
    P.bias = bias;
    P.sa_rows = sa_rows;
    P.sw_rows = sw_rows;
    P.out = out;
    P.M = M;
    P.N = N;
    P.scratch = scratch;
    P.tickets = tickets;
    P.s32_out = s32;
    P.timeout_ns = pipe_timeout_ns();
    P.status = status;
    if (BN == 16) return launch_tc<T, 16, true>(ma, mb, P, s);
    return launch_tc<T, 32, true>(ma, mb, P, s);
}

// scratch for the decode split-K: int32 [M, N] + tickets [4 per 128-row tile]
inline size_t small_scratch_bytes(int M, int N) {
    return ((size_t)M * N * 4 + (size_t)((N + 127) / 128) * 4 * 4 + 255) & ~(size_t)255;
}

static bool tc_args_ok(const void *a, const void *w, int M, int N, int K) {
    return M >= 1 && N >= 1 && K >= 16 && (K & 15) == 0 && ((uintptr_t)a & 15) == 0 && ((uintptr_t)w & 15) == 0;
}

}  // namespace vt

using namespace vt;

extern "C" {

// The reference's small-M tensor-core entry (vllm_turing/csrc/w8a8_gemv.cu:330-344: M 1..32, same signature and
// return convention): here tcgen05 kind::i8 with the weights as the MMA's A operand, split-K across the SMs.
int w8a8_mma(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M, int N,
             int K, int sa_rows, int sw_rows, int dtype, void *stream) {
    if (!tc_args_ok(a, w, M, N, K) || M > 32) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    if (int rc = ws_acquire(small_scratch_bytes(M, N), s, &scratch, &status)) return rc;
    int *sc = (int *)scratch;
    int *tk = sc + (size_t)M * N;
    if (dtype == 0)
        return small_gemm<__half>(a, w, (const float *)sa, (const float *)sw, bias, out, M, N, K, sa_rows, sw_rows, 0,
                                  sc, tk, status, s);
    return small_gemm<__nv_bfloat16>(a, w, (const float *)sa, (const float *)sw, bias, out, M, N, K, sa_rows, sw_rows,
                                     0, sc, tk, status, s);
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

// int32 accumulators acc[M, N] = a . w^T on the tensor cores (any M; bit-exact parity checks).
int vt_gemm_s32(const void *a, const void *w, void *acc, int M, int N, int K, void *stream) {
    if (!tc_args_ok(a, w, M, N, K)) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    if (M <= 32) {
        if (int rc = ws_acquire(small_scratch_bytes(M, N), s, &scratch, &status)) return rc;
        int *sc = (int *)scratch;
        return small_gemm<__nv_bfloat16>(a, w, nullptr, nullptr, nullptr, acc, M, N, K, 1, 1, 1, sc,
                                         sc + (size_t)M * N, status, s);
    }
    if (int rc = ws_acquire(0, s, &scratch, &status)) return rc;
    return big_gemm<__nv_bfloat16>(a, w, nullptr, nullptr, acc, M, N, K, 1, status, s);
}

}  // extern "C"

// W8A16 GEMM for the LM head on the B200 tensor cores: int8 weight rows with one fp32 scale each, 16-bit float
// activations (bf16 or fp16).
//
//   out[m, n] = T((sum_k x[m, k] * W[n, k]) * s[n] + bias[n])      x [M, K], W [N, K] int8 row-major, s [N] fp32
//
// The reference's W8A16 kernels (vllm_turing/csrc/w8a16_gemv.cu:27-107 on CUDA-core fp32 FMAs,
// vllm_turing/csrc/w8a16_mma.cu on fp16 mma.sync) form every product of an int8 weight and a 16-bit activation exactly
// in fp32, sum in fp32 and apply the row scale and the bias to the finished sum (w8a16_gemv.cu:103). Two kernels here:
//
// 1. Decode, M <= 8 token rows (the default there): the limb GEMM. Each activation row becomes four int8 rows of one
//    fixed-point integer per element (a power of two per token row, base-256 signed digits: exact for every element
//    down to 2^-19 of the row's absmax), the weights stay int8, and the contraction runs on the int8 tensor cores of
//    the W8A8 decode core (tc_core.cuh: tcgen05 kind::i8, weights as the A operand in 128-row tiles fed by TMA,
//    stream-K over the SMs, exact int32 split-K through LL slot words). The finisher combines the four limb sums of a
//    token into the exact int64 dot product and rounds it once to fp32 before the reference's epilogue: the results
//    are the correctly rounded sums, closer to the exact value than any fp32 summation order. No weight byte is
//    converted, so the kernel streams like the int8 decode GEMM.
// 2. M <= 64 (and M <= 8 with VLLM_TURING_W8A16_LIMBS=0): tcgen05 kind::f16 with fp32 accumulators in tensor memory
//    (TMEM); the int8 -> 16-bit conversion runs between shared memory and the tensor core, into TMEM. Only the order
//    of the fp32 additions differs from the reference's, so results agree to the rounding of fp32 sums.
//
// Work layout of kernel 2 (the decode orientation of the W8A8 core): the weights are the MMA's A operand in 128-row
// tiles of the vocabulary; the M <= 64 token rows are its B operand (BN = 16, 32 or 64 rows, zero-filled past M). The
// (tile, K block) index space is cut into one contiguous range per CTA (stream-K), so every SM streams the same share
// of the weights. A split tile is finished by its head CTA from the other CTAs' fp32 partial sums (LL slot words).
//   - warp 0 (one thread) TMA-loads each K block of weights (128 rows x 128 bytes, 128-byte swizzle) into a ring of
//     16 KB shared-memory stages; warp 6 (one thread) loads the K block's activations (two 64-element swizzle atoms
//     of BN rows) into a separate, smaller ring;
//   - warps 7.. convert, two per TMEM lane quarter taking whole K blocks in turn: a thread owns one weight row, reads
//     that row's 128 bytes (the swizzle spreads the 32 row reads of a warp over all banks), hands the weight stage
//     back to the producer at once, converts the bytes exactly to 16-bit floats and stores them with tcgen05.st into
//     a ring of A stages in TMEM (64 columns of two elements per row and K block);
//   - warp 1 (one thread) issues 8 MMAs (K = 16 each) per K block, A from TMEM, B from shared memory;
//   - warps 2..5 drain the accumulators (tcgen05.ld), apply the row scale and the bias and store the logits.
// Because the weight stage is free as soon as it is read, the bytes in flight from HBM are the whole weight ring,
// whatever the conversion and the MMAs take. (A variant with the 16-bit weights in shared memory and the MMA reading
// both operands by descriptor measured no faster.)
//
// Every wait is bounded (globaltimer); on a timeout the CTA records the status, stops issuing, waits (bounded) for the
// copies and MMAs it issued, frees its TMEM and returns.
//
// C ABI (include/vllm_turing_b200.h): w8a16_gemv, w8a16_gemv_rows, w8a16_mma (the reference's signatures,
// w8a16_gemv.cu:114-145 and w8a16_mma.cu:160-175), vt_w8a16_mm and vt_w8a16_ws_bytes (caller-owned workspace, an output
// row stride, M up to 64 in either dtype).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "tc_core.cuh"
#include "tma_host.h"

namespace vt {

// warps: 0 weight producer, 1 MMA, 2..5 epilogue, 6 activation producer, 7.. converters: NW per TMEM lane quarter,
// taking whole K blocks in turn (converter slot i of a quarter converts blocks i, i + NW, ...), so the per-block
// latency chain of one warp (shared loads, conversion, tcgen05.st, tcgen05.wait::st, the arrival) overlaps with the
// other slots' blocks
constexpr int WH_CONV0 = 7;                 // first converter warp
__host__ __device__ constexpr int wh_threads(int nw) { return 32 * (WH_CONV0 + 4 * nw); }
constexpr int WH_AS = 6;                    // A stages in TMEM, one K block (128 elements = 64 columns) each
constexpr int WH_ACOL = 128;                // first TMEM column of the A stages (the accumulators use columns < 128)
constexpr int WH_TMEM_COLS = 512;           // WH_ACOL + WH_AS * 64 = 512
constexpr int WH_W_BYTES = TC_BM * TC_BK;   // int8 weights of one K block: 128 rows x 128 bytes
constexpr int WH_BAR_BYTES = 1024;
constexpr int WH_MAX_M = 64;

// Shared memory: a ring of weight stages (16 KB each) and a separate ring of activation stages (the K block's two
// 64-element swizzle atoms of BN rows). The weight stage is released as soon as the converters have read it, so the
// bytes in flight from HBM are limited by the ring alone -- with weights and activations in one stage, a stage stayed
// occupied through the conversion and the MMAs as well, and at HBM latency under load that halved the stream.
template <int BN> struct WhLayout {
    static constexpr int X_ATOM = BN * 128;            // one 64-element, BN-row swizzle atom of the activations
    static constexpr int X_STAGE = 2 * X_ATOM;
    static constexpr int XS = X_STAGE * 8 <= 32768 ? 8 : 4;   // activation stages: 32 KB (64 KB at BN = 64)
};

struct WhArgs {
    TcArgs t;   // stream-K partition (tc_decode_args), t.sw = the row scales, t.bias, t.out, t.slots, t.status
    int ldo;    // output row stride in elements (>= N)
};

// D (TMEM, fp32) (+)= A (TMEM, 16-bit) . B (shared-memory descriptor)^T, kind::f16
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B both bf16 (bits 7-9, 10-12 = 1) or
// both fp16 (0), both K-major, MMA M x N.
template <typename T> __host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    constexpr uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// 32 consecutive 32-bit TMEM columns of the warp's 32 lanes (thread i writes lane base + i)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Four int8 (one word, element k in the low byte) -> two words of 16-bit floats {k, k+1}, {k+2, k+3} (element k in the
// low half), exactly. The bytes are first spread to 0x00b1_00b0 / 0x00b3_00b2.
//   bf16: with b = v - 128 s (v = b & 127, s = the sign bit), 0x4300 | v is bf16(128 + v) and 0x4300 | (b & 128) is
//         bf16(128 + 128 s); their difference is b (exact: both operands and the result are bf16 integers).
//   fp16: 0x6400 | (b ^ 128) is fp16(1024 + b + 128); minus fp16(1152) = 0x6480 it is b.
template <typename T> __device__ __forceinline__ uint32_t cvt_pair(uint32_t spread);
template <> __device__ __forceinline__ uint32_t cvt_pair<__nv_bfloat16>(uint32_t p) {
    const uint32_t hi = (p & 0x007F007Fu) | 0x43004300u, lo = (p & 0x00800080u) | 0x43004300u;
    __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162 *>(&hi), b = *reinterpret_cast<const __nv_bfloat162 *>(&lo);
    __nv_bfloat162 d = __hsub2(a, b);
    return *reinterpret_cast<uint32_t *>(&d);
}
template <> __device__ __forceinline__ uint32_t cvt_pair<__half>(uint32_t p) {
    const uint32_t u = (p ^ 0x00800080u) | 0x64006400u, c = 0x64806480u;
    __half2 a = *reinterpret_cast<const __half2 *>(&u), b = *reinterpret_cast<const __half2 *>(&c);
    __half2 d = __hsub2(a, b);
    return *reinterpret_cast<uint32_t *>(&d);
}
template <typename T> __device__ __forceinline__ void cvt_word(uint32_t w, uint32_t &o0, uint32_t &o1) {
    o0 = cvt_pair<T>(__byte_perm(w, 0u, 0x4140));
    o1 = cvt_pair<T>(__byte_perm(w, 0u, 0x4342));
}

// all lanes of the warp wait on the same barrier; the warp continues only if every lane saw it complete
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, deadline)) != 0;
}

template <typename T, int BN, int NW>
__global__ void __launch_bounds__(wh_threads(NW), 1)
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const WhArgs A) {
    using Lay = WhLayout<BN>;
    constexpr int XS = Lay::XS;
    const TcArgs &P = A.t;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *wring = tc_align1024(smem_raw);
    const int S = P.stages;                                              // weight stages
    unsigned char *xring = wring + (size_t)S * WH_W_BYTES;               // XS activation stages, 1024-aligned
    uint64_t *wfull = reinterpret_cast<uint64_t *>(xring + (size_t)XS * Lay::X_STAGE);
    uint64_t *wempty = wfull + S;       // [S] the 4 converter warps of the block read it
    uint64_t *xfull = wempty + S;       // [XS]
    uint64_t *xempty = xfull + XS;      // [XS] the MMAs reading it completed (commit)
    uint64_t *afull = xempty + XS;      // [WH_AS] converted K block in TMEM (one converter warp per quarter arrives)
    uint64_t *aempty = afull + WH_AS;   // [WH_AS] the MMAs reading it completed (commit)
    uint64_t *tfull = aempty + WH_AS;   // [2]
    uint64_t *tempty = tfull + 2;       // [2]
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *flags = reinterpret_cast<volatile int *>(tmem_slot + 4);   // [0] abort

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], 4);
        }
        for (int t = 0; t < XS; ++t) {
            mbar_init(&xfull[t], 1);
            mbar_init(&xempty[t], 1);
        }
        for (int a = 0; a < WH_AS; ++a) {
            mbar_init(&afull[a], 4);
            mbar_init(&aempty[a], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        flags[0] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, WH_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    // only the weight producer runs ahead of the previous kernel: the weights and scales are no kernel's output
    const bool wproducer = (warp == 0 && lane == 0);
    if (!wproducer) pdl_wait();
    uint64_t deadline = globaltimer() + P.timeout_ns;

    int ta, tb, kb0, kb1;
    if (warp == 0) {
        // ---------------- weight producer (TMA) ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();   // the head is read once per call
            int it = 0;
            bool dead = false, waited = false;
            TcPieces pc(P);
            while (!dead && pc.next(P, ta, tb, kb0, kb1)) {
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S;
                    if (it == S) {   // the first S stages went out before the wait on the previous kernel
                        pdl_wait();
                        waited = true;
                        deadline = globaltimer() + P.timeout_ns;
                    }
                    if (it >= S && (flags[0] || !mbar_wait(&wempty[s], ((uint32_t)(it / S) & 1u) ^ 1u, deadline))) {
                        if (!flags[0]) report(P.status, ST_PIPE_TIMEOUT | 0x110u);
                        flags[0] = 1;
                        dead = true;
                        break;
                    }
                    mbar_arrive_expect_tx(&wfull[s], (uint32_t)WH_W_BYTES);
                    tma_load_2d_hint(wring + (size_t)s * WH_W_BYTES, &tmap_w, kb * TC_BK, ta * TC_BM, &wfull[s], pol);
                    if (P.l2_runahead > 0) {   // the block l2_runahead units later in this CTA's range, into L2
                        const int v = ta * P.nkb + kb + P.l2_runahead;
                        if (v < pc.hi) tma_prefetch_l2_2d(&tmap_w, (v % P.nkb) * TC_BK, (v / P.nkb) * TC_BM);
                    }
                }
            }
            if (!waited) pdl_wait();   // (a range of at most S blocks never reached the wait above)
            if (dead) {   // let the copies already issued land before the shared memory is released
                const uint64_t d2 = globaltimer() + P.timeout_ns;
                for (int j = (it > S ? it - S : 0); j < it; ++j) mbar_wait(&wfull[j % S], (uint32_t)(j / S) & 1u, d2);
            }
        }
    } else if (warp == 6) {
        // ---------------- activation producer (TMA; the K block's two atoms of the BN token rows) ----------------
        if (lane == 0) {
            int it = 0;
            bool dead = false;
            TcPieces pc(P);
            while (!dead && pc.next(P, ta, tb, kb0, kb1)) {
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int t = it % XS;
                    if (it >= XS && (flags[0] || !mbar_wait(&xempty[t], ((uint32_t)(it / XS) & 1u) ^ 1u, deadline))) {
                        if (!flags[0]) report(P.status, ST_PIPE_TIMEOUT | 0x170u);
                        flags[0] = 1;
                        dead = true;
                        break;
                    }
                    unsigned char *xs = xring + (size_t)t * Lay::X_STAGE;
                    mbar_arrive_expect_tx(&xfull[t], (uint32_t)Lay::X_STAGE);
                    tma_load_2d(xs, &tmap_x, kb * TC_BK, 0, &xfull[t]);
                    tma_load_2d(xs + Lay::X_ATOM, &tmap_x, kb * TC_BK + 64, 0, &xfull[t]);
                }
            }
            if (dead) {
                const uint64_t d2 = globaltimer() + P.timeout_ns;
                for (int j = (it > XS ? it - XS : 0); j < it; ++j)
                    mbar_wait(&xfull[j % XS], (uint32_t)(j / XS) & 1u, d2);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<T>(TC_BM, BN);
            static_assert(2 * BN <= WH_ACOL, "accumulators overlap the A stages");
            int it = 0, ut = 0;
            TcPieces pc(P);
            while (pc.next(P, ta, tb, kb0, kb1)) {
                const int buf = ut & 1;
                const uint32_t use = (uint32_t)(ut >> 1);
                ++ut;
                if (!flags[0] && !mbar_wait(&tempty[buf], (use & 1u) ^ 1u, deadline)) {
                    report(P.status, ST_PIPE_TIMEOUT | 0x120u);
                    flags[0] = 1;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    if (flags[0]) break;   // aborted: issue nothing more
                    const int t = it % XS, a = it % WH_AS;
                    if (!mbar_wait(&xfull[t], (uint32_t)(it / XS) & 1u, deadline) ||
                        !mbar_wait(&afull[a], (uint32_t)(it / WH_AS) & 1u, deadline)) {
                        report(P.status, ST_PIPE_TIMEOUT | 0x130u);
                        flags[0] = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xb = smem_u32(xring + (size_t)t * Lay::X_STAGE);
                    const uint32_t at = tmem_base + (uint32_t)(WH_ACOL + a * 64);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {   // 16 elements (32 bytes: +2 in the descriptor, 8 TMEM columns)
                        const uint64_t bdesc = sw128_desc(xb + (uint32_t)((k >> 2) * Lay::X_ATOM)) + 2 * (k & 3);
                        umma_f16_ts(d, at + 8 * k, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(&aempty[a]);
                    umma_commit(&xempty[t]);
                }
                if (!flags[0]) umma_commit(&tfull[buf]);
            }
            // every MMA this thread issued has completed once `drain` flips (bounded: TMEM is freed after it)
            umma_commit(drain);
            mbar_wait(drain, 0u, globaltimer() + P.timeout_ns);
        }
    } else if (warp >= WH_CONV0) {
        // ---------------- converters: int8 rows (shared memory) -> 16-bit rows (TMEM) ----------------
        const int q = warp & 3;
        const int slot = (warp - WH_CONV0) >> 2;   // this warp converts the blocks it with it % NW == slot
        const int row = q * 32 + lane;
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)WH_ACOL;
        int it = 0;
        bool dead = false;
        TcPieces pc(P);
        while (!dead && pc.next(P, ta, tb, kb0, kb1)) {
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                if (it % NW != slot) continue;
                const int s = it % S, a = it % WH_AS;
                // warp-uniform decisions only: tcgen05.st below is a whole-warp instruction
                const bool aborted = __any_sync(0xffffffffu, flags[0] != 0);
                bool ok = !aborted;
                if (ok) ok = warp_wait(&wfull[s], (uint32_t)(it / S) & 1u, deadline);
                uint4 v[8];
                if (ok) {
                    const unsigned char *src = wring + (size_t)s * WH_W_BYTES + row * TC_BK;
#pragma unroll
                    for (int j = 0; j < 8; ++j)   // the row's 128 bytes; 16-byte chunk j sits at chunk j ^ (row % 8)
                        v[j] = *reinterpret_cast<const uint4 *>(src + ((j ^ (row & 7)) << 4));
                    // the weights are in registers: hand the stage back to the producer before converting
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&wempty[s]);
                    ok = warp_wait(&aempty[a], ((uint32_t)(it / WH_AS) & 1u) ^ 1u, deadline);
                }
                if (!ok) {
                    if (lane == 0 && !aborted) report(P.status, ST_PIPE_TIMEOUT | 0x140u);
                    flags[0] = 1;
                    dead = true;
                    break;
                }
                tc_fence_after();   // the MMAs that read this A stage before have completed
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t o[32];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 w = v[h * 4 + c];
                        cvt_word<T>(w.x, o[8 * c + 0], o[8 * c + 1]);
                        cvt_word<T>(w.y, o[8 * c + 2], o[8 * c + 3]);
                        cvt_word<T>(w.z, o[8 * c + 4], o[8 * c + 5]);
                        cvt_word<T>(w.w, o[8 * c + 6], o[8 * c + 7]);
                    }
                    tmem_st32(lane_base + (uint32_t)(a * 64 + h * 32), o);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[a]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..5 ----------------
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int hw = (P.M + 1) >> 1;
        const T *bias = reinterpret_cast<const T *>(P.bias);
        T *out = reinterpret_cast<T *>(P.out);
        int ut = 0;
        TcPieces pc(P);
        while (pc.next(P, ta, tb, kb0, kb1)) {
            const int buf = ut & 1;
            const uint32_t use = (uint32_t)(ut >> 1);
            ++ut;
            const int n = ta * TC_BM + row;
            const bool nok = n < P.N;
            const bool whole = (kb0 == 0 && kb1 == P.nkb);
            const bool head = (kb0 == 0 && !whole);
            float sn = 0.f, bn = 0.f;   // loads in flight while the MMAs run
            if (nok) {
                sn = P.sw[n];
                if (bias) bn = t2f<T>(bias[n]);
            }
            float acc[BN];
#pragma unroll
            for (int m = 0; m < BN; ++m) acc[m] = 0.f;
            if (head) {
                // the CTAs holding the tile's later K blocks left their fp32 sums in their slots: add them in CTA
                // order (a fixed order: the results do not depend on timing) and clear the slots for the next call
                const int clast = tc_owner(P, ta * P.nkb + P.nkb - 1);
                for (int c = blockIdx.x + 1; c <= clast; ++c) {
#pragma unroll
                    for (int h = 0; h < BN / 2; ++h) {
                        if (h >= hw) continue;
                        uint4 v = ld_volatile16(tc_slot(P, c, h, row));
                        uint32_t spin = 0;
                        while (v.y != 1u || v.w != 1u) {
                            if ((++spin & 255u) == 0 && globaltimer() > deadline) {
                                report(P.status, ST_PIPE_TIMEOUT | 0x150u);
                                break;
                            }
                            v = ld_volatile16(tc_slot(P, c, h, row));
                        }
                        acc[2 * h] += __uint_as_float(v.x);
                        acc[2 * h + 1] += __uint_as_float(v.z);
                        *tc_slot(P, c, h, row) = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
            }
            if (!__any_sync(0xffffffffu, flags[0] != 0) &&
                !__all_sync(0xffffffffu, mbar_wait_sleep(&tfull[buf], use & 1u, deadline, 256))) {
                if (lane == 0) report(P.status, ST_PIPE_TIMEOUT | 0x160u);
                flags[0] = 1;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
            uint32_t r[2][32];
            if (BN == 16) {
                tmem_ld16(taddr, r[0]);
            } else {
                tmem_ld32(taddr, r[0]);
                if (BN == 64) tmem_ld32(taddr + 32u, r[1]);
            }
            tmem_ld_wait();
            tc_fence_before();   // this warp's TMEM reads are done: the MMA may refill the buffer
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
#pragma unroll
            for (int m = 0; m < BN; ++m) acc[m] += __uint_as_float(r[m >> 5][m & 31]);
            if (whole || head) {
                if (nok) {
#pragma unroll
                    for (int m = 0; m < BN; ++m)   // (acc * s + b): the reference's fp32 epilogue, one rounding
                        if (m < P.M) out[(size_t)m * A.ldo + n] = f2t<T>(__fmaf_rn(acc[m], sn, bn));
                }
            } else {
                // the CTA's first piece, inside a tile another CTA finishes: leave its sums in this CTA's slot
#pragma unroll
                for (int h = 0; h < BN / 2; ++h)
                    if (h < hw)
                        ll_store(tc_slot(P, blockIdx.x, h, row), __float_as_uint(acc[2 * h]),
                                 __float_as_uint(acc[2 * h + 1]), 1u);
            }
        }
    }
    // all roles done: free TMEM after every TMEM access and MMA of the CTA has completed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, WH_TMEM_COLS);
    }
}

// ---- CUDA-core gather variant (rows != NULL): out[m, i] = x[m] . W[rows[i]] * s[rows[i]] + bias[rows[i]] ------------
// One warp per output row, lanes striding the weight row in 16-byte chunks (streamed past L1), fp32 FMAs, a shuffle
// reduction. For a subset of the head (a pruned draft vocabulary), where the rows are not tiles of the weight.
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <typename T>
__global__ void __launch_bounds__(256) w8a16_rows_kernel(const T *__restrict__ x, const int8_t *__restrict__ w,
                                                         const float *__restrict__ s, const T *__restrict__ bias,
                                                         T *__restrict__ out, int M, int N, int K,
                                                         const int *__restrict__ rows) {
    const int i = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (i >= N) return;
    const int src = rows ? rows[i] : i;
    const char *wr = reinterpret_cast<const char *>(w) + (size_t)src * K;
    float acc[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) acc[m] = 0.f;
    for (int c = lane; c < (K >> 4); c += 32) {
        const uint4 wv = ld_stream16(wr + (size_t)c * 16);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        float wf[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) wf[j] = (float)(int8_t)(ww[j >> 2] >> (8 * (j & 3)));
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            if (m >= M) break;
            const uint4 *xr = reinterpret_cast<const uint4 *>(x + (size_t)m * K + (size_t)c * 16);
            const uint4 a = __ldg(xr), b = __ldg(xr + 1);
            const uint32_t xs[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            float v = acc[m];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float2 f = unpack2<T>(xs[j]);
                v = __fmaf_rn(wf[2 * j], f.x, v);
                v = __fmaf_rn(wf[2 * j + 1], f.y, v);
            }
            acc[m] = v;
        }
    }
#pragma unroll
    for (int m = 0; m < 16; ++m)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    if (lane == 0) {
        const float sn = s[src], bn = bias ? t2f<T>(bias[src]) : 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m)
            if (m < M) out[(size_t)m * N + i] = f2t<T>(__fmaf_rn(acc[m], sn, bn));
    }
}

// ---- exact int8 limbs of the activations (decode: M <= 8 token rows) ------------------------------------------------
// A 16-bit float row x[m, :] is written as integers X[k] = round(x[k] * 2^-e[m]) with one power of two per row, chosen
// so that max |X| < 2^30: X is exact for every element of magnitude at least 2^-19 of the row's absmax (a bf16 / fp16
// value has at most 11 significant bits), smaller ones are rounded to a multiple of 2^e (an error below 2^-30 of the
// row's absmax). X is
// split into four signed base-256 digits ("limbs"), X = l3 2^24 + l2 2^16 + l1 2^8 + l0, l_j in [-128, 127]. The
// LM head then runs on the int8 tensor cores (kind::i8, int32 accumulators) with B = the 4M limb rows:
//   sum_k x[m, k] W[n, k] = 2^e[m] * sum_j 2^(8 j) * (sum_k l_j[m, k] W[n, k])
// where every inner sum is an exact int32 (|W l| <= 2^14, K < 2^17) and the combination is an exact int64 (< 2^53).
// The finisher rounds that exact sum once to fp32 and applies the reference's fp32 epilogue (acc * s + bias): the
// result is the correctly rounded dot product, not one fp32 summation order of it. No weight byte is converted.
constexpr int WL_MAX_M = 8;   // 4 limbs x 8 token rows = the 32 B rows of the decode core

// limbs [4M, K] int8 (row 4 m + j = limb j of token m), exps[m]: one CTA per token row. Launched with programmatic
// dependent launch: the GEMM after it starts its weight stream meanwhile.
template <typename T>
__global__ void __launch_bounds__(256) w8a16_limbs_kernel(const T *__restrict__ x, int K, int8_t *__restrict__ limbs,
                                                           int *__restrict__ exps) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T *xr = x + (size_t)m * K;
    float mx = 0.0f;
    for (int i = tid * 8; i < K; i += 256 * 8) {   // K % 16 == 0: whole 8-element vectors
        const uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = unpack2<T>(w[j]);
            mx = fmaxf(mx, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    int e = 0;
    if (mx > 0.0f) {   // mx = f 2^E2 with f in [0.5, 1): max |x| < 2^E2, so X < 2^30 with e = E2 - 30
        int E2;
        frexpf(mx, &E2);
        e = E2 - 30;
    }
    if (tid == 0) exps[m] = e;
    int8_t *l0 = limbs + (size_t)(4 * m) * K;
    for (int i = tid * 8; i < K; i += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t out[4][2] = {};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float2 f = unpack2<T>(w[j >> 1]);
            int X = __float2int_rn(ldexpf((j & 1) ? f.y : f.x, -e));
            const int sh = (j & 3) * 8, h = j >> 2;
#pragma unroll
            for (int l = 0; l < 3; ++l) {
                const int d = (int)(int8_t)(X & 0xff);   // the signed digit; X - d is a multiple of 256
                out[l][h] |= (uint32_t)(d & 0xff) << sh;
                X = (X - d) >> 8;
            }
            out[3][h] |= (uint32_t)(X & 0xff) << sh;   // |X| <= 65 here
        }
#pragma unroll
        for (int l = 0; l < 4; ++l)
            *reinterpret_cast<uint2 *>(l0 + (size_t)l * K + i) = make_uint2(out[l][0], out[l][1]);
    }
}

// Finisher of the limb GEMM (tc_phase, decode orientation, B rows = 4 M limb rows): thread = vocabulary row n,
// acc[4 m + j] the exact sums of limb j of token m.
template <typename T, int BN>
struct WhLimbEpi {
    static constexpr int kSmemFloats = 64;
    struct Prep {
        float sn, bn;
    };
    const int *exps;
    const float *s;
    const T *bias;
    T *out;
    int M, ldo;
    int *e_sm;
    __device__ __forceinline__ void on_start(const TcArgs &, float *sm) {
        e_sm = reinterpret_cast<int *>(sm);
        const int t = threadIdx.x - TC_EPI_LEAD;
        if (t < M) e_sm[t] = exps[t];
    }
    __device__ __forceinline__ void post_start() {}
    __device__ __forceinline__ Prep prep(const TcArgs &P, int n) const {
        Prep r{0.0f, 0.0f};
        if (n < P.N) {
            r.sn = s[n];
            if (bias) r.bn = t2f<T>(bias[n]);
        }
        return r;
    }
    __device__ __forceinline__ void operator()(const TcArgs &, int n, bool nok, const int (&acc)[BN],
                                               const Prep &pr) const {
        if (!nok) return;
#pragma unroll
        for (int m = 0; m < BN / 4; ++m) {
            if (m >= M) break;
            const long long S = (long long)acc[4 * m] + ((long long)acc[4 * m + 1] << 8) +
                                ((long long)acc[4 * m + 2] << 16) + ((long long)acc[4 * m + 3] << 24);
            // 2^e as a double built from its exponent field (e in [-180, 98]): the product is exact
            const double p2 = __longlong_as_double((long long)(e_sm[m] + 1023) << 52);
            const float v = __double2float_rn((double)S * p2);
            out[(size_t)m * ldo + n] = f2t<T>(__fmaf_rn(v, pr.sn, pr.bn));   // (acc * s + b): one fp32 rounding
        }
    }
};

template <typename T, int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    w8a16_limb_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_l,
                      TcArgs G, WhLimbEpi<T, BN> fin) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    tc_phase<T, BN, true, 4>(&tmap_w, &tmap_l, G, smem_raw, fin);
}

// ---- host side -------------------------------------------------------------------------------------------------------
template <int BN> inline int wh_stages(int dev) {   // weight stages
    const int fixed = 1024 + WH_BAR_BYTES + 1024 + WhLayout<BN>::XS * WhLayout<BN>::X_STAGE;
    const int s = (max_smem_optin(dev) - fixed) / WH_W_BYTES;
    return s > 16 ? 16 : s;
}
template <int BN> inline int wh_smem_bytes(int stages) {
    return stages * WH_W_BYTES + WhLayout<BN>::XS * WhLayout<BN>::X_STAGE + 1024 + WH_BAR_BYTES;
}

template <typename T, int BN, int NW>
static int launch_wh_nw(const CUtensorMap &mw, const CUtensorMap &mx, WhArgs A, cudaStream_t s) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    const int stages = wh_stages<BN>(dev);
    if (stages < 2) return VT_EARG;
    A.t.stages = stages;
    const int smem = wh_smem_bytes<BN>(stages);
    static bool attr[VT_MAX_DEV] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(w8a16_tc_kernel<T, BN, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    int g = num_sms(dev);
    if (g > A.t.units) g = A.t.units;
    return launch_k(w8a16_tc_kernel<T, BN, NW>, dim3(g), dim3(wh_threads(NW)), smem, s, true, mw, mx, A);
}

// Converter warps per TMEM lane quarter: VLLM_TURING_W8A16_NW = 1, 2 or 3 (default 2; 3 only up to 32 token rows).
inline int w8a16_nw() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_W8A16_NW");
        const int x = e ? atoi(e) : 2;
        v = (x == 1 || x == 3) ? x : 2;
    }
    return v;
}

template <typename T, int BN>
static int launch_wh(const CUtensorMap &mw, const CUtensorMap &mx, WhArgs A, cudaStream_t s) {
    const int nw = w8a16_nw();
    if (nw == 1) return launch_wh_nw<T, BN, 1>(mw, mx, A, s);
    if constexpr (BN <= 32)   // 64 token rows: the epilogue's registers leave room for 15 warps, not 19
        if (nw == 3) return launch_wh_nw<T, BN, 3>(mw, mx, A, s);
    return launch_wh_nw<T, BN, 2>(mw, mx, A, s);
}

// split-K slot bytes for M token rows on this device (one fp32 contribution of 128 x M per CTA, grid <= SMs)
static size_t wh_slot_bytes(int M) { return tc_decode_slot_bytes(M, num_sms(cur_device())); }

static bool wh_args_ok(const void *x, const void *w, const void *s, const void *out, int M, int N, int K, int ldo) {
    return x && w && s && out && M >= 1 && M <= WH_MAX_M && N >= 1 && K >= 16 && (K & 15) == 0 && ldo >= N &&
           ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0;
}

// Caller-owned workspace of vt_w8a16_mm: [256-byte status][limbs: 4 WL_MAX_M rows x K][exps: 256 bytes][split-K
// slots, zeroed]. Through the library workspace the slots come from the zeroed workspace and the limbs from the
// auxiliary buffer (host_util.h), since other kernels rely on the zeroed workspace staying zero.
static size_t wl_limb_bytes(int K) { return ((size_t)4 * WL_MAX_M * K + 255) & ~(size_t)255; }
static size_t wh_slots_bytes(int M) {
    const size_t v2 = wh_slot_bytes(M), limb = tc_decode_slot_bytes(4 * (M < WL_MAX_M ? M : WL_MAX_M),
                                                                    num_sms(cur_device()));
    return v2 > limb ? v2 : limb;
}
static size_t wh_ws_bytes(int M, int K) { return 256 + wl_limb_bytes(K) + 256 + wh_slots_bytes(M); }

// VLLM_TURING_W8A16_LIMBS=0 keeps M <= 8 on the int8 -> 16-bit converting kernel (default: the limb GEMM).
inline bool w8a16_limbs() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_W8A16_LIMBS");
        v = (e && atoi(e) == 0) ? 0 : 1;
    }
    return v != 0;
}

// limbs: wl_limb_bytes(K) + 256 bytes (the limbs, then the exponents), rewritten by every call; slots: zeroed split-K
// slots (left zeroed); status: the status word.
template <typename T, int BN>
static int launch_wl(const void *x, const void *w, const float *s, const void *bias, void *out, int M, int N, int K,
                     int ldo, unsigned *status, void *limbs_buf, void *slots, cudaStream_t st) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    int8_t *limbs = (int8_t *)limbs_buf;
    int *exps = reinterpret_cast<int *>(limbs + wl_limb_bytes(K));
    if (int rc = launch_k(w8a16_limbs_kernel<T>, dim3(M), dim3(256), 0, st, true, (const T *)x, K, limbs, exps))
        return rc;
    CUtensorMap mw, ml;
    if (!tc_make_map(&mw, w, N, K, TC_BM) || !tc_make_map(&ml, limbs, 4 * M, K, BN)) return VT_EARG;
    TcArgs G{};
    tc_decode_args(G, 4 * M, N, K);
    G.l2_prefetch_blocks = 0;
    G.slots = (uint4 *)slots;
    G.status = status;
    G.timeout_ns = pipe_timeout_ns();
    using Fin = WhLimbEpi<T, BN>;
    const int stages = tc_stages<BN, 4>(dev, Fin::kSmemFloats);
    if (stages < 2) return VT_EARG;
    G.stages = stages;
    const int smem = tc_smem_bytes<BN, 4>(stages, Fin::kSmemFloats);
    static bool attr[VT_MAX_DEV] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(w8a16_limb_kernel<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    int g = num_sms(dev);
    if (g > G.units) g = G.units;
    Fin fin{exps, s, (const T *)bias, (T *)out, M, ldo, nullptr};
    return launch_k(w8a16_limb_kernel<T, BN>, dim3(g), dim3(TC_THREADS), smem, st, true, mw, ml, G, fin);
}

// M <= WL_MAX_M runs the limb GEMM (limbs_buf as above) unless switched off; otherwise the converting kernel.
template <typename T>
static int w8a16_tc(const void *x, const void *w, const float *s, const void *bias, void *out, int M, int N, int K,
                    int ldo, unsigned *status, void *limbs_buf, void *slots, cudaStream_t st) {
    if (M <= WL_MAX_M && w8a16_limbs()) {
        if (M <= 4) return launch_wl<T, 16>(x, w, s, bias, out, M, N, K, ldo, status, limbs_buf, slots, st);
        return launch_wl<T, 32>(x, w, s, bias, out, M, N, K, ldo, status, limbs_buf, slots, st);
    }
    const int BN = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    CUtensorMap mw, mx;
    if (!tc_make_map(&mw, w, N, K, TC_BM) || !make_map_b16(&mx, x, M, K, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return VT_EARG;
    WhArgs A{};
    tc_decode_args(A.t, M, N, K);
    A.t.l2_prefetch_blocks = 0;
    A.t.sw = s;
    A.t.sw_rows = 1;
    A.t.bias = bias;
    A.t.out = out;
    A.t.slots = (uint4 *)slots;
    A.t.timeout_ns = pipe_timeout_ns();
    A.t.status = status;
    A.ldo = ldo;
    if (BN == 16) return launch_wh<T, 16>(mw, mx, A, st);
    if (BN == 32) return launch_wh<T, 32>(mw, mx, A, st);
    return launch_wh<T, 64>(mw, mx, A, st);
}

template <typename T>
static int w8a16_rows(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K,
                      const int *rows, cudaStream_t st) {
    const long long threads = (long long)N * 32;
    w8a16_rows_kernel<T><<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        (const T *)x, (const int8_t *)w, (const float *)s, (const T *)bias, (T *)out, M, N, K, rows);
    return (int)cudaGetLastError();
}

static int w8a16_dispatch(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N,
                          int K, int ldo, int dtype, cudaStream_t st) {
    void *scratch, *limbs = nullptr;
    unsigned *status;
    if (int rc = ws_acquire(wh_slots_bytes(M), st, &scratch, &status)) return rc;
    if (M <= WL_MAX_M && w8a16_limbs())
        if (int rc = aux_acquire(wl_limb_bytes(K) + 256, st, &limbs)) return rc;
    if (dtype == 0) return w8a16_tc<__half>(x, w, (const float *)s, bias, out, M, N, K, ldo, status, limbs, scratch, st);
    return w8a16_tc<__nv_bfloat16>(x, w, (const float *)s, bias, out, M, N, K, ldo, status, limbs, scratch, st);
}

}  // namespace vt

using namespace vt;

extern "C" {

// The reference's W8A16 GEMV entry (vllm_turing/csrc/w8a16_gemv.cu:119-123: M 1..16, K % 16 == 0, dtype 0 fp16 /
// 1 bf16, -1 on bad arguments): here the tcgen05 kernel above. Split-K slots come from the library's per-device
// workspace (grown outside stream capture only).
int w8a16_gemv(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K,
               int dtype, void *stream) {
    if (!wh_args_ok(x, w, s, out, M, N, K, N) || M > 16) return VT_EARG;
    return w8a16_dispatch(x, w, s, bias, out, M, N, K, N, dtype, (cudaStream_t)stream);
}

// The reference's gathered variant (w8a16_gemv.cu:125-145): with rows (int32 [N], indices of weight rows) the output
// is [M, N] over that subset, computed by the CUDA-core kernel; without rows it is w8a16_gemv. The caller guarantees
// that every rows[i] indexes a row of w (the reference's contract; nothing here knows the weight's row count).
int w8a16_gemv_rows(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K,
                    int dtype, const void *rows, void *stream) {
    if (!rows) return w8a16_gemv(x, w, s, bias, out, M, N, K, dtype, stream);
    if (!wh_args_ok(x, w, s, out, M, N, K, N) || M > 16) return VT_EARG;
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == 0) return w8a16_rows<__half>(x, w, s, bias, out, M, N, K, (const int *)rows, st);
    return w8a16_rows<__nv_bfloat16>(x, w, s, bias, out, M, N, K, (const int *)rows, st);
}

// The reference's tensor-core W8A16 entry (vllm_turing/csrc/w8a16_mma.cu:160-175: fp16 activations, M 1..64, N even,
// -1 on bad arguments; cfg picks the reference's tiling and is accepted and ignored here).
int w8a16_mma(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K, int cfg,
              void *stream) {
    (void)cfg;
    if (!wh_args_ok(x, w, s, out, M, N, K, N) || (N & 1)) return VT_EARG;
    return w8a16_dispatch(x, w, s, bias, out, M, N, K, N, 0, (cudaStream_t)stream);
}

// Zeroed workspace bytes vt_w8a16_mm needs for M token rows and K (256-byte status header included).
size_t vt_w8a16_ws_bytes(int M, int K) { return wh_ws_bytes(M < 1 ? 1 : M, K < 16 ? 16 : K); }

// W8A16 for M 1..64 in either dtype, with an output row stride ldo (>= N: e.g. this rank's columns of a gathered
// [M, world * N] logits buffer) and a caller-owned workspace of vt_w8a16_ws_bytes(M, K) bytes, zeroed once before its
// first use (the kernels leave its split-K slots zeroed); calls sharing a workspace must be stream-ordered. The first
// 256 bytes hold the status word.
int vt_w8a16_mm(const void *x, const void *w, const void *s, const void *bias, void *out, int M, int N, int K, int ldo,
                int dtype, void *workspace, size_t ws_bytes, void *stream) {
    if (!wh_args_ok(x, w, s, out, M, N, K, ldo) || !workspace || ws_bytes < vt_w8a16_ws_bytes(M, K) ||
        ((uintptr_t)workspace & 255))
        return VT_EARG;
    cudaStream_t st = (cudaStream_t)stream;
    unsigned *status = (unsigned *)workspace;
    char *limbs = (char *)workspace + 256, *slots = limbs + wl_limb_bytes(K) + 256;
    if (dtype == 0)
        return w8a16_tc<__half>(x, w, (const float *)s, bias, out, M, N, K, ldo, status, limbs, slots, st);
    return w8a16_tc<__nv_bfloat16>(x, w, (const float *)s, bias, out, M, N, K, ldo, status, limbs, slots, st);
}

}  // extern "C"

// The tcgen05 kind::i8 GEMM core shared by the W8A8 GEMMs (w8a8_tc.cu) and the fused tensor-parallel row-linear
// (tp_fused.cu): int32 accumulators in tensor memory (TMEM), operands staged by TMA (cp.async.bulk.tensor, 128-byte
// swizzle, no multicast).
//
//   D[rows, cols] = A[rows, K] . B[cols, K]^T   (both K-major int8)
//
// Two orientations:
//   prefill (SWAP = false): A = activations (128-row tiles of M), B = weights (BN-row tiles of N). Whole tiles are
//            dealt round robin to the CTAs; the epilogue thread is a token row m, its columns are output features n.
//   decode  (SWAP = true):  A = weights (128-row tiles of N), B = a few token rows (BN = 16 or 32). Stream-K: the
//            (tile, K block) index space is cut into one contiguous range per CTA, so every SM streams the same number
//            of weight bytes (+-1 K block of 16 KB). A CTA's range falls into "pieces" (one tile, a K-block range).
//            A piece that covers its whole tile is finished in registers. A split tile is finished by the CTA holding
//            its first K blocks (the "head" piece, the last piece of that CTA's range). Every other piece of it is
//            the first piece of its CTA, whose int32 sums go into that CTA's slot of LL words ({sum, 1, sum, 1}:
//            value and flag in each 8-byte half). The head CTA collects the slots (bounded waits) while its own MMAs
//            run, clears them, adds them to its registers (integer sums: exact in any order) and hands the
//            accumulators to the caller's finisher `fin(P, n, n_ok, acc[BN])` (thread = output feature n, acc[m]
//            for token rows m; fin.on_start() runs once in every epilogue thread before the first piece).
//
// CTA = 6 warps: warp 0 issues TMA loads into a ring of shared-memory stages (KBS K blocks of 128 bytes per stage, so
// one barrier round trip moves KBS x 16 KB of weights), warp 1 allocates TMEM and one of its threads issues the MMAs
// (128 x BN x 32 each, 4 per K block) and commits their completion to mbarriers, warps 2..5 drain TMEM (tcgen05.ld;
// warp w may read TMEM lanes 32 (w % 4) .. + 31). TMEM holds two accumulator buffers so the epilogue of one piece
// overlaps the MMAs of the next. Every wait is bounded (globaltimer): on a timeout the CTA records the status, stops
// issuing, waits (bounded) for the copies and MMAs it already issued, frees its TMEM and returns.
//
// Programmatic dependent launch: the phase lets the next kernel in the stream launch as soon as all of its own CTAs
// are resident, and only the producer thread runs before pdl_wait -- it loads the weight half of its first stages,
// which no kernel writes, so the weight stream of a decode layer starts while the previous kernel finishes. (The
// kernels' shared memory keeps two of them off one SM, so their TMEM allocations never wait on each other.)
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "tma_host.h"

namespace vt {

constexpr int TC_THREADS = 192;
constexpr int TC_BK = 128;        // bytes of K per K block (= one 128-byte swizzle row)
constexpr int TC_BM = 128;        // MMA M (rows of operand A per tile)
constexpr int TC_EPI_BAR = 1;     // named barrier of the four epilogue warps
constexpr int TC_EPI_LEAD = 64;   // first epilogue thread (warp 2, lane 0)

// ---- tcgen05 primitives (PTX ISA 8.6+, sm_100a) -------------------------------------------------------------------
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
// 32 TMEM lanes x 32 (16) consecutive 32-bit columns; thread i of the warp receives lane (base lane + i)
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

// ---- work description ------------------------------------------------------------------------------------------------
struct TcArgs {
    int n_tiles_a, n_tiles_b;   // tiles along A rows (128) and B rows (BN)
    int nkb;                    // K blocks of 128 bytes per tile
    int units;                  // prefill: tiles (n_tiles_a * n_tiles_b); decode: K blocks of all tiles (n_tiles_a * nkb)
    int stream_k;               // 1: decode stream-K ranges; 0: whole tiles round robin
    int group_m;                // prefill raster: A tiles per group (each group covers all B tiles)
    int split_tail;             // wide prefill: a last round that fills at most half the grid goes as 128-row halves
    int blocked_a;              // decode: A (the weight) in the tile-blocked layout (tc_a_coords)
    int l2_prefetch_blocks;     // decode: weight K blocks past the ring prefetched into L2 before pdl_wait
    int l2_runahead;            // decode: with each weight K block loaded, the one this many blocks later is
                                // prefetched into L2 (0: off)
    const float *sa, *sw;       // per token, per output feature (NULL in int32 mode)
    const void *bias;           // [N] output dtype or NULL
    int sa_rows, sw_rows;       // 1: per row / feature, 0: one value
    void *out;                  // [M, N] row-major
    int M, N;                   // tokens, output features
    uint4 *slots;               // stream-K: split-K LL slots [grid][hw][128] (16-byte words), zero between calls
    int s32_out;                // write int32 accumulators instead of dequantised values
    int stages;
    uint64_t timeout_ns;
    unsigned *status;
};

template <int BN, int KBS> struct TcLayout {
    static constexpr int A_BYTES = TC_BM * TC_BK;   // one K block of operand A
    static constexpr int B_BYTES = BN * TC_BK;      // one K block of operand B
    static constexpr int KB_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGE = KBS * KB_BYTES;    // stage = [KBS A blocks][KBS B blocks]
    static constexpr int TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
    static constexpr int BAR_BYTES = 512;           // mbarriers, TMEM slot and flags; the finisher's floats follow
};

// The CTA's pieces: (A tile, B tile, K-block range). Identical sequence in every role of the CTA.
struct TcPieces {
    int idx, hi;
    __device__ __forceinline__ explicit TcPieces(const TcArgs &P) {
        if (P.stream_k) {
            idx = (int)((long long)P.units * blockIdx.x / gridDim.x);
            hi = (int)((long long)P.units * (blockIdx.x + 1) / gridDim.x);
        } else {
            idx = blockIdx.x;
            hi = P.units;
        }
    }
    __device__ __forceinline__ bool next(const TcArgs &P, int &ta, int &tb, int &kb0, int &kb1) {
        if (idx >= hi) return false;
        int tile;
        if (P.stream_k) {
            tile = idx / P.nkb;
            kb0 = idx - tile * P.nkb;
            kb1 = min(P.nkb, kb0 + (hi - idx));
            idx += kb1 - kb0;
            ta = tile % P.n_tiles_a;
            tb = tile / P.n_tiles_a;
        } else {
            // grouped raster: tiles in groups of group_m A tiles x all B tiles, A tile fastest, so the ~gridDim
            // tiles in flight at once share a few A and B tiles in L2 instead of streaming all of A per wave
            tile = idx;
            kb0 = 0;
            kb1 = P.nkb;
            idx += gridDim.x;
            const int per_group = P.group_m * P.n_tiles_b;
            const int g = tile / per_group, r = tile - g * per_group;
            const int gm = min(P.group_m, P.n_tiles_a - g * P.group_m);   // the last group may be narrower
            ta = g * P.group_m + r % gm;
            tb = r / gm;
        }
        return true;
    }
};

// Box coordinates of K block kb of A tile ta: the plain row-major [rows, K] operand (x = bytes of K, y = rows), or
// the tile-blocked weight layout [tile][K block][128 rows][128 B] seen as rows of 128 bytes, where each box is one
// contiguous 16 KB block and a CTA's K range of a tile one contiguous stream.
__device__ __forceinline__ void tc_a_coords(const TcArgs &P, int ta, int kb, int &x, int &y) {
    if (P.blocked_a) {
        x = 0;
        y = (ta * P.nkb + kb) * TC_BM;
    } else {
        x = kb * TC_BK;
        y = ta * TC_BM;
    }
}

// First K-block unit of CTA c in the stream-K partition (the formula TcPieces uses), and the CTA holding unit u.
__device__ __forceinline__ int tc_range_lo(const TcArgs &P, int c) {
    return (int)((long long)P.units * c / gridDim.x);
}
__device__ __forceinline__ int tc_owner(const TcArgs &P, int u) {
    int c = (int)((long long)u * gridDim.x / P.units);
    if (c + 1 < (int)gridDim.x && tc_range_lo(P, c + 1) <= u) ++c;
    return c;
}
// Split-K slot words: CTA c's contribution (its first piece, when that piece is not a tile's head), row r of the
// tile, token-row pair h: {acc[2h], 1, acc[2h + 1], 1} (an LL word: each 8-byte half carries its own flag).
__device__ __forceinline__ uint4 *tc_slot(const TcArgs &P, int c, int h, int r) {
    return P.slots + ((size_t)c * ((P.M + 1) >> 1) + h) * TC_BM + r;
}

__device__ __forceinline__ unsigned char *tc_align1024(unsigned char *p) {
    return reinterpret_cast<unsigned char *>(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}

// Output finisher of the decode orientation: thread = output feature n, acc[m] for the token rows. Finisher
// interface: on_start(P, sm) once per epilogue thread after pdl_wait (sm: Fin::kSmemFloats >= 64 floats of shared
// memory the finisher owns), then the epilogue warps synchronise and each calls post_start() (per-thread state in registers); prep(P, n)
// before the piece's accumulators are ready (global loads whose latency then hides behind the MMAs);
// operator()(P, n, nok, acc, prep) with the accumulators.
template <typename T, int BN>
struct TcOutEpi {
    static constexpr int kSmemFloats = 64;
    struct Prep {
        float swn, bn;
    };
    float *sa_sm;   // the token scales, loaded once per CTA
    __device__ __forceinline__ void on_start(const TcArgs &P, float *sm) {
        sa_sm = sm;
        const int t = threadIdx.x - 64;   // the decode finisher reads sa_sm[m] for m < BN <= 32
        if (!P.s32_out && t < P.M && t < kSmemFloats) sm[t] = P.sa[P.sa_rows ? t : 0];
    }
    __device__ __forceinline__ void post_start() {}
    __device__ __forceinline__ Prep prep(const TcArgs &P, int n) const {
        Prep r{0.f, 0.f};
        if (!P.s32_out && n < P.N) {   // scales and bias only in dequant mode (NULL for int32 output)
            r.swn = P.sw[P.sw_rows ? n : 0];
            if (P.bias) r.bn = t2f<T>(reinterpret_cast<const T *>(P.bias)[n]);
        }
        return r;
    }
    __device__ __forceinline__ void operator()(const TcArgs &P, int n, bool nok, const int (&acc)[BN],
                                               const Prep &pr) const {
        if (!nok) return;
        if (P.s32_out) {
#pragma unroll
            for (int m = 0; m < BN; ++m)
                if (m < P.M) reinterpret_cast<int *>(P.out)[(size_t)m * P.N + n] = acc[m];
            return;
        }
#pragma unroll
        for (int m = 0; m < BN; ++m) {
            if (m >= P.M) continue;
            const float sam = sa_sm[m];
            const float v = P.bias ? dequant1b(acc[m], sam, pr.swn, pr.bn) : dequant1(acc[m], sam, pr.swn);
            reinterpret_cast<T *>(P.out)[(size_t)m * P.N + n] = f2t<T>(v);
        }
    }
};

// Prefill epilogue of one accumulator tile: thread = token row m (A row), BN output features from column 0 of taddr.
template <typename T, int BN>
__device__ __forceinline__ void tc_prefill_epilogue(const TcArgs &P, int m, int tb, uint32_t taddr) {
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
        // the reference's CUTLASS epilogue order: sa[m] * (sw[n] * acc) (vllm_turing/csrc/w8a8_big.cu:26-35)
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
                if (n < P.N) o[n] = f2t<T>(__fmul_rn(sam, __fmul_rn(P.sw[P.sw_rows ? n : 0], (float)(int)r[j])));
            }
        }
    }
}

// A finisher with `static constexpr bool kPrefillHooks` takes over the prefill orientation's tiles: the epilogue warps
// call fin.prefill_tile(P, m, ta, tb, taddr) (thread = A row m of tile (ta, tb), its BN accumulators from TMEM column
// 0 of taddr) and, after releasing the TMEM buffer, fin.prefill_tile_done(P, ta, tb, bar, lead) (the four epilogue
// warps that stored the tile: named barrier `bar`, first thread `lead`).
template <class F, class = void> struct TcPrefillHooks : std::false_type {};
template <class F> struct TcPrefillHooks<F, std::void_t<decltype(F::kPrefillHooks)>> : std::true_type {};

// The GEMM phase: every thread of the CTA (TC_THREADS) calls it; it returns after the CTA's pieces are done and its
// TMEM is freed (a __syncthreads is the last thing it does, so the caller may reuse the shared memory). `fin` is the
// calling thread's own finisher object: state it keeps (in the epilogue threads) is there after the phase.
template <typename T, int BN, bool SWAP, int KBS, class Fin>
__device__ __forceinline__ void tc_phase(const CUtensorMap *tmap_a, const CUtensorMap *tmap_b, const TcArgs &P,
                                         unsigned char *smem_raw, Fin &fin) {
    using Lay = TcLayout<BN, KBS>;
    static_assert(!SWAP || BN <= 32, "decode orientation holds at most 32 token rows");
    unsigned char *tiles = tc_align1024(smem_raw);
    const int S = P.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + (size_t)S * Lay::STAGE);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;     // [2]
    uint64_t *tempty = tfull + 2;    // [2]
    uint64_t *drain = tempty + 2;    // [1]: the MMA issuer's last commit
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *flags = reinterpret_cast<volatile int *>(tmem_slot + 4);   // [0] abort
    // the finisher's shared floats (Fin::kSmemFloats, at least 64) after the barriers
    float *epi_sm = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(full) + Lay::BAR_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();   // once every CTA of this grid got here, the next kernel may take SMs as they free up

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        flags[0] = 0;
        flags[1] = 0;
        fence_mbar_init();
        tma_prefetch_desc(tmap_a);
        tma_prefetch_desc(tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Lay::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    // Everything but the weight stream depends on earlier kernels (activations, scales, scratch, outputs): only the
    // producer thread runs ahead, loading the weight half of its first stages before it waits.
    const bool producer = (warp == 0 && lane == 0);
    if (!producer) pdl_wait();
    uint64_t deadline = globaltimer() + P.timeout_ns;   // the bound starts once the kernel's inputs are ready

    int ta, tb, kb0, kb1;
    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();   // decode weights are read once per call
            // (1) before the wait: the weight (SWAP) half of the first S stages -- their ring slots are free and
            // nothing an earlier kernel writes is read
            int pre = 0;
            if (SWAP) {
                TcPieces pp(P);
                while (pre < S && pp.next(P, ta, tb, kb0, kb1)) {
                    for (int kb = kb0; kb < kb1 && pre < S; kb += KBS, ++pre) {
                        const int nb = min(KBS, kb1 - kb);
                        mbar_arrive_expect_tx(&full[pre], (uint32_t)(nb * Lay::KB_BYTES));
                        unsigned char *st = tiles + (size_t)pre * Lay::STAGE;
                        for (int j = 0; j < nb; ++j) {
                            int ax, ay;
                            tc_a_coords(P, ta, kb + j, ax, ay);
                            tma_load_2d_hint(st + j * Lay::A_BYTES, tmap_a, ax, ay, &full[pre], pol);
                        }
                    }
                }
                // and the next l2_prefetch_blocks weight blocks of the range into L2, so the stream keeps going past
                // the ring while the previous kernel finishes
                TcPieces pq(P);
                int stage = 0, left = P.l2_prefetch_blocks;
                while (left > 0 && pq.next(P, ta, tb, kb0, kb1)) {
                    for (int kb = kb0; kb < kb1 && left > 0; kb += KBS, ++stage) {
                        if (stage < pre) continue;
                        for (int j = 0; j < min(KBS, kb1 - kb) && left > 0; ++j, --left) {
                            int ax, ay;
                            tc_a_coords(P, ta, kb + j, ax, ay);
                            tma_prefetch_l2_2d(tmap_a, ax, ay);
                        }
                    }
                }
            }
            pdl_wait();
            deadline = globaltimer() + P.timeout_ns;
            // (2) the stream: activations for the pre-issued stages, then whole stages
            int it = 0;
            bool dead = false;
            TcPieces pc(P);
            while (!dead && pc.next(P, ta, tb, kb0, kb1)) {
                for (int kb = kb0; kb < kb1; kb += KBS) {
                    const int nb = min(KBS, kb1 - kb);
                    const int s = it % S;
                    const uint32_t r = (uint32_t)(it / S);
                    unsigned char *st = tiles + (size_t)s * Lay::STAGE;
                    if (it >= pre) {
                        if (flags[0] || !mbar_wait(&empty[s], (r & 1u) ^ 1u, deadline)) {
                            if (!flags[0]) report(P.status, ST_PIPE_TIMEOUT | 0x10u);
                            flags[0] = 1;
                            dead = true;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], (uint32_t)(nb * Lay::KB_BYTES));
                        for (int j = 0; j < nb; ++j) {
                            int ax, ay;
                            tc_a_coords(P, ta, kb + j, ax, ay);
                            if (SWAP)
                                tma_load_2d_hint(st + j * Lay::A_BYTES, tmap_a, ax, ay, &full[s], pol);
                            else
                                tma_load_2d(st + j * Lay::A_BYTES, tmap_a, ax, ay, &full[s]);
                        }
                    }
                    if (SWAP && P.l2_runahead > 0) {
                        // L2 run-ahead: the weight block l2_runahead units later in this CTA's range, so that its
                        // stage load finds it in L2 and the bytes in flight are not bounded by the ring alone
                        for (int j = 0; j < nb; ++j) {
                            const int v = ta * P.nkb + kb + j + P.l2_runahead;
                            if (v >= pc.hi) break;
                            int ax, ay;
                            tc_a_coords(P, v / P.nkb, v % P.nkb, ax, ay);
                            tma_prefetch_l2_2d(tmap_a, ax, ay);
                        }
                    }
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(st + KBS * Lay::A_BYTES + j * Lay::B_BYTES, tmap_b, (kb + j) * TC_BK, tb * BN,
                                    &full[s]);
                    ++it;
                }
            }
            if (dead) {   // let the copies already issued land before the shared memory is released
                const uint64_t d2 = globaltimer() + P.timeout_ns;
                for (int j = (it > S ? it - S : 0); j < it; ++j) mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, d2);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(TC_BM, BN);
            int it = 0, ut = 0;
            TcPieces pc(P);
            while (pc.next(P, ta, tb, kb0, kb1)) {
                const int buf = ut & 1;
                const uint32_t use = (uint32_t)(ut >> 1);
                ++ut;
                if (!flags[0] && !mbar_wait(&tempty[buf], (use & 1u) ^ 1u, deadline)) {
                    report(P.status, ST_PIPE_TIMEOUT | 0x20u);
                    flags[0] = 1;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                for (int kb = kb0; kb < kb1; kb += KBS, ++it) {
                    const int nb = min(KBS, kb1 - kb);
                    const int s = it % S;
                    const uint32_t r = (uint32_t)(it / S);
                    if (flags[0]) break;   // aborted: issue nothing more
                    if (!mbar_wait(&full[s], r & 1u, deadline)) {
                        report(P.status, ST_PIPE_TIMEOUT | 0x30u);
                        flags[0] = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = smem_u32(tiles + (size_t)s * Lay::STAGE);
                    for (int j = 0; j < nb; ++j) {
                        const uint64_t adesc = sw128_desc(sbase + j * Lay::A_BYTES);
                        const uint64_t bdesc = sw128_desc(sbase + KBS * Lay::A_BYTES + j * Lay::B_BYTES);
#pragma unroll
                        for (int k = 0; k < TC_BK / 32; ++k)   // 32 bytes of K per MMA: +2 in the 16-byte field
                            umma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > kb0 || j > 0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                }
                if (!flags[0]) umma_commit(&tfull[buf]);
            }
            // every MMA this thread issued has completed once `drain` flips (bounded: TMEM is freed after it)
            umma_commit(drain);
            mbar_wait(drain, 0u, globaltimer() + P.timeout_ns);
        }
    } else {
        // ---------------- epilogue warps 2..5 ----------------
        const int q = warp & 3;   // TMEM lane quarter this warp may access
        const int row = q * 32 + lane;   // row of the 128-row A tile this thread holds
        fin.on_start(P, epi_sm);  // after pdl_wait: e.g. the token scales, the communicator's call number
        named_sync(TC_EPI_BAR, 128);
        fin.post_start();         // per-thread state from what on_start shared
        const int hw = (P.M + 1) >> 1;
        int ut = 0;
        TcPieces pc(P);
        while (pc.next(P, ta, tb, kb0, kb1)) {
            const int buf = ut & 1;
            const uint32_t use = (uint32_t)(ut >> 1);
            ++ut;
            const int arow = ta * TC_BM + row;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
            if constexpr (!SWAP) {
                if (!flags[0] && !mbar_wait(&tfull[buf], use & 1u, deadline)) {
                    report(P.status, ST_PIPE_TIMEOUT | 0x40u);
                    flags[0] = 1;
                }
                tc_fence_after();
                if constexpr (TcPrefillHooks<Fin>::value)
                    fin.prefill_tile(P, arow, ta, tb, taddr);   // the finisher's own destination for the tile
                else
                    tc_prefill_epilogue<T, BN>(P, arow, tb, taddr);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
                if constexpr (TcPrefillHooks<Fin>::value) fin.prefill_tile_done(P, ta, tb, TC_EPI_BAR, TC_EPI_LEAD);
            } else {
                const int n = arow;
                const bool nok = n < P.N;
                const bool whole = (kb0 == 0 && kb1 == P.nkb);
                const bool head = (kb0 == 0 && !whole);
                const auto pr = fin.prep(P, n);   // scale loads in flight while the MMAs run
                int acc[BN];
#pragma unroll
                for (int m = 0; m < BN; ++m) acc[m] = 0;
                if (head) {
                    // This CTA finishes the tile: the CTAs holding its other K blocks (each one's first piece) left
                    // their sums in their slots, normally long ago -- collect them while this piece's MMAs still run,
                    // and clear the slots for the next launch.
                    // One contributor at a time, its words in flight together. (Tried: all contributors' words in one
                    // flight. It measured slower, likely because this code runs once per CTA per launch from a cold
                    // instruction cache, where the larger unrolled body costs more in fetches than the round trips
                    // it saves.)
                    const int clast = tc_owner(P, ta * P.nkb + P.nkb - 1);
                    for (int c = blockIdx.x + 1; c <= clast; ++c) {
                        uint4 v[BN / 2];
#pragma unroll
                        for (int h = 0; h < BN / 2; ++h)
                            if (h < hw) v[h] = ld_volatile16(tc_slot(P, c, h, row));
#pragma unroll
                        for (int h = 0; h < BN / 2; ++h) {
                            if (h >= hw) continue;
                            uint32_t it = 0;
                            while (v[h].y != 1u || v[h].w != 1u) {
                                if ((++it & 255u) == 0 && globaltimer() > deadline) {
                                    report(P.status, ST_PIPE_TIMEOUT | 0x50u);
                                    break;
                                }
                                v[h] = ld_volatile16(tc_slot(P, c, h, row));
                            }
                            acc[2 * h] += (int)v[h].x;
                            acc[2 * h + 1] += (int)v[h].z;
                            *tc_slot(P, c, h, row) = make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
                }
                if (!flags[0] && !mbar_wait(&tfull[buf], use & 1u, deadline)) {
                    report(P.status, ST_PIPE_TIMEOUT | 0x40u);
                    flags[0] = 1;
                }
                tc_fence_after();
                uint32_t r[32];
                if (BN == 16)
                    tmem_ld16(taddr, r);
                else
                    tmem_ld32(taddr, r);
                tmem_ld_wait();
                tc_fence_before();   // this warp's TMEM reads are done: the MMA may refill the buffer
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
#pragma unroll
                for (int m = 0; m < BN; ++m) acc[m] += (int)r[m];
                if (whole || head) {
                    fin(P, n, nok, acc, pr);
                } else {
                    // the CTA's first piece, inside a tile another CTA finishes: leave its sums in this CTA's slot
#pragma unroll
                    for (int h = 0; h < BN / 2; ++h)
                        if (h < hw) ll_store(tc_slot(P, blockIdx.x, h, row), (uint32_t)acc[2 * h],
                                             (uint32_t)acc[2 * h + 1], 1u);
                }
            }
        }
    }
    // all roles done: free TMEM (the allocating warp) after every TMEM read and MMA has completed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Lay::TMEM_COLS);
    }
    __syncthreads();
}

// ---- prefill, wide tiles: 256 x 256 per CTA ------------------------------------------------------------------------
// The prefill orientation with two 128-row A halves per tile sharing one 256-row B tile: per 128-byte K block a stage
// holds A0 | A1 | B (16 + 16 + 32 KB) and feeds 2 x 4 MMAs (128 x 256 x 32) into two accumulators, a0 in TMEM
// columns [0, 256) and a1 in [256, 512). Against 128 x 256 tiles this moves a third fewer bytes from L2 to the SM per
// MMA (64 KB per two 128 x 256 x 128 blocks instead of 2 x 48 KB), and three 64 KB stages cover 3 x 1024 tensor cycles
// of L2 latency instead of 4 x 512. TMEM holds one tile: two groups of four epilogue warps drain a0 and a1 at the same
// time and hand each back on its own barrier (the block has 10 warps, TCW_THREADS). A 128-row half is the unit the
// finisher sees: tile index ta2 = 2 ta + h (the prefill hooks' `ta`), rows 128 ta2 .. + 127; a half entirely past M is
// skipped (the loads read zeros there).
constexpr int TCW_BN = 256;
constexpr int TCW_THREADS = 320;   // producer warp, MMA warp, two groups of four epilogue warps (one per half)
struct TcWideLayout {
    static constexpr int A_BYTES = TC_BM * TC_BK;                 // one 128-row half, one K block
    static constexpr int B_BYTES = TCW_BN * TC_BK;
    static constexpr int STAGE = 2 * A_BYTES + B_BYTES;           // 64 KB
    static constexpr int TMEM_COLS = 512;
    static constexpr int BAR_BYTES = 512;
};

// The wide phase's pieces: whole 256 x 256 tiles dealt round robin over the grid (grouped raster, as TcPieces), except
// that when the last round would keep at most half the CTAs busy, its tiles are dealt as 128-row halves instead (twice
// the pieces, half the work each: that round ends in about half the time). A piece is (ta, tb, half): half = -1 for
// a whole tile, 0 or 1 for one 128-row half (rows 256 ta + 128 half ..), which goes through accumulator a0 only.
struct TcWidePieces {
    int idx, total, whole;
    __device__ __forceinline__ explicit TcWidePieces(const TcArgs &P) {
        const int G = gridDim.x, U = P.units;
        const int rounds = U / G, rem = U - rounds * G;
        whole = (P.split_tail && rem > 0 && 2 * rem <= G) ? rounds * G : U;
        total = whole + 2 * (U - whole);
        idx = blockIdx.x;
    }
    __device__ __forceinline__ bool next(const TcArgs &P, int &ta, int &tb, int &half) {
        for (;;) {
            if (idx >= total) return false;
            int t;
            if (idx < whole) {
                t = idx;
                half = -1;
            } else {
                t = whole + ((idx - whole) >> 1);
                half = (idx - whole) & 1;
            }
            idx += gridDim.x;
            const int per_group = P.group_m * P.n_tiles_b;
            const int g = t / per_group, r = t - g * per_group;
            const int gm = min(P.group_m, P.n_tiles_a - g * P.group_m);
            ta = g * P.group_m + r % gm;
            tb = r / gm;
            const bool dead1 = (2 * ta + 1) * TC_BM >= P.M;   // the tile's second half holds no rows of A
            if (half < 0 && dead1) half = 0;                 // a whole tile over M's last 128 rows: its first half
            if (half == 1 && dead1) continue;                // a half past M: nothing to compute
            return true;
        }
    }
};

template <typename T, class Fin>
__device__ __forceinline__ void tc_phase_wide(const CUtensorMap *tmap_a, const CUtensorMap *tmap_b, const TcArgs &P,
                                              unsigned char *smem_raw, Fin &fin) {
    using Lay = TcWideLayout;
    unsigned char *tiles = tc_align1024(smem_raw);
    const int S = P.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + (size_t)S * Lay::STAGE);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;     // [1]: the tile's last MMAs completed
    uint64_t *tempty = tfull + 1;    // [2]: a0 / a1 drained by the four epilogue warps
    uint64_t *drain = tempty + 2;    // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *flags = reinterpret_cast<volatile int *>(tmem_slot + 4);
    float *epi_sm = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(full) + Lay::BAR_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(&tempty[0], 4);
        mbar_init(&tempty[1], 4);
        mbar_init(drain, 1);
        flags[0] = 0;
        fence_mbar_init();
        tma_prefetch_desc(tmap_a);
        tma_prefetch_desc(tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Lay::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    pdl_wait();
    const uint64_t deadline = globaltimer() + P.timeout_ns;

    int ta, tb, kb0, kb1;
    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int it = 0, half;
            bool dead = false;
            TcWidePieces pc(P);
            while (!dead && pc.next(P, ta, tb, half)) {
                for (int kb = 0; kb < P.nkb; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t r = (uint32_t)(it / S);
                    if (flags[0] || !mbar_wait(&empty[s], (r & 1u) ^ 1u, deadline)) {
                        if (!flags[0]) report(P.status, ST_PIPE_TIMEOUT | 0x11u);
                        flags[0] = 1;
                        dead = true;
                        break;
                    }
                    unsigned char *st = tiles + (size_t)s * Lay::STAGE;
                    if (half < 0) {
                        mbar_arrive_expect_tx(&full[s], (uint32_t)Lay::STAGE);
                        tma_load_2d(st, tmap_a, kb * TC_BK, ta * 2 * TC_BM, &full[s]);
                        tma_load_2d(st + Lay::A_BYTES, tmap_a, kb * TC_BK, ta * 2 * TC_BM + TC_BM, &full[s]);
                    } else {   // one 128-row half: its A rows into the first A slot
                        mbar_arrive_expect_tx(&full[s], (uint32_t)(Lay::A_BYTES + Lay::B_BYTES));
                        tma_load_2d(st, tmap_a, kb * TC_BK, ta * 2 * TC_BM + half * TC_BM, &full[s]);
                    }
                    tma_load_2d(st + 2 * Lay::A_BYTES, tmap_b, kb * TC_BK, tb * TCW_BN, &full[s]);
                }
            }
            if (dead) {
                const uint64_t d2 = globaltimer() + P.timeout_ns;
                for (int j = (it > S ? it - S : 0); j < it; ++j) mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, d2);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(TC_BM, TCW_BN);
            int it = 0, ut = 0, half;
            TcWidePieces pc(P);
            while (pc.next(P, ta, tb, half)) {
                const uint32_t use = (uint32_t)ut++;
                kb0 = 0;
                kb1 = P.nkb;
                const int nh = half < 0 ? 2 : 1;   // accumulators this piece writes (a half piece: a0 only)
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t r = (uint32_t)(it / S);
                    if (flags[0]) break;
                    if (!mbar_wait(&full[s], r & 1u, deadline)) {
                        report(P.status, ST_PIPE_TIMEOUT | 0x31u);
                        flags[0] = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = smem_u32(tiles + (size_t)s * Lay::STAGE);
                    const uint64_t bdesc = sw128_desc(sbase + 2 * Lay::A_BYTES);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (h >= nh) break;
                        if (kb == kb0 && use > 0) {   // accumulator h of the previous piece drained
                            if (!flags[0] && !mbar_wait(&tempty[h], (use - 1) & 1u, deadline)) {
                                report(P.status, ST_PIPE_TIMEOUT | 0x21u);
                                flags[0] = 1;
                            }
                            tc_fence_after();
                        }
                        const uint64_t adesc = sw128_desc(sbase + h * Lay::A_BYTES);
                        const uint32_t d = tmem_base + (uint32_t)(h * TCW_BN);
#pragma unroll
                        for (int k = 0; k < TC_BK / 32; ++k)
                            umma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                }
                // a half piece leaves a1 alone, but still takes a1's hand-back of the previous piece, so that every
                // piece moves a1's barrier by one phase whatever the order of whole and half pieces
                if (nh == 1 && use > 0 && !flags[0]) {
                    if (!mbar_wait(&tempty[1], (use - 1) & 1u, deadline)) {
                        report(P.status, ST_PIPE_TIMEOUT | 0x22u);
                        flags[0] = 1;
                    }
                }
                if (!flags[0]) umma_commit(tfull);
            }
            umma_commit(drain);
            mbar_wait(drain, 0u, globaltimer() + P.timeout_ns);
        }
    } else {
        // ---------------- epilogue: warps 2..5 drain a0, warps 6..9 drain a1, concurrently ----------------
        const int q = warp & 3;          // the TMEM lane quarter this warp may access
        const int h = (warp - 2) >> 2;   // the accumulator half it drains
        const int row = q * 32 + lane;
        const int bar = TC_EPI_BAR + h, lead = TC_EPI_LEAD + 128 * h;   // this half's four warps
        fin.on_start(P, epi_sm);
        named_sync(TC_EPI_BAR + 2, 256);   // all eight epilogue warps (barrier ids 1, 2: the halves; 3: all)
        fin.post_start();
        int ut = 0, half;
        TcWidePieces pc(P);
        while (pc.next(P, ta, tb, half)) {
            const uint32_t use = (uint32_t)ut++;
            if (!flags[0] && !mbar_wait_sleep(tfull, use & 1u, deadline, 256)) {
                report(P.status, ST_PIPE_TIMEOUT | 0x41u);
                flags[0] = 1;
            }
            tc_fence_after();
            // a whole tile: group h drains a_h (rows 128 (2 ta + h) ..); a half piece: group 0 drains a0 (its rows),
            // group 1 has nothing to drain but still hands a1 back (the MMA side counts one hand-back per piece)
            const int ta2 = half < 0 ? ta * 2 + h : ta * 2 + half;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * TCW_BN);
            const bool live = (half < 0 || h == 0) && ta2 * TC_BM < P.M;   // a half past M holds only zero rows
            if (live) {
                if constexpr (TcPrefillHooks<Fin>::value)
                    fin.prefill_tile(P, ta2 * TC_BM + row, ta2, tb, taddr);
                else
                    tc_prefill_epilogue<T, TCW_BN>(P, ta2 * TC_BM + row, tb, taddr);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[h]);
            if constexpr (TcPrefillHooks<Fin>::value)
                if (live) fin.prefill_tile_done(P, ta2, tb, bar, lead);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Lay::TMEM_COLS);
    }
    __syncthreads();
}

// Grid of the wide phase: one CTA per SM, or per whole tile when there are fewer; with split_tail, at most half the
// SMs' worth of tiles runs as 128-row halves on twice the CTAs (TcWidePieces: all pieces are then halves).
inline int tc_wide_grid(int sms, const TcArgs &P) {
    if (P.units >= sms) return sms;
    if (P.split_tail && 2 * P.units <= sms) return 2 * P.units;
    return P.units;
}

inline int tc_wide_stages(int dev, int epi_floats = 64) {
    const int cap = max_smem_optin(dev);
    int s = (cap - 1024 - TcWideLayout::BAR_BYTES - 4 * epi_floats - 1024) / TcWideLayout::STAGE;
    return s > 8 ? 8 : s;
}
inline int tc_wide_smem_bytes(int stages, int epi_floats = 64) {
    return stages * TcWideLayout::STAGE + 1024 + TcWideLayout::BAR_BYTES + 4 * epi_floats;
}

// VLLM_TURING_PREFILL_WIDE=0 selects the 128 x 256 prefill tiles (tc_phase) instead of the 256 x 256 ones.
inline bool prefill_wide() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_PREFILL_WIDE");
        v = (e && atoi(e) == 0) ? 0 : 1;
    }
    return v != 0;
}

// VLLM_TURING_PREFILL_SPLIT=0 keeps the wide phase's last round as whole tiles (TcArgs::split_tail).
inline int prefill_split_tail() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_PREFILL_SPLIT");
        v = (e && atoi(e) == 0) ? 0 : 1;
    }
    return v;
}

// ---- host side -------------------------------------------------------------------------------------------------------
// rows x K int8 operand, box = 128 bytes of K x box_rows rows, 128-byte swizzle (the UMMA K-major SW128 layout)
inline bool tc_make_map(CUtensorMap *m, const void *base, int rows, int K, int box_rows) {
    return make_map_i8(m, base, rows, K, TC_BK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Stages that fit the opt-in shared memory, less the 1024-byte alignment slack, the barriers, the finisher's
// `epi_floats` shared floats and up to 1 KB of static shared variables of the kernel.
// budget: dynamic shared memory to stay under (0 = the device's opt-in maximum).
template <int BN, int KBS>
inline int tc_stages(int dev, int epi_floats = 64, int budget = 0) {
    using Lay = TcLayout<BN, KBS>;
    const int cap = budget > 0 && budget < max_smem_optin(dev) ? budget : max_smem_optin(dev);
    int s = (cap - 1024 - Lay::BAR_BYTES - 4 * epi_floats - 1024) / Lay::STAGE;
    return s > 16 ? 16 : s;
}

// Shared-memory budget of the decode kernels: VLLM_TURING_TC_SMEM_KB (default 0 = all of it). Under half an SM's
// shared memory, the next decode kernel's CTAs can become resident beside the current one's (programmatic dependent
// launch) and fill their pipelines during its tail. Measured on the 64-layer stack: 112 KB with 2 K blocks per stage
// is even at TP4 and 5 % slower at TP1 (the halved pipeline costs more than the overlap gains), so it is off.
inline int decode_smem_budget() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_TC_SMEM_KB");
        v = e ? atoi(e) * 1024 : 0;
        if (v < 0) v = 0;
    }
    return v;
}
template <int BN, int KBS>
inline int tc_smem_bytes(int stages, int epi_floats = 64) {
    return stages * TcLayout<BN, KBS>::STAGE + 1024 + TcLayout<BN, KBS>::BAR_BYTES + 4 * epi_floats;
}

// K blocks per pipeline stage of the decode orientation: VLLM_TURING_TC_KBS (1, 2 or 4; default 4)
inline int decode_kbs() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_TC_KBS");
        const int x = e ? atoi(e) : 4;
        v = (x == 1 || x == 2) ? x : 4;
    }
    return v;
}

// Decode stream-K work: weights w [N, K] as operand A, M token rows as operand B.
// Weight bytes per CTA prefetched into L2 ahead of pdl_wait: VLLM_TURING_L2_PREFETCH_KB (default 0 = off; on the
// 64-layer decode stack 512 KB measured 5 % slower and 2 MB 8 % slower -- the prefetches compete with the previous
// kernel's own weight stream for HBM).
inline int l2_prefetch_blocks() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_L2_PREFETCH_KB");
        const int kb = e ? atoi(e) : 0;
        v = kb > 0 ? kb * 1024 / (TC_BM * TC_BK) : 0;
    }
    return v;
}

// L2 run-ahead of the decode weight stream, in K blocks of 16 KB: VLLM_TURING_L2_RUNAHEAD (default 0 = off)
inline int l2_runahead() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_L2_RUNAHEAD");
        const int x = e ? atoi(e) : 0;
        v = x > 0 ? (x > 4096 ? 4096 : x) : 0;
    }
    return v;
}

inline void tc_decode_args(TcArgs &P, int M, int N, int K) {  // (the launch grid is min(SMs, units))
    P.n_tiles_a = (N + TC_BM - 1) / TC_BM;
    P.n_tiles_b = 1;
    P.nkb = (K + TC_BK - 1) / TC_BK;
    P.units = P.n_tiles_a * P.nkb;
    P.stream_k = 1;
    P.l2_prefetch_blocks = pdl_enabled() ? l2_prefetch_blocks() : 0;
    P.l2_runahead = l2_runahead();
    P.M = M;
    P.N = N;
}

// split-K slots of the decode orientation: one contribution of up to 128 x M int32 per CTA, as 16-byte LL words
inline size_t tc_decode_slot_bytes(int M, int grid) {
    return (size_t)grid * ((M + 1) / 2) * TC_BM * 16;
}

}  // namespace vt

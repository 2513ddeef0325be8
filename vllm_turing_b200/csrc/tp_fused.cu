// Fused tensor-parallel row-linear layer tail for B200 (sm_100a), decode shapes (M <= 32 token rows), ONE kernel:
//
//   partial_r = bf16( (a_r . w_r^T) * sa_r[m] * sw_r[n] )           this rank's K-slice   (vllm_turing/w8a8.py path)
//   reduced   = bf16( sum_r float(partial_r) )  in rank order         the TP all-reduce      (host_ar.cu:90-101)
//   residual  = bf16( reduced + residual )                            written in place
//   y         = bf16( residual * rsqrt(mean(residual^2) + eps) * norm_w )
//   q, scales = per-token int8 quantisation of y                     (the vLLM op the reference calls at
//                                                                     vllm_turing/tailoverlap.py:200; arithmetic of
//                                                                     tests/test_quantfuse.py:45-48, quantfuse.py:18-24)
//
// The reference runs these as three or more kernels (GEMV, LL all-reduce, compiled norm + quant); here one kernel:
//  1. GEMM phase, one of
//     - tcgen05 (default, tc_core.cuh): weights as the MMA's A operand, stream-K over the SMs; the CTA that completes
//       a 128-feature tile finishes it,
//     - dp4a GEMV (VLLM_TURING_FUSED_GEMV=1, M <= 16; gemv_core.cuh): the CTA that finishes a 32-feature row-block.
//  2. The tail, one of
//     - tile owners (default with tcgen05, N <= 8192): the CTA that finished a tile exchanges its partial with the
//       same CTA on every peer (LL words over NVLink), sums the ranks in order, adds the residual and publishes the
//       tile's RMSNorm statistics; two mailbox rounds over all tiles then give every owner the row's 1 / rms and absmax
//       for its features (see "tile-owner tail" below),
//     - row CTAs (VLLM_TURING_DECODE_TAIL=rows, and the GEMV phase): the finisher pushes its values as LL words into
//       every rank's receive slot; token row m is owned by E CTAs (CTA index m * E + g), each for a contiguous 1/E of
//       the row's columns, which poll the LL words of all ranks, sum them in rank order, add the residual, and combine
//       the sum of squares and then the absmax across the E CTAs through a seq-tagged 8-byte mailbox word per CTA
//       (combined in CTA order: identical on every rank, no atomics).
//     Either way: NVLink stores of the finished values, no staging buffer, no flag round trip.
// With world = 1 (no tensor parallelism) the same kernel is the TP1 "fused epilogue without collective".
// All waits are bounded; timeouts land in the communicator's status word.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "comm.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "host_util.h"
#include "tc_core.cuh"
#include "tma_host.h"

namespace vt {

template <typename T>
struct FusedArgs {
    CommView c;
    const int8_t *a, *w;
    const float *sa, *sw;
    int M, N, K, stages, E;
    T *residual;
    const T *norm_w;
    float eps;
    int8_t *q;
    float *scales;
    T *reduced;
    uint64_t pipe_timeout, peer_timeout;
    int tt_two_rounds;   // tile-owner tail: always take the absmax through the second mailbox round
};

template <typename T>
struct LLPushEpi {
    const CommView *c;
    const float *sa, *sw;
    int M, N;
    unsigned seq, p;
    __device__ __forceinline__ void operator()(int rb, const int *tile, int tid) const {
        const int W4 = N >> 2, nwords = M * 8, world = c->world, rank = c->rank;
        for (int idx = tid; idx < nwords * world; idx += GV_CTHREADS) {
            const int k = idx / nwords, wi = idx - k * nwords, m = wi >> 3, j = wi & 7;
            const int col = rb * GV_RB + 4 * j;
            if (col >= N) continue;
            const float sam = sa[m];
            const int *t = tile + m * 32 + 4 * j;
            const float v0 = dequant1(t[0], sam, sw[col]), v1 = dequant1(t[1], sam, sw[col + 1]);
            const float v2 = dequant1(t[2], sam, sw[col + 2]), v3 = dequant1(t[3], sam, sw[col + 3]);
            const int dst = (rank + k) % world;
            ll_store(c->ll_slot(dst, p, rank) + ((size_t)m * W4 + (col >> 2)) * 16, pack2<T>(v0, v1),
                     pack2<T>(v2, v3), seq);
        }
    }
};

__device__ __forceinline__ float block_sum_n(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = red[0];
    for (int i = 1; i < nw; ++i) t += red[i];
    return t;
}
__device__ __forceinline__ float block_max_n(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = red[0];
    for (int i = 1; i < nw; ++i) t = fmaxf(t, red[i]);
    return t;
}

// Publish this CTA's value for (row m, group g, slot) and combine the E values of the row's group in group order.
// Lane q of warp 0 polls group q's mailbox word (all E in flight at once: one L2 round trip, not E in a row); the
// values are then folded in group order 0, 1, .., E - 1, so every CTA of the row and every rank gets identical bits.
__device__ __forceinline__ float group_combine(const CommView &c, int m, int g, int E, int slot, float v, bool is_max,
                                               unsigned seq, uint64_t deadline, float *bcast) {
    unsigned long long *mb = c.mbox();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        if (lane == 0)
            st_volatile8(&mb[((size_t)m * COMM_MBOX_GROUPS + g) * 2 + slot],
                         ((unsigned long long)seq << 32) | (unsigned long long)__float_as_uint(v));
        __syncwarp();
        float val = 0.0f;
        if (lane < E) {
            const unsigned long long *p = &mb[((size_t)m * COMM_MBOX_GROUPS + lane) * 2 + slot];
            unsigned long long x = ld_volatile8(p);
            uint32_t it = 0;
            while ((unsigned)(x >> 32) != seq) {
                if ((++it & 63u) == 0 && globaltimer() > deadline) {
                    report(c.status(), ST_GROUP_TIMEOUT | (unsigned)(m * 64 + lane));
                    break;
                }
                x = ld_volatile8(p);
            }
            val = __uint_as_float((unsigned)(x & 0xffffffffu));
        }
        float t = 0.0f;
        for (int q = 0; q < E; ++q) {
            const float vq = __shfl_sync(0xffffffffu, val, q);
            t = is_max ? fmaxf(t, vq) : (q == 0 ? vq : t + vq);
        }
        if (lane == 0) *bcast = t;
    }
    __syncthreads();
    return *bcast;
}

// Phase 2 of the fused kernel (all threads of every CTA call it once the GEMM phase has pushed this rank's values):
// CTA m * E + g owns columns [w0, w1) (in 4-column LL words) of token row m; the other CTAs return at once. Loads are
// issued in batches (KW words per thread, all ranks' LL words of a batch at once) so a batch costs about one memory
// round trip, not one per word. (KW = 8 measured slower than 4, likely because this code runs once per launch from a
// cold instruction cache, where the larger unrolled body costs more in fetches than the second batch.) E = 1 (the usual case up to two ranks) needs no cross-CTA combine at all.
// smem: free shared memory of at least ceil(N / 4 / E) * 24 bytes; red: 32 floats; bcast: one float. publish_seq:
// the kernel's CTAs read the call number before their first piece and every piece feeds row 0, so CTA 0 publishes
// the next number once row 0 is complete (residual mode only; the caller counts CTAs out otherwise).
template <typename T, int KW>
__device__ __forceinline__ void row_epilogue(const FusedArgs<T> &P, const CommView &c, unsigned seq, unsigned p,
                                             unsigned char *smem, float *red, float *bcast, bool publish_seq) {
    // every field in registers: the LL polls are asm with a memory clobber, after which values read through pointers
    // (the kernel's parameter block included) would be read again
    const int M = P.M, N = P.N, E = P.E, W4 = N >> 2, world = c.world;
    if ((int)blockIdx.x >= M * E) return;
    const int m = blockIdx.x / E, g = blockIdx.x - m * E;
    const int w0 = (int)((long long)W4 * g / E), w1 = (int)((long long)W4 * (g + 1) / E);
    const int nw = w1 - w0, nt = blockDim.x, tid = threadIdx.x;
    T *const residual = P.residual, *const reduced = P.reduced;
    const T *const norm_w = P.norm_w;
    int8_t *const qout = P.q;
    float *const scales = P.scales;
    const float eps = P.eps;
    unsigned *const status = c.status();
    const char *src[COMM_MAX_RANKS];   // rank r's LL words for this CTA's columns of row m
#pragma unroll
    for (int r = 0; r < COMM_MAX_RANKS; ++r)
        src[r] = r < world ? c.ll_slot(c.rank, p, r) + ((size_t)m * W4 + w0) * 16 : nullptr;
    float *hbuf = reinterpret_cast<float *>(smem);          // [nw * 4] the new residual, then the normalised row
    uint2 *nbuf = reinterpret_cast<uint2 *>(hbuf + 4 * nw);  // [nw] norm weight words, loaded with the residual
    const uint64_t deadline = globaltimer() + P.peer_timeout;
    bool dead = false;
    float ss = 0.0f;
    for (int b = 0; b < nw; b += nt * KW) {
        uint2 ru[KW], wv[KW];
        if (residual) {   // this batch's residual and norm weight: independent of the peers, in flight with the polls
#pragma unroll
            for (int k = 0; k < KW; ++k) {
                const int i = b + tid + k * nt;
                if (i < nw) {
                    ru[k] = *reinterpret_cast<const uint2 *>(residual + (size_t)m * N + (size_t)(w0 + i) * 4);
                    wv[k] = *reinterpret_cast<const uint2 *>(norm_w + (size_t)(w0 + i) * 4);
                }
            }
        }
        float s[KW][4];
#pragma unroll
        for (int r = 0; r < COMM_MAX_RANKS; ++r) {   // ranks in order: the float sums are identical on every rank
            if (r >= world) break;
            const char *slot = src[r];
            uint4 v[KW];
#pragma unroll
            for (int k = 0; k < KW; ++k) {
                const int i = b + tid + k * nt;
                if (i < nw) v[k] = ld_volatile16(slot + (size_t)i * 16);
            }
#pragma unroll
            for (int k = 0; k < KW; ++k) {
                const int i = b + tid + k * nt;
                if (i >= nw) continue;
                uint32_t it = 0;
                while (!dead && (v[k].y != seq || v[k].w != seq)) {
                    if ((++it & 255u) == 0 && globaltimer() > deadline) {
                        report(status, ST_PEER_TIMEOUT | 0x500u | (unsigned)r);
                        dead = true;
                        break;
                    }
                    v[k] = ld_volatile16(slot + (size_t)i * 16);
                }
                const float2 x0 = unpack2<T>(v[k].x), x1 = unpack2<T>(v[k].z);
                if (r == 0) {
                    s[k][0] = x0.x; s[k][1] = x0.y; s[k][2] = x1.x; s[k][3] = x1.y;
                } else {
                    s[k][0] += x0.x; s[k][1] += x0.y; s[k][2] += x1.x; s[k][3] += x1.y;
                }
            }
        }
#pragma unroll
        for (int k = 0; k < KW; ++k) {
            const int i = b + tid + k * nt;
            if (i >= nw) continue;
            const size_t e0 = (size_t)m * N + (size_t)(w0 + i) * 4;
            if (reduced)
                *reinterpret_cast<uint2 *>(reduced + e0) =
                    make_uint2(pack2<T>(s[k][0], s[k][1]), pack2<T>(s[k][2], s[k][3]));
            if (residual) {
                const float2 r0 = unpack2<T>(ru[k].x), r1 = unpack2<T>(ru[k].y);
                const float h0 = rnd<T>(rnd<T>(s[k][0]) + r0.x), h1 = rnd<T>(rnd<T>(s[k][1]) + r0.y);
                const float h2 = rnd<T>(rnd<T>(s[k][2]) + r1.x), h3 = rnd<T>(rnd<T>(s[k][3]) + r1.y);
                *reinterpret_cast<uint2 *>(residual + e0) = make_uint2(pack2<T>(h0, h1), pack2<T>(h2, h3));
                nbuf[i] = wv[k];
                hbuf[4 * i] = h0;
                hbuf[4 * i + 1] = h1;
                hbuf[4 * i + 2] = h2;
                hbuf[4 * i + 3] = h3;
                ss += h0 * h0 + h1 * h1 + h2 * h2 + h3 * h3;
            }
        }
    }
    if (!residual) return;
    ss = block_sum_n(ss, red);
    const float tot = E > 1 ? group_combine(c, m, g, E, 0, ss, false, seq, deadline, bcast) : ss;
    if (publish_seq && blockIdx.x == 0 && tid == 0) {
        // Row 0 is complete across all its CTAs: every tile was finished and pushed, so every CTA of the grid has
        // read this call's number -- publish it now, for the next call on the communicator (the kernel boundary
        // makes it visible), instead of counting CTAs out at the end.
        *reinterpret_cast<volatile unsigned *>(c.seq_ptr()) = seq;
    }
    const float rs = __frsqrt_rn(__fdiv_rn(tot, (float)N) + eps);
    float amax = 0.0f;
    for (int i = tid; i < nw; i += nt) {
        const uint2 wu = nbuf[i];
        const float2 wa = unpack2<T>(wu.x), wb = unpack2<T>(wu.y);
        const float y0 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i], rs), wa.x));
        const float y1 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i + 1], rs), wa.y));
        const float y2 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i + 2], rs), wb.x));
        const float y3 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i + 3], rs), wb.y));
        hbuf[4 * i] = y0;
        hbuf[4 * i + 1] = y1;
        hbuf[4 * i + 2] = y2;
        hbuf[4 * i + 3] = y3;
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(y0), fabsf(y1)), fmaxf(fabsf(y2), fabsf(y3))));
    }
    amax = block_max_n(amax, red);
    if (E > 1) amax = group_combine(c, m, g, E, 1, amax, true, seq, deadline, bcast);
    const float inv = quant_inv(amax);
    if (g == 0 && tid == 0) scales[m] = __fdiv_rn(amax, 127.0f);
    for (int i = tid; i < nw; i += nt) {
        *reinterpret_cast<char4 *>(qout + (size_t)m * N + (size_t)(w0 + i) * 4) =
            make_char4(quant1(hbuf[4 * i], inv), quant1(hbuf[4 * i + 1], inv), quant1(hbuf[4 * i + 2], inv),
                       quant1(hbuf[4 * i + 3], inv));
    }
}

// CTAs per token row in the row epilogue: one up to two ranks (no cross-CTA combine); more ranks bring world x more
// LL words per row, shared by world / 2 CTAs (at most the mailbox's groups and one CTA per row per SM).
inline int row_ctas(int world, int M, int grid) {
    static int forced = -1;   // VLLM_TURING_ROW_CTAS: a fixed E (tests run the multi-CTA combine on one GPU)
    if (forced < 0) {
        const char *e = getenv("VLLM_TURING_ROW_CTAS");
        forced = e ? atoi(e) : 0;
    }
    int E = forced > 0 ? forced : world / 2;
    if (E < 1) E = 1;
    if (E > COMM_MBOX_GROUPS) E = COMM_MBOX_GROUPS;
    while (E > 1 && E * M > grid) --E;
    return E;
}

template <typename T, int MT>
__global__ void __launch_bounds__(GV_THREADS, 1)
    tp_row_linear_kernel(const __grid_constant__ CUtensorMap wmap, FusedArgs<T> P) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ unsigned s_seq;
    __shared__ float red[32];
    __shared__ float bcast;
    const CommView &c = P.c;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t t0 = globaltimer();
    LLPushEpi<T> push{&c, P.sa, P.sw, P.M, P.N, seq, p};
    gemv_phase<MT>(P.a, &wmap, P.M, P.N, P.K, c.scratch(), c.tickets(), smem, P.stages, t0 + P.pipe_timeout,
                   c.status(), push);
    __syncthreads();

    row_epilogue<T, 4>(P, c, seq, p, smem + GV_HDR, red, &bcast, false);   // the GEMV ring is free now
    comm_end(c, seq);
}

// tcgen05 finisher of the fused kernel: thread = output feature n of a finished 128-feature tile; dequantises its
// accumulators ((acc * sa[m]) * sw[n], the GEMV's order) and lane 4j of each warp pushes the LL word of features
// n .. n + 3 (gathered by shuffles) to every rank's receive slot.
template <typename T, int BN>
struct TcLLPushEpi {
    static constexpr int kSmemFloats = 64;
    struct Prep {
        float swn;
    };
    const CommView *c;
    const float *sa, *sw;
    int M, N;
    unsigned *s_seq;   // shared: this call's sequence number, read after pdl_wait
    float *sa_sm;      // shared: the token scales
    // registers from post_start: the call's sequence number and this rank's LL slot in every rank's region, in push
    // order (own rank first). The pushes are asm with a memory clobber; values kept in registers are not re-read.
    unsigned seq;
    int world;
    char *dst[COMM_MAX_RANKS];
    __device__ __forceinline__ void on_start(const TcArgs &, float *sm) {
        sa_sm = sm;
        const int t = threadIdx.x - TC_EPI_LEAD;
        if (t < M) sm[t] = sa[t];
        if (t == 0) *s_seq = *reinterpret_cast<volatile unsigned *>(c->seq_ptr()) + 1u;
    }
    __device__ __forceinline__ void post_start() {
        seq = *s_seq;
        world = c->world;
        const int rank = c->rank;
#pragma unroll
        for (int k = 0; k < COMM_MAX_RANKS; ++k)
            dst[k] = k < world ? c->ll_slot((rank + k) % world, seq & 1u, rank) : nullptr;
    }
    __device__ __forceinline__ Prep prep(const TcArgs &, int n) const { return Prep{n < N ? sw[n] : 0.0f}; }
    __device__ __forceinline__ void operator()(const TcArgs &, int n, bool nok, const int (&acc)[BN],
                                               const Prep &pr) const {
        const int W4 = N >> 2, Mr = M, nw = world;
        const unsigned sq = seq;
        const int lane = threadIdx.x & 31;
        float v[BN];
#pragma unroll
        for (int m = 0; m < BN; ++m) v[m] = (m < Mr && nok) ? dequant1(acc[m], sa_sm[m], pr.swn) : 0.0f;
#pragma unroll
        for (int m = 0; m < BN; ++m) {
            if (m >= Mr) break;   // M is uniform: the whole warp leaves together
            const float v1 = __shfl_down_sync(0xffffffffu, v[m], 1);
            const float v2 = __shfl_down_sync(0xffffffffu, v[m], 2);
            const float v3 = __shfl_down_sync(0xffffffffu, v[m], 3);
            if ((lane & 3) == 0 && nok) {   // n % 4 == 0 here and N % 4 == 0: features n .. n + 3 all exist
                const uint32_t lo = pack2<T>(v[m], v1), hi = pack2<T>(v2, v3);
                const size_t off = ((size_t)m * W4 + (n >> 2)) * 16;
#pragma unroll
                for (int k = 0; k < COMM_MAX_RANKS; ++k)
                    if (k < nw) ll_store(dst[k] + off, lo, hi, sq);
            }
        }
    }
};

// Launched with programmatic dependent launch: the call number is read after pdl_wait (by the epilogue lead in
// fin.on_start), not at kernel entry, since the previous call on this communicator may still be finishing then.
template <typename T, int BN, int KBS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tp_row_linear_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                            TcArgs G, FusedArgs<T> P) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ unsigned s_seq;
    __shared__ float red[32];
    __shared__ float bcast;
    const CommView &c = P.c;
    TcLLPushEpi<T, BN> push{&c, P.sa, P.sw, P.M, P.N, &s_seq, nullptr, 0u, 0, {}};
    tc_phase<T, BN, true, KBS>(&tmap_w, &tmap_a, G, smem_raw, push);   // ends with __syncthreads
    const unsigned seq = s_seq, p = seq & 1u;
    const bool publish = P.residual != nullptr;   // residual mode: row 0's CTA publishes the call number
    row_epilogue<T, 4>(P, c, seq, p, tc_align1024(smem_raw), red, &bcast, publish);   // the stage ring is free now
    if (!publish) comm_end(c, seq);
}

// ---- tile-owner tail (the default decode tail of the tcgen05 phase) ------------------------------------------------
// The CTA that finishes a 128-feature tile (its head, or the CTA holding it whole) is that tile's owner for the rest of
// the call: thread = feature n holds the dequantised partial of all M token rows in registers, so the all-reduce, the
// residual add and the tile's share of the RMSNorm statistics run right there, spread over the N / 128 owners instead
// of a few CTAs per token row.
//  1. finisher (in the GEMM phase): world > 1: push the partial as 16-byte LL words (rows 4i .. 4i + 3 of feature n)
//     into the same owner's slot on every peer (the stream-K partition is identical on every rank), then poll the
//     peers' words for the same features, all peers in flight at once, and sum the ranks in order 0 .. world - 1
//     (own partial from registers). Write `reduced`; add the residual (loaded before the MMAs completed) and write it
//     back; the tile's sum of squares per token row goes into the tile mailbox (seq-tagged word per tile and row).
//  2. after the GEMM phase: gather every tile's sums of squares (one poll round), fold them in tile order (identical on
//     every CTA and rank), normalise the owned features, publish the tile's absmax per row, gather all tiles' maxima,
//     quantise. The owner of tile 0 writes the scales and publishes the call number.
// Per call after the weight stream: split-K collection, [the NVLink exchange], two mailbox rounds -- with the work of
// each round spread over the tile owners.
// Products |h w| within this factor of a row's largest are near-ties: a normalised value of such a product may round
// above the largest one's (two fp32 roundings, 2^-24 each, then the 16-bit rounding); farther ones cannot.
constexpr float TT_NEAR = 1.0f - 1.0f / 524288.0f;   // 1 - 2^-19, exact in fp32

template <typename T> __device__ __forceinline__ unsigned short t2bits(float x) {
    const T v = f2t<T>(x);
    return *reinterpret_cast<const unsigned short *>(&v);
}
template <typename T> __device__ __forceinline__ float bits2f(uint32_t b) {
    const unsigned short u = (unsigned short)b;
    return t2f<T>(*reinterpret_cast<const T *>(&u));
}

template <typename T, int BN>
struct TcTileTailEpi {
    // shared floats: [0, 32) token scales, [32, 160) per-warp sums of squares [4][32], [160, 416) per-warp largest
    // products as 64-bit keys [4][32], [416, 544) per-warp near-tie counts [4][32], [544, 576) the |h|, |w| pair of
    // each row's largest product, [576, 608) per-row 1 / rms, [608, 640) per-row absmax, [640, 672) per-row flags,
    // [672, 674) ints: owned-tile count, the owned tile
    static constexpr int kSmemFloats = 704;
    __device__ __forceinline__ static int *owned_of(float *smp) { return reinterpret_cast<int *>(smp + 672); }
    struct Prep {
        float swn, wn;
        float res[BN];
    };
    const FusedArgs<T> *F;
    unsigned *s_seq;
    float *sm;
    unsigned seq;
    int M, N, world, rank;
    __device__ __forceinline__ int *owned() const { return owned_of(sm); }
    __device__ __forceinline__ void on_start(const TcArgs &, float *smp) {
        sm = smp;
        const int t = threadIdx.x - TC_EPI_LEAD;
        if (t < F->M) sm[t] = F->sa[t];
        if (t == 0) {
            *s_seq = *reinterpret_cast<volatile unsigned *>(F->c.seq_ptr()) + 1u;
            owned()[0] = 0;
        }
    }
    __device__ __forceinline__ void post_start() {
        seq = *s_seq;
        M = F->M;
        N = F->N;
        world = F->c.world;
        rank = F->c.rank;
    }
    __device__ __forceinline__ Prep prep(const TcArgs &, int n) const {
        Prep r;
        const bool ok = n < N;
        r.swn = ok ? F->sw[n] : 0.0f;
        r.wn = (ok && F->residual) ? t2f<T>(F->norm_w[n]) : 0.0f;
        const T *res = F->residual;
#pragma unroll
        for (int m = 0; m < BN; ++m) r.res[m] = (res && ok && m < M) ? t2f<T>(res[(size_t)m * N + n]) : 0.0f;
        return r;
    }
    __device__ __forceinline__ void operator()(const TcArgs &, int n, bool nok, const int (&acc)[BN],
                                               const Prep &pr) const {
        const int Mr = M, Nr = N, nw = world, rk = rank, nq = (Mr + 3) >> 2;
        const unsigned sq = seq, par = sq & 1u;
        float s[BN];
#pragma unroll
        for (int m = 0; m < BN; ++m) s[m] = (m < Mr && nok) ? rnd<T>(dequant1(acc[m], sm[m], pr.swn)) : 0.0f;
        if (nw > 1) {
            if (nok) {
#pragma unroll
                for (int k = 1; k < COMM_MAX_RANKS; ++k) {
                    if (k >= nw) break;
                    int dst = rk + k;
                    if (dst >= nw) dst -= nw;
                    char *base = F->c.ll_slot(dst, par, rk) + (size_t)n * 16;
#pragma unroll
                    for (int i = 0; i < BN / 4; ++i) {
                        if (i >= nq) break;
                        ll_store(base + (size_t)i * Nr * 16, pack2<T>(s[4 * i], s[4 * i + 1]),
                                 pack2<T>(s[4 * i + 2], s[4 * i + 3]), sq);
                    }
                }
            }
            const uint64_t deadline = globaltimer() + F->peer_timeout;
            bool dead = false;
            // eight token rows (two words per peer) at a time; a poll round re-loads every peer's words and tests all
            // tags (a tight loop), so the exchange ends one round trip after the last word lands
#pragma unroll
            for (int i0 = 0; i0 < BN / 4; i0 += 2) {
                if (i0 >= nq) break;
                uint4 v[COMM_MAX_RANKS][2];
                const bool two = i0 + 1 < nq;
                uint32_t it = 0;
                while (nok && !dead) {
#pragma unroll
                    for (int r = 0; r < COMM_MAX_RANKS; ++r) {
                        if (r >= nw || r == rk) continue;
                        const char *src = F->c.ll_slot(rk, par, r) + ((size_t)i0 * Nr + n) * 16;
                        v[r][0] = ld_volatile16(src);
                        if (two) v[r][1] = ld_volatile16(src + (size_t)Nr * 16);
                    }
                    bool ready = true;
#pragma unroll
                    for (int r = 0; r < COMM_MAX_RANKS; ++r) {
                        if (r >= nw || r == rk) continue;
                        ready = ready && v[r][0].y == sq && v[r][0].w == sq;
                        if (two) ready = ready && v[r][1].y == sq && v[r][1].w == sq;
                    }
                    if (ready) break;
                    if ((++it & 255u) == 0 && globaltimer() > deadline) {
                        report(F->c.status(), ST_PEER_TIMEOUT | 0x500u | (unsigned)(rk == 0 ? 1 : 0));
                        dead = true;
                    }
                }
                // rank-ordered float sum, own partial from registers (rank 0's value first, as the oracle)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int m = 4 * (i0 + j) + e;
                        if (m >= BN) continue;
                        float t = 0.0f;
#pragma unroll
                        for (int r = 0; r < COMM_MAX_RANKS; ++r) {
                            if (r >= nw) break;
                            float x = s[m];
                            if (r != rk) {
                                const uint32_t w32 = (e < 2) ? v[r][j].x : v[r][j].z;
                                const float2 f = unpack2<T>(w32);
                                x = (e & 1) ? f.y : f.x;
                            }
                            t = (r == 0) ? x : t + x;
                        }
                        if (i0 + j < nq) s[m] = t;
                    }
                }
            }
        }
        T *const red = F->reduced;
        if (red && nok) {
#pragma unroll
            for (int m = 0; m < BN; ++m)
                if (m < Mr) red[(size_t)m * Nr + n] = f2t<T>(s[m]);
        }
        T *const res = F->residual;
        if (!res) return;
        // The tile's statistics per token row, published in one 16-byte LL word: the sum of squares of the new
        // residual h over the tile's features, and for the absmax of the normalised row y = rnd(rnd(h * rs) * w):
        // the |h|, |w| pair of the largest product |h w| (exact in fp32; the smallest feature index among equal ones)
        // and a flag when a second feature's product lies within 2^-19 of it. |y| grows with |h w| except for
        // products that close, so every owner can derive the row's absmax exactly from these pairs; a flagged
        // candidate sends the call through a second mailbox round instead.
        const int t = threadIdx.x - TC_EPI_LEAD, q = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
        float *part = sm + 32;
        unsigned long long *pkey = reinterpret_cast<unsigned long long *>(sm + 160);
        int *pcnt = reinterpret_cast<int *>(sm + 416);
        uint32_t *phw = reinterpret_cast<uint32_t *>(sm + 544);
        const float aw = fabsf(pr.wn);
#pragma unroll
        for (int m = 0; m < BN; ++m) {
            if (m >= Mr) break;   // uniform
            const float h = rnd<T>(rnd<T>(s[m]) + pr.res[m]);
            s[m] = h;
            if (nok) res[(size_t)m * Nr + n] = f2t<T>(h);
            float x = nok ? h * h : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
            const float pm = nok ? fabsf(h) * aw : 0.0f;
            unsigned long long key = ((unsigned long long)__float_as_uint(pm) << 32) | (0xffffffffu - (unsigned)n);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                key = k2 > key ? k2 : key;
            }
            if (lane == 0) {
                part[q * 32 + m] = x;
                pkey[q * 32 + m] = key;
            }
        }
        named_sync(TC_EPI_BAR, 128);
#pragma unroll
        for (int m = 0; m < BN; ++m) {
            if (m >= Mr) break;
            unsigned long long k = pkey[m];
#pragma unroll
            for (int j = 1; j < 4; ++j) k = pkey[j * 32 + m] > k ? pkey[j * 32 + m] : k;
            const float pmax = __uint_as_float((unsigned)(k >> 32));
            const float pm = nok ? fabsf(s[m]) * aw : 0.0f;
            if (nok && (unsigned)n == 0xffffffffu - (unsigned)k)
                phw[m] = (uint32_t)t2bits<T>(fabsf(s[m])) | ((uint32_t)t2bits<T>(aw) << 16);
            const unsigned close = __ballot_sync(0xffffffffu, nok && pm >= pmax * TT_NEAR);
            if (lane == 0) pcnt[q * 32 + m] = __popc(close);
        }
        named_sync(TC_EPI_BAR, 128);
        const int ta = n >> 7;
        if (t < Mr) {
            const float x = ((part[t] + part[32 + t]) + part[64 + t]) + part[96 + t];
            const int cnt = pcnt[t] + pcnt[32 + t] + pcnt[64 + t] + pcnt[96 + t];
            ll_store(F->c.tm_stat(ta, t), __float_as_uint(x), phw[t] | (cnt >= 2 ? 0x80000000u : 0u), sq);
        }
        if (t == 0) {   // at most one tile per CTA (the launch checks it)
            int *o = owned();
            o[0] = 1;
            o[1] = ta;
        }
    }
};

// Gathers every tile's statistics word for the M token rows: sums of squares into bss[m * 64 + tile], the pair words
// into bhw (all threads of the CTA). A poll round re-loads all of a thread's words and tests their tags (a tight loop),
// so the gather ends one round trip after the last word lands; the words are stored once all have arrived.
constexpr int TT_GMAX = (COMM_TMBOX_TILES * COMM_MBOX_ROWS + TC_THREADS - 1) / TC_THREADS;
__device__ __forceinline__ void tt_gather_stats(const CommView &c, int NT, int M, unsigned seq, float *bss,
                                                uint32_t *bhw, uint64_t deadline) {
    const int total = NT * M;
    const uint4 *ptr[TT_GMAX];
    int dst[TT_GMAX];
#pragma unroll
    for (int i = 0; i < TT_GMAX; ++i) {
        const int j = threadIdx.x + i * TC_THREADS, m = j / NT, tile = j - m * NT;
        ptr[i] = j < total ? c.tm_stat(tile, m) : nullptr;
        dst[i] = m * COMM_TMBOX_TILES + tile;
    }
    uint4 v[TT_GMAX];
    uint32_t it = 0;
    while (true) {
#pragma unroll
        for (int i = 0; i < TT_GMAX; ++i)
            if (ptr[i]) v[i] = ld_volatile16(ptr[i]);
        bool ready = true;
#pragma unroll
        for (int i = 0; i < TT_GMAX; ++i)
            if (ptr[i]) ready = ready && v[i].y == seq && v[i].w == seq;
        if (ready) break;
        if ((++it & 63u) == 0 && globaltimer() > deadline) {
            report(c.status(), ST_GROUP_TIMEOUT | 0x700u);
            break;
        }
    }
#pragma unroll
    for (int i = 0; i < TT_GMAX; ++i) {
        if (!ptr[i]) continue;
        bss[dst[i]] = __uint_as_float(v[i].x);
        bhw[dst[i]] = v[i].z;
    }
}

// The same for the absmax words of the second round (buf[m * 64 + tile]).
__device__ __forceinline__ void tt_gather_amax(const CommView &c, int NT, int M, unsigned seq, float *buf,
                                               uint64_t deadline) {
    const int total = NT * M;
    const unsigned long long *ptr[TT_GMAX];
    int dst[TT_GMAX];
#pragma unroll
    for (int i = 0; i < TT_GMAX; ++i) {
        const int j = threadIdx.x + i * TC_THREADS, m = j / NT, tile = j - m * NT;
        ptr[i] = j < total ? c.tm_amax(tile, m) : nullptr;
        dst[i] = m * COMM_TMBOX_TILES + tile;
    }
    unsigned long long v[TT_GMAX];
    uint32_t it = 0;
    while (true) {
#pragma unroll
        for (int i = 0; i < TT_GMAX; ++i)
            if (ptr[i]) v[i] = ld_volatile8(ptr[i]);
        bool ready = true;
#pragma unroll
        for (int i = 0; i < TT_GMAX; ++i)
            if (ptr[i]) ready = ready && (unsigned)(v[i] >> 32) == seq;
        if (ready) break;
        if ((++it & 63u) == 0 && globaltimer() > deadline) {
            report(c.status(), ST_GROUP_TIMEOUT | 0x701u);
            break;
        }
    }
#pragma unroll
    for (int i = 0; i < TT_GMAX; ++i)
        if (ptr[i]) buf[dst[i]] = __uint_as_float((unsigned)v[i]);
}

// Phase 2 of the tile-owner tail: every thread of the CTA calls it after the GEMM phase (residual mode). The launch
// guarantees that a CTA owns at most one tile (its stream-K range is shorter than a tile's K range, or one unit).
template <typename T, int BN>
__device__ __forceinline__ void tile_tail_post(const FusedArgs<T> &P, unsigned seq, float *sm, float *buf) {
    using Epi = TcTileTailEpi<T, BN>;
    const int *own = Epi::owned_of(sm);
    if (own[0] == 0) return;   // uniform: this CTA finished no tile
    const int ta = own[1];
    const CommView &c = P.c;
    const int M = P.M, N = P.N, NT = (N + TC_BM - 1) / TC_BM;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    const bool epi = tid >= TC_EPI_LEAD;
    // epilogue thread -> feature of the tile as in the GEMM phase (TMEM lane quarter warp % 4): each thread re-reads
    // the residual values it wrote there
    const int q = warp & 3, t = tid - TC_EPI_LEAD;
    const int n = ta * TC_BM + q * 32 + lane;
    const bool nok = epi && n < N;
    T *const res = P.residual;
    float *part = sm + 32, *rs = sm + 576, *amax = sm + 608;
    int *fb = reinterpret_cast<int *>(sm + 640);
    float *bss = buf;
    uint32_t *bhw = reinterpret_cast<uint32_t *>(buf + COMM_MBOX_ROWS * COMM_TMBOX_TILES);
    float *bam = buf + 2 * COMM_MBOX_ROWS * COMM_TMBOX_TILES;
    const uint64_t deadline = globaltimer() + P.peer_timeout;
    // the new residual and the norm weight: loads in flight during the gather
    float y[BN];
#pragma unroll
    for (int m = 0; m < BN; ++m) y[m] = (nok && m < M) ? t2f<T>(res[(size_t)m * N + n]) : 0.0f;
    const float wn = nok ? t2f<T>(P.norm_w[n]) : 0.0f;
    tt_gather_stats(c, NT, M, seq, bss, bhw, deadline);
    __syncthreads();
    // per token row (one warp each): 1 / rms from the sums of squares folded in tile order, and the absmax from the
    // candidate pairs -- exact unless a candidate is flagged (then fb[m] = 1 and the second round decides)
    for (int m = warp; m < M; m += nwarps) {
        const float *ss = bss + m * COMM_TMBOX_TILES;
        const uint32_t *hw = bhw + m * COMM_TMBOX_TILES;
        float x = lane < NT ? ss[lane] : 0.0f;
        if (lane + 32 < NT) x += ss[lane + 32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        const float r = __frsqrt_rn(__fdiv_rn(x, (float)N) + P.eps);
        float hh[2], ww[2], pp[2];
        bool fl[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int tile = lane + 32 * k;
            const uint32_t u = tile < NT ? hw[tile] : 0u;
            hh[k] = bits2f<T>(u & 0xffffu);
            ww[k] = bits2f<T>((u >> 16) & 0x7fffu);
            fl[k] = (u >> 31) != 0;
            pp[k] = tile < NT ? hh[k] * ww[k] : -1.0f;
        }
        float pmx = fmaxf(pp[0], pp[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pmx = fmaxf(pmx, __shfl_xor_sync(0xffffffffu, pmx, o));
        float a = 0.0f;
        bool flagged = false;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (pp[k] >= pmx * TT_NEAR) {
                a = fmaxf(a, rnd<T>(__fmul_rn(__fmul_rn(hh[k], r), ww[k])));
                flagged |= fl[k];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        flagged = __any_sync(0xffffffffu, flagged);
        if (lane == 0) {
            rs[m] = r;
            amax[m] = a;
            fb[m] = flagged ? 1 : 0;
        }
    }
    __syncthreads();
    // Every tile was finished, so every CTA of the grid has read this call's number: publish it for the next call.
    if (tid == 0 && ta == 0) *reinterpret_cast<volatile unsigned *>(c.seq_ptr()) = seq;
    bool second = P.tt_two_rounds != 0;   // uniform: every CTA decides from the same gathered words
    for (int m = 0; m < M; ++m) second |= fb[m] != 0;
#pragma unroll
    for (int m = 0; m < BN; ++m) {
        if (m >= M) break;
        y[m] = nok ? rnd<T>(__fmul_rn(__fmul_rn(y[m], rs[m]), wn)) : 0.0f;
    }
    if (second) {   // the tile's absmax per row, one more mailbox round over all tiles
        if (epi) {
#pragma unroll
            for (int m = 0; m < BN; ++m) {
                if (m >= M) break;
                float a = fabsf(y[m]);
#pragma unroll
                for (int k = 16; k > 0; k >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, k));
                if (lane == 0) part[q * 32 + m] = a;
            }
        }
        __syncthreads();
        if (epi && t < M) {
            const float a = fmaxf(fmaxf(part[t], part[32 + t]), fmaxf(part[64 + t], part[96 + t]));
            st_volatile8(c.tm_amax(ta, t), ((unsigned long long)seq << 32) | __float_as_uint(a));
        }
        tt_gather_amax(c, NT, M, seq, bam, deadline);
        __syncthreads();
        for (int m = warp; m < M; m += nwarps) {   // max: the same in any order
            float a = lane < NT ? bam[m * COMM_TMBOX_TILES + lane] : 0.0f;
            if (lane + 32 < NT) a = fmaxf(a, bam[m * COMM_TMBOX_TILES + lane + 32]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            if (lane == 0) amax[m] = a;
        }
        __syncthreads();
    }
    if (ta == 0 && tid < M) P.scales[tid] = __fdiv_rn(amax[tid], 127.0f);
    if (!nok) return;
    int8_t *const qo = P.q;
#pragma unroll
    for (int m = 0; m < BN; ++m) {
        if (m >= M) break;
        qo[(size_t)m * N + n] = quant1(y[m], quant_inv(amax[m]));
    }
}

// The fused kernel with the tile-owner tail. Launched with programmatic dependent launch (see tp_row_linear_tc_kernel).
template <typename T, int BN, int KBS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tp_row_linear_tt_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                            TcArgs G, FusedArgs<T> P) {
    using Lay = TcLayout<BN, KBS>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ unsigned s_seq;
    TcTileTailEpi<T, BN> fin{&P, &s_seq, nullptr, 0u, 0, 0, 0, 0};
    tc_phase<T, BN, true, KBS>(&tmap_w, &tmap_a, G, smem_raw, fin);   // ends with __syncthreads
    const unsigned seq = s_seq;
    unsigned char *ring = tc_align1024(smem_raw);
    float *sm = reinterpret_cast<float *>(ring + (size_t)G.stages * Lay::STAGE + Lay::BAR_BYTES);
    if (P.residual)
        tile_tail_post<T, BN>(P, seq, sm, reinterpret_cast<float *>(ring));   // the stage ring is free now
    else
        comm_end(P.c, seq);
}

// VLLM_TURING_TT_ROUNDS=2 makes the tile-owner tail take every row's absmax through the second mailbox round (the
// path a near-tie takes; tests compare both).
static int tt_two_rounds() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_TT_ROUNDS");
        v = (e && atoi(e) == 2) ? 1 : 0;
    }
    return v;
}

// VLLM_TURING_DECODE_TAIL=rows selects the row-CTA epilogue (tp_row_linear_tc_kernel) instead of the tile owners.
static bool decode_tail_rows() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_DECODE_TAIL");
        v = (e && strcmp(e, "rows") == 0) ? 1 : 0;
    }
    return v != 0;
}

// Grid of the tile-owner kernel: one CTA per SM; with few K blocks per tile (a tensor-parallel rank's share of
// K, nkb <= 34), two CTAs per tile instead: every tile then has one contributor, whose split-K hand-off is cheaper
// than collecting three or four, while the weight stream per CTA stays short. Measured with a per-CTA timer, M = 5:
// K = 2176 12.5 -> 11.8 us, K = 4352 14.7 -> 13.9 us; at K = 17408 one CTA per SM stays faster (24.6 vs 25.1 us: a
// CTA streams at most ~60 GB/s with its ring in flight, so 80 CTAs cannot carry 89 MB as fast as 148).
inline long long tt_grid(int dev, int NT, int nkb) {
    const long long units = (long long)NT * nkb, sms = num_sms(dev);
    if (nkb <= 34 && nkb >= 2 && 2LL * NT <= sms) return 2LL * NT;
    return sms < units ? sms : units;
}

// The tile-owner tail's limits: N / 128 tiles in the mailbox, each peer's LL words ((M + 3) / 4 x 16 bytes per
// feature) in one LL slot, and at most one tile owned per CTA: every CTA's stream-K range (ceil(units / grid) K
// blocks) shorter than a tile's K blocks, or a single unit.
inline bool tile_tail_fits(const CommView &c, int M, int N, int K) {
    const int NT = (N + TC_BM - 1) / TC_BM, nkb = (K + TC_BK - 1) / TC_BK;
    if (NT > COMM_TMBOX_TILES) return false;
    const int dev = cur_device();
    if (dev < 0) return false;
    const long long units = (long long)NT * nkb, g = tt_grid(dev, NT, nkb);
    const long long L = (units + g - 1) / g;
    if (!(L < nkb || L == 1)) return false;
    return c.world == 1 || (size_t)((M + 3) / 4) * 16 * (size_t)N <= c.L.ll_slot;
}

template <typename T, int BN, int KBS>
static int launch_fused_tt(FusedArgs<T> P, cudaStream_t s) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    using Epi = TcTileTailEpi<T, BN>;
    CUtensorMap mw, ma;
    if (!tc_make_map(&mw, P.w, P.N, P.K, TC_BM) || !tc_make_map(&ma, P.a, P.M, P.K, BN)) return VT_EARG;
    TcArgs G{};
    tc_decode_args(G, P.M, P.N, P.K);
    G.sa = P.sa;
    G.sw = P.sw;
    G.sa_rows = 1;
    G.sw_rows = 1;
    char *local = P.c.base[P.c.rank];
    G.slots = reinterpret_cast<uint4 *>(local + P.c.L.scratch_off);
    G.status = reinterpret_cast<unsigned *>(local + 128);
    G.timeout_ns = P.pipe_timeout;
    const int stages = tc_stages<BN, KBS>(dev, Epi::kSmemFloats, decode_smem_budget());
    if (stages < 2) return VT_EARG;
    G.stages = stages;
    const int smem = tc_smem_bytes<BN, KBS>(stages, Epi::kSmemFloats);
    static bool attr_set[VT_MAX_DEV] = {false};
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(tp_row_linear_tt_kernel<T, BN, KBS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
            return (int)cudaGetLastError();
        attr_set[dev] = true;
    }
    const int g = (int)tt_grid(dev, G.n_tiles_a, G.nkb);
    if (tc_decode_slot_bytes(P.M, g) > P.c.L.scratch_bytes) return VT_EARG;
    P.tt_two_rounds = tt_two_rounds();
    // the post phase's three gather buffers ([32][64] words each) in the stage ring
    if ((size_t)3 * COMM_MBOX_ROWS * COMM_TMBOX_TILES * 4 > (size_t)stages * TcLayout<BN, KBS>::STAGE) return VT_EARG;
    return launch_k(tp_row_linear_tt_kernel<T, BN, KBS>, dim3(g), dim3(TC_THREADS), smem, s, true, mw, ma, G, P);
}

template <typename T, int BN, int KBS>
static int launch_fused_tc(FusedArgs<T> P, cudaStream_t s) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    CUtensorMap mw, ma;
    if (!tc_make_map(&mw, P.w, P.N, P.K, TC_BM) || !tc_make_map(&ma, P.a, P.M, P.K, BN)) return VT_EARG;
    TcArgs G{};
    tc_decode_args(G, P.M, P.N, P.K);
    G.sa = P.sa;
    G.sw = P.sw;
    G.sa_rows = 1;
    G.sw_rows = 1;
    char *local = P.c.base[P.c.rank];
    G.slots = reinterpret_cast<uint4 *>(local + P.c.L.scratch_off);
    G.status = reinterpret_cast<unsigned *>(local + 128);
    G.timeout_ns = P.pipe_timeout;
    const int stages = tc_stages<BN, KBS>(dev, 64, decode_smem_budget());
    if (stages < 2) return VT_EARG;
    G.stages = stages;
    const int smem = tc_smem_bytes<BN, KBS>(stages);
    static bool attr_set[VT_MAX_DEV] = {false};
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(tp_row_linear_tc_kernel<T, BN, KBS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
            return (int)cudaGetLastError();
        attr_set[dev] = true;
    }
    int g = num_sms(dev);
    if (g > G.units) g = G.units;
    if (P.M > g || tc_decode_slot_bytes(P.M, g) > P.c.L.scratch_bytes) return VT_EARG;
    const int E = row_ctas(P.c.world, P.M, g);
    P.E = E;
    // row epilogue buffers: ceil(N / 4 / E) words of 4 floats and a norm weight word each, in the (free) stage ring
    if ((size_t)((P.N / 4 + E - 1) / E) * 24 > (size_t)stages * TcLayout<BN, KBS>::STAGE) return VT_EARG;
    return launch_k(tp_row_linear_tc_kernel<T, BN, KBS>, dim3(g), dim3(TC_THREADS), smem, s, true, mw, ma, G, P);
}

template <typename T, int BN>
static int fused_tc_kbs(FusedArgs<T> P, cudaStream_t s) {
    if (!decode_tail_rows() && tile_tail_fits(P.c, P.M, P.N, P.K)) {
        switch (decode_kbs()) {
            case 1: return launch_fused_tt<T, BN, 1>(P, s);
            case 2: return launch_fused_tt<T, BN, 2>(P, s);
            default: return launch_fused_tt<T, BN, 4>(P, s);
        }
    }
    switch (decode_kbs()) {
        case 1: return launch_fused_tc<T, BN, 1>(P, s);
        case 2: return launch_fused_tc<T, BN, 2>(P, s);
        default: return launch_fused_tc<T, BN, 4>(P, s);
    }
}

template <typename T, int MT>
static int launch_fused(FusedArgs<T> P, cudaStream_t s) {
    const int dev = cur_device();
    const int avail = gv_smem_budget(dev);
    int stages = (avail - GV_HDR - gv_align128((long long)MT * P.K)) / GV_STAGE;
    if (stages > GV_MAXSTAGES) stages = GV_MAXSTAGES;
    if (stages < 2) return VT_EARG;
    P.stages = stages;
    const int smem = gv_smem_bytes(MT, P.K, stages);
    static bool attr_set[VT_MAX_DEV] = {false};
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(tp_row_linear_kernel<T, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, avail) !=
            cudaSuccess)
            return (int)cudaGetLastError();
        attr_set[dev] = true;
    }
    const int G = num_sms(dev);
    if (P.M > G) return VT_EARG;
    const int E = row_ctas(P.c.world, P.M, G);
    P.E = E;
    if ((size_t)((P.N / 4 + E - 1) / E) * 24 + GV_HDR > (size_t)smem) return VT_EARG;   // row epilogue buffers
    CUtensorMap wmap;
    if (!make_map_i8(&wmap, P.w, P.N, P.K, GV_SEGB / 2, GV_RB, CU_TENSOR_MAP_SWIZZLE_NONE)) return VT_EARG;
    tp_row_linear_kernel<T, MT><<<G, GV_THREADS, smem, s>>>(wmap, P);
    return (int)cudaGetLastError();
}

// VLLM_TURING_FUSED_GEMV=1 selects the dp4a GEMV phase for M <= 16 (default: the tcgen05 phase for every M <= 32).
static bool fused_use_gemv() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_FUSED_GEMV");
        v = (e && atoi(e) != 0) ? 1 : 0;
    }
    return v != 0;
}

template <typename T>
static int dispatch_fused(FusedArgs<T> P, cudaStream_t s) {
    const int M = P.M;
    if (!fused_use_gemv() || M > 16) {
        if (M <= 16) return fused_tc_kbs<T, 16>(P, s);
        return fused_tc_kbs<T, 32>(P, s);
    }
    if (M <= 1) return launch_fused<T, 1>(P, s);
    if (M <= 2) return launch_fused<T, 2>(P, s);
    if (M <= 3) return launch_fused<T, 3>(P, s);
    if (M <= 4) return launch_fused<T, 4>(P, s);
    if (M <= 5) return launch_fused<T, 5>(P, s);
    if (M <= 6) return launch_fused<T, 6>(P, s);
    if (M <= 8) return launch_fused<T, 8>(P, s);
    if (M <= 12) return launch_fused<T, 12>(P, s);
    return launch_fused<T, 16>(P, s);
}

template <typename T>
static void preload_fused() {
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 1>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 2>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 3>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 4>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 5>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 6>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 8>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 12>);
    cudaFuncGetAttributes(&fa, tp_row_linear_kernel<T, 16>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tc_kernel<T, 16, 1>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tc_kernel<T, 16, 2>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tc_kernel<T, 16, 4>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tc_kernel<T, 32, 1>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tc_kernel<T, 32, 2>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tc_kernel<T, 32, 4>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tt_kernel<T, 16, 1>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tt_kernel<T, 16, 2>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tt_kernel<T, 16, 4>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tt_kernel<T, 32, 1>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tt_kernel<T, 32, 2>);
    cudaFuncGetAttributes(&fa, tp_row_linear_tt_kernel<T, 32, 4>);
}

}  // namespace vt

using namespace vt;

extern "C" {

// tp_prefill.cu
int vt_tp_row_linear_prefill(void *comm, const void *a, const void *w, const void *sa, const void *sw,
                             void *residual, const void *norm_w, float eps, void *q, void *scales, void *reduced,
                             int M, int N, int K, int dtype, void *stream);
int vt_tp_prefill_preload(void);

// The fused row-parallel layer tail on communicator `comm` (all ranks call it in the same order with the same M, N):
//   a [M, K] int8 (this rank's activation slice), w [N, K] int8 (this rank's weight slice), sa [M], sw [N] float32;
//   residual [M, N] (updated in place), norm_w [N], eps, q [M, N] int8, scales [M] float32 -- or residual = NULL for
//   a plain row-linear + all-reduce; reduced [M, N] (optional; required without residual) receives the all-reduced
//   sum. dtype 0 fp16 / 1 bf16. 1 <= M <= 32: this file's one-kernel decode tail (N % 4 == 0, K % 16 == 0,
//   M * N * 2 <= the communicator's LL capacity); M > 32: the prefill tail of tp_prefill.cu (its requirements).
int vt_tp_row_linear(void *comm, const void *a, const void *w, const void *sa, const void *sw, void *residual,
                     const void *norm_w, float eps, void *q, void *scales, void *reduced, int M, int N, int K,
                     int dtype, void *stream) {
    Comm *ch = reinterpret_cast<Comm *>(comm);
    if (ch && M > COMM_MBOX_ROWS)
        return vt_tp_row_linear_prefill(comm, a, w, sa, sw, residual, norm_w, eps, q, scales, reduced, M, N, K, dtype,
                                        stream);
    if (!ch || M < 1 || M > COMM_MBOX_ROWS || N < 4 || (N & 3) || K < 16 || (K & 15) || ((uintptr_t)a & 15) ||
        ((uintptr_t)w & 15))
        return VT_EARG;
    if (!residual && !reduced) return VT_EARG;
    if (residual && (!norm_w || !q || !scales || ((uintptr_t)residual & 7) || ((uintptr_t)norm_w & 7) ||
                     ((uintptr_t)q & 3)))
        return VT_EARG;
    if (reduced && ((uintptr_t)reduced & 7)) return VT_EARG;
    const CommLayout &L = ch->v.L;
    if ((size_t)M * N * 2 > L.ll_slot / 2 || (size_t)M * N * 4 > L.scratch_bytes || (N + 31) / 32 > COMM_TICKETS)
        return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == 0) {
        FusedArgs<__half> P{ch->v, (const int8_t *)a, (const int8_t *)w, (const float *)sa, (const float *)sw,
                            M, N, K, 0, 0, (__half *)residual, (const __half *)norm_w, eps, (int8_t *)q,
                            (float *)scales, (__half *)reduced, pipe_timeout_ns(), peer_timeout_ns()};
        return dispatch_fused(P, s);
    }
    FusedArgs<__nv_bfloat16> P{ch->v, (const int8_t *)a, (const int8_t *)w, (const float *)sa, (const float *)sw,
                               M, N, K, 0, 0, (__nv_bfloat16 *)residual, (const __nv_bfloat16 *)norm_w, eps,
                               (int8_t *)q, (float *)scales, (__nv_bfloat16 *)reduced, pipe_timeout_ns(),
                               peer_timeout_ns()};
    return dispatch_fused(P, s);
}

// Loads the fused kernels' module now (see vt_comm_create).
int vt_tp_preload(void) {
    preload_fused<__half>();
    preload_fused<__nv_bfloat16>();
    if (int rc = vt_tp_prefill_preload()) return rc;
    return (int)cudaGetLastError();
}

}  // extern "C"

// The decode-shape W8A8 GEMV core (M <= 16 token rows), HBM-bound.
//
// out[m, n] = sum_k a[m, k] * w[n, k] in int32, w the row-major [N, K] int8 weight (vLLM's [K, N] view with stride
// (1, K), vllm_turing/csrc/w8a8_gemv.cu:5), followed by an epilogue on whole 32-column row-blocks.
//
// Layout and schedule (one CTA per SM, 8 consumer warps + 1 producer warp):
//  * The activations a[M, K] are copied once into shared memory with one bulk copy.
//  * The work is the flat list of units (row-block rb of 32 weight rows, 16-byte chunk c of K), row-block major. CTA b
//    of G owns units [b T / G, (b + 1) T / G): every SM streams the same number of weight bytes whatever N and K are
//    (no wave quantisation on 148 SMs). A CTA's range cuts at most two row-blocks; their partial int32 sums meet in
//    a zero-initialised global scratch through atomicAdd (exact: integer addition commutes), and the CTA that brings a
//    row-block's ticket to K / 16 chunks finishes it (then zeroes the scratch and the ticket for the next call).
//  * The producer warp streams the owned weight rows segment by segment (32 rows x 512 bytes = 16 KB) into a ring of
//    shared-memory stages with two 2-D TMA tensor loads per stage (box 256 bytes x 32 rows; L2 evict-first), one
//    mbarrier per stage for "full" (bytes landed) and one for "empty" (the 8 consumer warps are done). Up to 128 KB per
//    SM are in flight, decoupled from registers; few large TMA operations per stage, because the number of TMA
//    operations a SM keeps in flight (not their bytes) bounded a first design with one 512-byte copy per row.
//    Boxes reaching past K or N read zeros (OOB fill) and still count their full bytes.
//  * Consumer warp w owns rows 4w .. 4w+3 of the row-block; lane l the 16-byte chunk l of the segment: 4 weight
//    vectors and M activation vectors from shared memory (conflict-free, consecutive lanes read consecutive 16 bytes)
//    feed 16 M dp4a. At the end of a piece the 32 lanes reduce with xor shuffles.
// Every wait is bounded (globaltimer); a timeout is reported into the status word and the CTA runs on without waiting
// (keeping every barrier uniform, so nothing can hang), producing garbage that the host discards on the status.
#pragma once
#include "common.cuh"

namespace vt {

constexpr int GV_RB = 32;                   // weight rows (output features) per row-block
constexpr int GV_SEGC = 32;                 // 16-byte chunks per row segment of a stage
constexpr int GV_SEGB = GV_SEGC * 16;       // 512 bytes
constexpr int GV_STAGE = GV_RB * GV_SEGB;   // 16 KB
constexpr int GV_CWARPS = 8;
constexpr int GV_CTHREADS = GV_CWARPS * 32;
constexpr int GV_THREADS = GV_CTHREADS + 32;
constexpr int GV_MAXSTAGES = 8;
constexpr int GV_HDR = 4096;                // barriers (256 B), tile [16][32] int32 (2 KB), control words

__host__ __device__ constexpr int gv_align128(long long x) { return (int)((x + 127) & ~127LL); }
__host__ __device__ inline int gv_smem_bytes(int MT, int K, int stages) {
    return GV_HDR + gv_align128((long long)MT * K) + stages * GV_STAGE;
}

struct GvSeg {
    int rb, c0, c1;
    bool last;   // the segment ends this CTA's piece of row-block rb
};

struct GvWalker {
    long long u, end;
    int K16;
    __device__ GvWalker(long long u0, long long u1, int k16) : u(u0), end(u1), K16(k16) {}
    __device__ __forceinline__ bool next(GvSeg &s) {
        if (u >= end) return false;
        s.rb = (int)(u / K16);
        s.c0 = (int)(u - (long long)s.rb * K16);
        long long lim = s.c0 + GV_SEGC;
        if (lim > K16) lim = K16;
        if (lim > s.c0 + (end - u)) lim = s.c0 + (end - u);
        s.c1 = (int)lim;
        u += s.c1 - s.c0;
        s.last = (s.c1 == K16) || (u == end);
        return true;
    }
};

struct GvSmem {
    uint64_t *full, *empty, *act_bar;
    int *tile;              // [MT][32] int32: the finished row-block's accumulators
    volatile int *ctl;      // [0] finisher flag, [1] abort
    int8_t *act;
    unsigned char *ring;
};

__device__ __forceinline__ GvSmem gv_carve(unsigned char *smem, int MT, int K) {
    GvSmem s;
    s.full = reinterpret_cast<uint64_t *>(smem);
    s.empty = s.full + GV_MAXSTAGES;
    s.act_bar = s.empty + GV_MAXSTAGES;
    s.tile = reinterpret_cast<int *>(smem + 256);
    s.ctl = reinterpret_cast<volatile int *>(smem + 256 + 16 * 32 * 4);   // ends before GV_HDR
    s.act = reinterpret_cast<int8_t *>(smem + GV_HDR);
    s.ring = smem + GV_HDR + gv_align128((long long)MT * K);
    return s;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// The GEMV phase. All GV_THREADS threads of the CTA call it. fin(rb, tile, tid) is called by the 256 consumer threads
// (tid 0..255) for every row-block this CTA finishes, with the row-block's int32 accumulators in tile[m * 32 + j]
// (column n = rb * 32 + j); named barrier 1 spans the consumer threads. Returns false if any wait of this CTA timed out.
template <int MT, class Fin>
__device__ __forceinline__ bool gemv_phase(const int8_t *__restrict__ a, const CUtensorMap *wmap, int M, int N,
                                           int K, int *__restrict__ scratch, int *__restrict__ tickets,
                                           unsigned char *smem, int stages, uint64_t deadline, unsigned *status,
                                           Fin &fin) {
    const int K16 = K >> 4;
    const int nrb = (N + GV_RB - 1) / GV_RB;
    const long long T = (long long)nrb * K16;
    const int G = gridDim.x, b = blockIdx.x;
    const long long u0 = T * b / G, u1 = T * (b + 1) / G;
    GvSmem sm = gv_carve(smem, MT, K);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], GV_CWARPS);
        }
        mbar_init(sm.act_bar, 1);
        sm.ctl[0] = 0;
        sm.ctl[1] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == GV_CWARPS) {
        // ---------------- producer warp ----------------
        if (lane == 0) {
            tma_prefetch_desc(wmap);
            mbar_arrive_expect_tx(sm.act_bar, (uint32_t)(M * K));
            bulk_g2s(sm.act, a, (uint32_t)(M * K), sm.act_bar);
        }
        const uint64_t pol = policy_evict_first();
        GvWalker it(u0, u1, K16);
        GvSeg sg;
        int i = 0;
        while (it.next(sg)) {
            const int s = i % stages;
            const uint32_t r = (uint32_t)(i / stages);
            if (lane == 0 && !sm.ctl[1]) {
                if (!mbar_wait(&sm.empty[s], (r & 1u) ^ 1u, deadline)) {
                    report(status, ST_PIPE_TIMEOUT | 1u);
                    sm.ctl[1] = 1;
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&sm.full[s], (uint32_t)GV_STAGE);
                unsigned char *st = sm.ring + (size_t)s * GV_STAGE;
                tma_load_2d_hint(st, wmap, sg.c0 * 16, sg.rb * GV_RB, &sm.full[s], pol);
                tma_load_2d_hint(st + GV_STAGE / 2, wmap, sg.c0 * 16 + GV_SEGB / 2, sg.rb * GV_RB, &sm.full[s], pol);
            }
            ++i;
        }
        return sm.ctl[1] == 0;
    }

    // ---------------- consumer warps ----------------
    const int tid = threadIdx.x;   // 0..255
    if (!mbar_wait(sm.act_bar, 0, deadline)) {
        report(status, ST_PIPE_TIMEOUT | 2u);
        sm.ctl[1] = 1;
    }
    int acc[4][MT];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[j][m] = 0;

    GvWalker it(u0, u1, K16);
    GvSeg sg;
    int i = 0, pc0 = -1;
    const unsigned char *act = reinterpret_cast<const unsigned char *>(sm.act);
    while (it.next(sg)) {
        const int s = i % stages;
        const uint32_t r = (uint32_t)(i / stages);
        if (!sm.ctl[1] && !mbar_wait(&sm.full[s], r & 1u, deadline)) {
            report(status, ST_PIPE_TIMEOUT | 3u);
            sm.ctl[1] = 1;
        }
        if (pc0 < 0) pc0 = sg.c0;
        const int nch = sg.c1 - sg.c0;
        if (lane < nch) {
            // stage layout: [box (lane / 16)][row 0..31][256 bytes]
            const unsigned char *st = sm.ring + (size_t)s * GV_STAGE + (lane >> 4) * (GV_STAGE / 2) +
                                      (warp * 4) * (GV_SEGB / 2) + (lane & 15) * 16;
            int4 wv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const int4 *>(st + j * (GV_SEGB / 2));
            const unsigned char *ap = act + (size_t)(sg.c0 + lane) * 16;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int4 av = *reinterpret_cast<const int4 *>(ap + (size_t)m * K);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[j][m] = dp4a(wv[j].x, av.x, acc[j][m]);
                    acc[j][m] = dp4a(wv[j].y, av.y, acc[j][m]);
                    acc[j][m] = dp4a(wv[j].z, av.z, acc[j][m]);
                    acc[j][m] = dp4a(wv[j].w, av.w, acc[j][m]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
        ++i;
        if (!sg.last) continue;

        // ---- end of a piece: reduce the 32 lanes, stage the row-block tile ----
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                int v = acc[j][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) sm.tile[m * 32 + warp * 4 + j] = v;
                acc[j][m] = 0;
            }
        named_sync(1, GV_CTHREADS);
        const int rb = sg.rb;
        const bool whole = (pc0 == 0 && sg.c1 == K16);
        if (whole) {
            fin(rb, sm.tile, tid);
        } else {
            for (int idx = tid; idx < M * 32; idx += GV_CTHREADS) {
                const int n = rb * GV_RB + (idx & 31);
                if (n < N) atomicAdd(&scratch[(long long)(idx >> 5) * N + n], sm.tile[idx]);
            }
            __threadfence();
            named_sync(1, GV_CTHREADS);
            if (tid == 0) {
                const int add = sg.c1 - pc0;
                const int old = atomicAdd(&tickets[rb], add);
                sm.ctl[0] = (old + add == K16) ? 1 : 0;
            }
            named_sync(1, GV_CTHREADS);
            if (sm.ctl[0]) {
                __threadfence();
                for (int idx = tid; idx < M * 32; idx += GV_CTHREADS) {
                    const int n = rb * GV_RB + (idx & 31);
                    if (n < N) {
                        int *p = &scratch[(long long)(idx >> 5) * N + n];
                        sm.tile[idx] = __ldcg(p);
                        *p = 0;
                    }
                }
                if (tid == 0) tickets[rb] = 0;
                named_sync(1, GV_CTHREADS);
                fin(rb, sm.tile, tid);
            }
        }
        named_sync(1, GV_CTHREADS);
        pc0 = -1;
    }
    return sm.ctl[1] == 0;
}

}  // namespace vt

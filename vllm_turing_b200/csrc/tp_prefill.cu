// Fused tensor-parallel row-linear layer tail for prefill shapes (M > 32 token rows) on B200 (sm_100a): the two-shot
// all-reduce is folded into the GEMM and the residual add + RMSNorm + int8 quantisation into the all-reduce.
//
//   partial_r = bf16( sa[m] * (sw[n] * (a_r . w_r^T)) )             this rank's K-slice    (vllm_turing/w8a8.py
//                                                                    big path, the CUTLASS order of w8a8_big.cu:26-35)
//   reduced   = bf16( sum_r float(partial_r) )  in rank order         the TP all-reduce      (ce_ar.cu:103-146)
//   residual  = bf16( reduced + residual );  y = bf16(residual * rsqrt(mean(residual^2) + eps) * norm_w)
//   q, scales = per-token int8 quantisation of y                     (tailoverlap.py:200, quantfuse.py:18-24)
//
// The reference runs the GEMM, then the all-reduce (copy-engine two-shot for large messages), then vLLM's norm + quant,
// and overlaps them only by chunking the token rows across two streams (vllm_turing/tailoverlap.py:165-204). Here the
// rows are owned by ranks (rank o owns rows [o R, (o + 1) R), R = M / world) and two kernels run per call:
//
//  1. tp_prefill_gemm_kernel: the tcgen05 prefill GEMM (tc_core.cuh, 256 x 256 tiles). Its epilogue writes each
//     finished tile, dequantised, straight into the receive buffer of the rank owning the tile's rows (NVLink stores for
//     a peer, HBM for itself) and then releases a per-tile flag there. The reduce-scatter's traffic thus leaves tile by
//     tile while the tensor cores work on the next tiles; no partial is ever written to this rank's own memory first.
//  2. tp_prefill_tail_kernel: phase A -- for each owned row, once every source's tiles of its 128-row block are flagged,
//     sum the sources' partials in rank order (identical bits on every rank), push the reduced row into every peer's
//     receive buffer (NVLink stores, in flight while the CTA goes on) and run the residual add + RMSNorm + quant on it
//     while it is in registers. Phase B -- once the peers' same CTA flagged its pushed rows, read them locally and run
//     the same row epilogue on them. (Pulling the peers' rows in phase B instead put a load latency over NVLink on
//     the critical path of every row.) Each row is handled by one group of N / 8 / VPT threads with the register-resident
//     arithmetic of vt_rms_norm_quant (same VPT, same summation order), so the outputs equal the unfused chain's bits.
//
// NVLink bytes per rank: (world - 1) / world x 2 M N out in (1) and in (2), the two-shot's bus traffic, of which (1)'s
// half overlaps the GEMM. All waits are bounded (globaltimer); timeouts land in the communicator's status word.
// Requirements: M % (128 x world) == 0, N % 8 == 0 with N / 8 / VPT in [64, 256] (a multiple of 32) for some
// VPT <= 8, K % 16 == 0; larger M runs in pieces that fit the communicator's two-shot buffers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.cuh"
#include "common.cuh"
#include "host_util.h"
#include "tc_core.cuh"
#include "tma_host.h"

extern "C" int vt_rms_norm_quant(const void *x, void *residual, const void *weight, float eps, void *q, void *scales,
                                 void *normed, int M, int N, int dtype, void *stream);   // norm_quant.cu

namespace vt {

constexpr int PF_BN = 256;          // GEMM tile columns (output features)
constexpr int PF_TAIL_THREADS = 512;

template <typename T>
struct PfArgs {
    CommView c;
    int M, N;                    // rows of this piece (M % (128 world) == 0), output features
    int R;                       // rows per rank (M / world)
    int ntb;                     // GEMM tiles along N
    int tpr;                     // tail: threads per row (N / 8 / VPT)
    T *residual;                 // [M, N] in place (NULL: only `reduced` is produced)
    const T *norm_w;             // [N]
    float eps;
    int8_t *q;                   // [M, N]
    float *scales;               // [M]
    T *reduced;                  // [M, N] or NULL
    uint64_t peer_timeout;
    int stage_rs;                // the GEMM epilogue stages its reduce-scatter stores through shared memory
};

// The reduce-scatter stores are staged (whole 64-byte row segments per store instruction) when peers are written;
// VLLM_TURING_PF_STAGE=0 never stages, =2 stages at one rank too (a test of the staged path on one GPU).
inline int pf_stage_rs(int world) {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_PF_STAGE");
        v = e ? atoi(e) : 1;
    }
    return (v == 2 || (v == 1 && world > 1)) ? 1 : 0;
}

// ---- kernel 1: GEMM whose epilogue scatters the tiles to their owners --------------------------------------------------
constexpr int PF_STAGE_ROWB = 80;   // bytes per row of a warp's staging chunk (64 data + 16 pad: conflict-free)

template <typename T>
struct PfRsEpi {
    static constexpr bool kPrefillHooks = true;
    // 64 floats for the core, then a 32-row x 32-column staging chunk per epilogue warp (up to 8 warps)
    static constexpr int kSmemFloats = 64 + 8 * 32 * PF_STAGE_ROWB / 4;
    const PfArgs<T> *A;
    unsigned seq, p;
    unsigned char *stage;   // this warp's staging chunk
    __device__ __forceinline__ void on_start(const TcArgs &, float *sm) {
        seq = *reinterpret_cast<volatile unsigned *>(A->c.seq_ptr()) + 1u;   // this call's number (after pdl_wait)
        p = A->c.world == 1 ? 0u : (seq & 1u);   // one rank: no peer, no double buffering (the host reads parity 0)
        stage = reinterpret_cast<unsigned char *>(sm + 64) + (size_t)((threadIdx.x >> 5) - 2) * 32 * PF_STAGE_ROWB;
    }
    __device__ __forceinline__ void post_start() {}

    // thread = row m of tile (ta, tb): dequantise its 256 accumulators and store them into the owner's RS buffer.
    // A warp holds 32 consecutive rows of one owner. Staged (A->stage_rs): each 32-column chunk goes through the warp's
    // shared-memory chunk, so every store instruction writes 8 rows x 64 contiguous bytes (a peer's memory over NVLink
    // takes whole segments); otherwise each thread stores its own row, 16 bytes per instruction and row.
    __device__ __forceinline__ void prefill_tile(const TcArgs &P, int m, int ta, int tb, uint32_t taddr) const {
        const int N = A->N, R = A->R;
        const int owner = m / R, lr = m - owner * R;
        char *rs = A->c.rs_buf(owner, p, A->c.rank);
        T *orow = reinterpret_cast<T *>(rs + (size_t)lr * N * sizeof(T));
        const float sam = P.sa[m];
        const int lane = threadIdx.x & 31;
        const bool staged = A->stage_rs != 0;
#pragma unroll 1
        for (int c = 0; c < PF_BN; c += 32) {
            uint32_t r[32];
            tmem_ld32(taddr + (uint32_t)c, r);
            tmem_ld_wait();
            const int n0 = tb * PF_BN + c;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint32_t w4[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const int n = min(n0 + j + 2 * h, N - 2);   // clamped past N: those granules are not stored
                    // the reference's CUTLASS epilogue order sa[m] * (sw[n] * acc) (vllm_turing/csrc/w8a8_big.cu:26-35)
                    const float v0 = __fmul_rn(sam, __fmul_rn(P.sw[n], (float)(int)r[j + 2 * h]));
                    const float v1 = __fmul_rn(sam, __fmul_rn(P.sw[n + 1], (float)(int)r[j + 2 * h + 1]));
                    w4[h] = pack2<T>(v0, v1);
                }
                if (staged)
                    *reinterpret_cast<uint4 *>(stage + lane * PF_STAGE_ROWB + j * 2) = make_uint4(w4[0], w4[1], w4[2],
                                                                                                  w4[3]);
                else if (n0 + j < N)   // N % 8 == 0: a granule is whole or absent
                    *reinterpret_cast<uint4 *>(orow + n0 + j) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            if (staged) {
                __syncwarp();
                const int g = lane & 3;   // this lane's 16-byte granule of a row's 64 bytes
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int rw = i * 8 + (lane >> 2);   // the row (of the warp's 32) this lane stores
                    if (n0 + g * 8 < N) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(stage + rw * PF_STAGE_ROWB + g * 16);
                        *reinterpret_cast<uint4 *>(rs + (size_t)(lr - lane + rw) * N * sizeof(T) +
                                                   (size_t)(n0 + g * 8) * sizeof(T)) = v;
                    }
                }
                __syncwarp();   // the chunk is read: the next one may overwrite it
            }
        }
    }
    // the four epilogue warps that stored the tile (named barrier `bar`, first thread `lead`): the stores are
    // performed (system scope) before the tile's flag is released
    __device__ __forceinline__ void prefill_tile_done(const TcArgs &, int ta, int tb, int bar, int lead) const {
        if (A->c.world == 1) return;   // the next kernel in the stream reads the tiles; no flags
        __threadfence_system();
        named_sync(bar, 128);
        if ((int)threadIdx.x == lead) {
            const int rbpr = A->R / TC_BM;   // 128-row blocks per rank
            const int owner = ta / rbpr;
            const int tile = (ta - owner * rbpr) * A->ntb + tb;
            st_release_sys(A->c.pf_tile_flag(owner, p, A->c.rank, tile), seq);
        }
    }
};

// WIDE: 256 x 256 tiles (tc_phase_wide, whose halves the finisher sees as 128-row tiles); else 128 x 256 (tc_phase).
template <typename T, bool WIDE>
__global__ void __launch_bounds__(WIDE ? TCW_THREADS : TC_THREADS, 1)
    tp_prefill_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           TcArgs P, const __grid_constant__ PfArgs<T> A) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    PfRsEpi<T> fin{&A, 0u, 0u};
    if constexpr (WIDE)
        tc_phase_wide<T>(&tmap_a, &tmap_b, P, smem_raw, fin);
    else
        tc_phase<T, PF_BN, false, 1>(&tmap_a, &tmap_b, P, smem_raw, fin);
}

// ---- kernel 2: reduce owned rows, all-gather by pulls, residual add + RMSNorm + quant ------------------------------------
// Sum over the threads of one row group (tpr threads, warps in order: the arithmetic of block_sum in norm_quant.cu).
__device__ __forceinline__ float group_sum(float v, float *red, int bar, int tpr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = (threadIdx.x % tpr) >> 5, lane = threadIdx.x & 31;
    named_sync(bar, tpr);
    if (lane == 0) red[w] = v;
    named_sync(bar, tpr);
    float t = 0.0f;
    for (int i = 0; i < (tpr >> 5); ++i) t += red[i];
    return t;
}
__device__ __forceinline__ float group_max(float v, float *red, int bar, int tpr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = (threadIdx.x % tpr) >> 5, lane = threadIdx.x & 31;
    named_sync(bar, tpr);
    if (lane == 0) red[w] = v;
    named_sync(bar, tpr);
    float t = 0.0f;
    for (int i = 0; i < (tpr >> 5); ++i) t = fmaxf(t, red[i]);
    return t;
}

// The row epilogue of one reduced row x (thread t holds elements 8 (t + k tpr) .. + 7 for k < VPT, rounded to T):
// residual := rnd(x + residual); y = rnd((h * rsqrt(mean(h^2) + eps)) * w); q, scale = quant(y). The arithmetic and
// summation order of rms_norm_quant_vec_kernel (norm_quant.cu) at the same VPT and threads per row.
// rv(k): the residual row's vector k of this thread (from registers or from a shared-memory slot).
template <typename T, int VPT, class RV>
__device__ __forceinline__ void pf_row_epilogue(const PfArgs<T> &A, size_t gr, int t, const float (&x)[VPT * 8],
                                                RV rv, float *red, int bar) {
    const int tpr = A.tpr, N = A.N;
    uint4 *rr = reinterpret_cast<uint4 *>(A.residual + gr * N);
    uint4 wv[VPT];   // the norm weight (L1 / L2 after the first row): issued now, used after the row's sum
#pragma unroll
    for (int k = 0; k < VPT; ++k) wv[k] = __ldg(reinterpret_cast<const uint4 *>(A.norm_w) + t + k * tpr);
    float h[VPT * 8];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint4 r4 = rv(k);
        const uint32_t rs_[4] = {r4.x, r4.y, r4.z, r4.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 b = unpack2<T>(rs_[e]);
            const float h0 = rnd<T>(x[8 * k + 2 * e] + b.x), h1 = rnd<T>(x[8 * k + 2 * e + 1] + b.y);
            h[8 * k + 2 * e] = h0;
            h[8 * k + 2 * e + 1] = h1;
            ss += h0 * h0 + h1 * h1;
            o[e] = pack2<T>(h0, h1);
        }
        rr[t + k * tpr] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    ss = group_sum(ss, red, bar, tpr);
    const float rs = __frsqrt_rn(__fdiv_rn(ss, (float)N) + A.eps);
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t ws[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 wf = unpack2<T>(ws[e]);
            const float y0 = rnd<T>(__fmul_rn(__fmul_rn(h[8 * k + 2 * e], rs), wf.x));
            const float y1 = rnd<T>(__fmul_rn(__fmul_rn(h[8 * k + 2 * e + 1], rs), wf.y));
            h[8 * k + 2 * e] = y0;
            h[8 * k + 2 * e + 1] = y1;
            amax = fmaxf(amax, fmaxf(fabsf(y0), fabsf(y1)));
        }
    }
    amax = group_max(amax, red, bar, tpr);
    const float inv = quant_inv(amax);
    if (t == 0) A.scales[gr] = __fdiv_rn(amax, 127.0f);
    uint2 *qr = reinterpret_cast<uint2 *>(A.q + gr * N);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        uint32_t b[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const float *v = &h[8 * k + 4 * hh];
            b[hh] = (uint32_t)(uint8_t)quant1(v[0], inv) | ((uint32_t)(uint8_t)quant1(v[1], inv) << 8) |
                    ((uint32_t)(uint8_t)quant1(v[2], inv) << 16) | ((uint32_t)(uint8_t)quant1(v[3], inv) << 24);
        }
        qr[t + k * tpr] = make_uint2(b[0], b[1]);
    }
}

// x (floats of the reduced row) from packed vectors
template <typename T, int VPT>
__device__ __forceinline__ void pf_unpack(const uint4 (&v)[VPT], float (&x)[VPT * 8]) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t u[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<T>(u[e]);
            x[8 * k + 2 * e] = f.x;
            x[8 * k + 2 * e + 1] = f.y;
        }
    }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(PF_TAIL_THREADS, 1) tp_prefill_tail_kernel(const __grid_constant__ PfArgs<T> A) {
    __shared__ unsigned s_seq;
    __shared__ float red_all[PF_TAIL_THREADS / 64][8];   // [row group][warp of the group]
    pdl_wait();   // residual, norm weight and the outputs' previous readers belong to earlier kernels
    const CommView &c = A.c;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t deadline = globaltimer() + A.peer_timeout;
    const int tpr = A.tpr, N = A.N, R = A.R, W = c.world, me = c.rank;
    const int g = threadIdx.x / tpr, t = threadIdx.x - g * tpr;
    const int RG = blockDim.x / tpr;
    const long long S = (long long)gridDim.x * RG, slot = (long long)blockIdx.x * RG + g;
    const int lr0 = (int)(R * slot / S), lr1 = (int)(R * (slot + 1) / S);   // this group's rows of every chunk
    const int bar = 1 + g;
    float *red = red_all[g];
    const size_t rowb = (size_t)N * sizeof(T);
    bool dead = false;

    // ---- phase A: this rank's rows ----
    int cur_rb = -1;
    for (int lr = lr0; lr < lr1; ++lr) {
        const int rb = lr / TC_BM;
        if (rb != cur_rb) {   // every source's GEMM tiles of this 128-row block have landed
            cur_rb = rb;
            for (int i = t; i < W * A.ntb; i += tpr) {
                const int src = i / A.ntb, tb = i - src * A.ntb;
                if (!dead && !flag_wait(c.pf_tile_flag(me, p, src, rb * A.ntb + tb), seq, deadline)) {
                    report(c.status(), ST_PEER_TIMEOUT | 0xb00u | (unsigned)src);
                    dead = true;
                }
            }
            named_sync(bar, tpr);
        }
        const size_t gr = (size_t)me * R + lr;
        float x[VPT * 8];
        for (int src = 0; src < W; ++src) {   // rank order: identical bits on every rank
            const uint4 *pr = reinterpret_cast<const uint4 *>(c.rs_buf(me, p, src) + (size_t)lr * rowb);
            uint4 v[VPT];
#pragma unroll
            for (int k = 0; k < VPT; ++k) v[k] = __ldcg(pr + t + k * tpr);   // written by peers: L2, not L1
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const uint32_t u[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = unpack2<T>(u[e]);
                    x[8 * k + 2 * e] = src == 0 ? f.x : x[8 * k + 2 * e] + f.x;
                    x[8 * k + 2 * e + 1] = src == 0 ? f.y : x[8 * k + 2 * e + 1] + f.y;
                }
            }
        }
        uint4 ov[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k)
            ov[k] = make_uint4(pack2<T>(x[8 * k], x[8 * k + 1]), pack2<T>(x[8 * k + 2], x[8 * k + 3]),
                               pack2<T>(x[8 * k + 4], x[8 * k + 5]), pack2<T>(x[8 * k + 6], x[8 * k + 7]));
        for (int k2 = 1; k2 < W; ++k2) {   // push the reduced row into every peer's receive buffer (NVLink stores)
            uint4 *agr = reinterpret_cast<uint4 *>(c.agr_buf((me + k2) % W, p, me) + (size_t)lr * rowb);
#pragma unroll
            for (int k = 0; k < VPT; ++k) agr[t + k * tpr] = ov[k];
        }
        if (A.reduced) {
#pragma unroll
            for (int k = 0; k < VPT; ++k) reinterpret_cast<uint4 *>(A.reduced + gr * N)[t + k * tpr] = ov[k];
        }
        if (A.residual) {
            uint4 rv[VPT];   // loaded after the sums: fewer registers live across the sources' loads
#pragma unroll
            for (int k = 0; k < VPT; ++k) rv[k] = reinterpret_cast<const uint4 *>(A.residual + gr * N)[t + k * tpr];
            pf_unpack<T, VPT>(ov, x);   // the rounded sum
            pf_row_epilogue<T, VPT>(A, gr, t, x, [&](int k) { return rv[k]; }, red, bar);
        }
    }

    // ---- phase B: the peers' rows, pushed into this rank's receive buffer by their owners ----
    if (W > 1) {
        __threadfence_system();   // the pushes of this CTA's rows are performed before their flags
        __syncthreads();
        if ((int)threadIdx.x < W && (int)threadIdx.x != me)
            st_release_sys(c.pf_ag_flag(threadIdx.x, p, me, blockIdx.x), seq);
        for (int k = 1; k < W; ++k) {
            const int src = (me + k) % W;
            if (threadIdx.x == 0 && !dead && !flag_wait(c.pf_ag_flag(me, p, src, blockIdx.x), seq, deadline)) {
                report(c.status(), ST_PEER_TIMEOUT | 0xc00u | (unsigned)src);
                dead = true;
            }
            __syncthreads();
            const uint4 *agp = reinterpret_cast<const uint4 *>(c.agr_buf(me, p, src));
            for (int lr = lr0; lr < lr1; ++lr) {
                const size_t gr = (size_t)src * R + lr;
                uint4 rv[VPT], v[VPT];
#pragma unroll
                for (int j = 0; j < VPT; ++j) v[j] = __ldcg(agp + (size_t)lr * (N / 8) + t + j * tpr);
                if (A.residual) {
#pragma unroll
                    for (int j = 0; j < VPT; ++j)
                        rv[j] = reinterpret_cast<const uint4 *>(A.residual + gr * N)[t + j * tpr];
                }
                if (A.reduced) {
#pragma unroll
                    for (int j = 0; j < VPT; ++j) reinterpret_cast<uint4 *>(A.reduced + gr * N)[t + j * tpr] = v[j];
                }
                if (A.residual) {
                    float x[VPT * 8];
                    pf_unpack<T, VPT>(v, x);
                    pf_row_epilogue<T, VPT>(A, gr, t, x, [&](int k) { return rv[k]; }, red, bar);
                }
            }
        }
    }
    comm_end(c, seq);
}

// ---- kernel 2, staged variant: rows land in shared memory by bulk copies ----------------------------------------------
// The same two phases and arithmetic as tp_prefill_tail_kernel, but a row group does not load its rows into registers:
// its first thread keeps PF_SLOTS whole rows (a source's partial row, a peer's reduced row, the residual row) in flight
// as 1-D bulk copies (cp.async.bulk, the TMA engine) into a ring of shared-memory slots, completed on an mbarrier per
// slot, so the bytes in flight per SM are set by shared memory (PF_SLOTS x N x 2 per group), not by registers. Each
// slot is handed back after the group has read it (a named barrier), and the issuing thread fences the async proxy
// before reusing it. Peer rows are read the same way over NVLink (a bulk load from a peer's memory, no multicast).
constexpr int PF_SLOTS = 4;

template <typename T>
struct PfRing {   // one row group's ring
    unsigned char *slot0;
    uint64_t *full;
    uint32_t rowb;
    int issued, used;   // items issued / consumed (the same count in every thread of the group)
};

__device__ __forceinline__ void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <typename T, int VPT>
__global__ void __launch_bounds__(PF_TAIL_THREADS, 1)
    tp_prefill_tail_bulk_kernel(const __grid_constant__ PfArgs<T> A) {
    extern __shared__ __align__(128) unsigned char pf_smem[];
    __shared__ unsigned s_seq;
    __shared__ float red_all[PF_TAIL_THREADS / 64][8];
    __shared__ __align__(8) uint64_t bars[PF_TAIL_THREADS / 64][PF_SLOTS];
    pdl_wait();
    const CommView &c = A.c;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t deadline = globaltimer() + A.peer_timeout;
    const int tpr = A.tpr, N = A.N, R = A.R, W = c.world, me = c.rank;
    const int g = threadIdx.x / tpr, t = threadIdx.x - g * tpr;
    const int RG = blockDim.x / tpr;
    const long long S = (long long)gridDim.x * RG, slot = (long long)blockIdx.x * RG + g;
    const int lr0 = (int)(R * slot / S), lr1 = (int)(R * (slot + 1) / S);
    const int bar = 1 + g;
    const uint32_t rowb = (uint32_t)N * sizeof(T);
    float *red = red_all[g];
    uint64_t *full = bars[g];
    unsigned char *ring = pf_smem + (size_t)g * PF_SLOTS * rowb;
    const bool lead = t == 0;
    if (lead)
        for (int s = 0; s < PF_SLOTS; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    __syncthreads();
    bool dead = false;
    // the source of item i of a row: partials 0..nsrc-1 (phase A) or the peer's reduced row (phase B), then residual
    const int per_row_a = W + (A.residual ? 1 : 0);
    int issued = 0, used = 0;

    // ---- phase A ----
    // every source's tiles of the row blocks of this group's rows have landed (one cooperative wait up front)
    if (lr1 > lr0) {
        for (int rb = lr0 / TC_BM; rb <= (lr1 - 1) / TC_BM; ++rb)
            for (int i = t; i < W * A.ntb; i += tpr) {
                const int src = i / A.ntb, tb = i - src * A.ntb;
                if (!dead && !flag_wait(c.pf_tile_flag(me, p, src, rb * A.ntb + tb), seq, deadline)) {
                    report(c.status(), ST_PEER_TIMEOUT | 0xb00u | (unsigned)src);
                    dead = true;
                }
            }
        named_sync(bar, tpr);
    }
    const int items_a = (lr1 - lr0) * per_row_a;
    auto src_a = [&](int i) -> const void * {
        const int lr = lr0 + i / per_row_a, k = i - (i / per_row_a) * per_row_a;
        if (k < W) return c.rs_buf(me, p, k) + (size_t)lr * rowb;
        return A.residual + ((size_t)me * R + lr) * N;
    };
    if (lead) {
        fence_async_global();   // the flags were acquired by generic loads; the bulk copies read through the async proxy
        for (; issued < items_a && issued < PF_SLOTS; ++issued) {
            mbar_arrive_expect_tx(&full[issued % PF_SLOTS], rowb);
            bulk_g2s(ring + (size_t)(issued % PF_SLOTS) * rowb, src_a(issued), rowb, &full[issued % PF_SLOTS]);
        }
    }
    // wait for the slot of item `used`; its data as 16-byte vectors
    auto take = [&](uint32_t code) -> const uint4 * {
        const int s = used % PF_SLOTS;
        if (!mbar_wait(&full[s], (uint32_t)(used / PF_SLOTS) & 1u, deadline) && !dead) {
            report(c.status(), ST_PIPE_TIMEOUT | code);
            dead = true;
        }
        return reinterpret_cast<const uint4 *>(ring + (size_t)s * rowb);
    };
    for (int lr = lr0; lr < lr1; ++lr) {
        float x[VPT * 8];
        for (int k = 0; k < W; ++k) {   // the sources' partial rows, summed in rank order
            const uint4 *sv = take(0xd00u);
#pragma unroll
            for (int j = 0; j < VPT; ++j) {
                const uint4 v = sv[t + j * tpr];
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = unpack2<T>(u[e]);
                    x[8 * j + 2 * e] = k == 0 ? f.x : x[8 * j + 2 * e] + f.x;
                    x[8 * j + 2 * e + 1] = k == 0 ? f.y : x[8 * j + 2 * e + 1] + f.y;
                }
            }
            named_sync(bar, tpr);   // the slot is read: hand it back
            ++used;
            if (lead && issued < items_a) {
                fence_async_shared();
                const int s2 = issued % PF_SLOTS;
                mbar_arrive_expect_tx(&full[s2], rowb);
                bulk_g2s(ring + (size_t)s2 * rowb, src_a(issued), rowb, &full[s2]);
                ++issued;
            }
        }
        const size_t gr = (size_t)me * R + lr;
        uint4 ov[VPT];
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            ov[j] = make_uint4(pack2<T>(x[8 * j], x[8 * j + 1]), pack2<T>(x[8 * j + 2], x[8 * j + 3]),
                               pack2<T>(x[8 * j + 4], x[8 * j + 5]), pack2<T>(x[8 * j + 6], x[8 * j + 7]));
        for (int k2 = 1; k2 < W; ++k2) {   // push the reduced row into every peer's receive buffer (NVLink stores)
            uint4 *agr = reinterpret_cast<uint4 *>(c.agr_buf((me + k2) % W, p, me) + (size_t)lr * rowb);
#pragma unroll
            for (int j = 0; j < VPT; ++j) agr[t + j * tpr] = ov[j];
        }
        if (A.reduced) {
#pragma unroll
            for (int j = 0; j < VPT; ++j) reinterpret_cast<uint4 *>(A.reduced + gr * N)[t + j * tpr] = ov[j];
        }
        if (A.residual) {   // the residual row's slot is read inside the epilogue, then handed back
            const uint4 *rs = take(0xd00u);
            pf_unpack<T, VPT>(ov, x);
            pf_row_epilogue<T, VPT>(A, gr, t, x, [&](int k) { return rs[t + k * tpr]; }, red, bar);
            named_sync(bar, tpr);
            ++used;
            if (lead && issued < items_a) {
                fence_async_shared();
                const int s2 = issued % PF_SLOTS;
                mbar_arrive_expect_tx(&full[s2], rowb);
                bulk_g2s(ring + (size_t)s2 * rowb, src_a(issued), rowb, &full[s2]);
                ++issued;
            }
        }
    }

    // ---- phase B: the peers' rows, pushed into this rank's receive buffer by their owners (local reads) ----
    if (W > 1) {
        __threadfence_system();   // the pushes of this CTA's rows are performed before their flags
        __syncthreads();
        if ((int)threadIdx.x < W && (int)threadIdx.x != me)
            st_release_sys(c.pf_ag_flag(threadIdx.x, p, me, blockIdx.x), seq);
        const int per_row_b = A.residual ? 2 : 1;
        const int rows = lr1 - lr0;
        const int items_b = (W - 1) * rows * per_row_b;
        // item i: peer k = 1 + i / (rows per_row_b), row lr0 + (i / per_row_b) % rows; the peer's reduced row, then
        // the residual row
        auto src_b = [&](int i) -> const void * {
            const int k = 1 + i / (rows * per_row_b), r = (i / per_row_b) % rows, e = i % per_row_b;
            const int srk = (me + k) % W;
            if (e == 0) return c.agr_buf(me, p, srk) + (size_t)(lr0 + r) * rowb;
            return A.residual + ((size_t)srk * R + lr0 + r) * N;
        };
        int ib = 0;   // items of phase B issued (by the group's first thread); the ring continues from phase A
        auto issue_b = [&]() {
            // a peer's first item: its CTA blockIdx.x must have pushed its reduced rows here
            const int k = 1 + ib / (rows * per_row_b);
            if (ib % (rows * per_row_b) == 0) {
                const int srk = (me + k) % W;
                if (!dead && !flag_wait(c.pf_ag_flag(me, p, srk, blockIdx.x), seq, deadline)) {
                    report(c.status(), ST_PEER_TIMEOUT | 0xc00u | (unsigned)srk);
                    dead = true;
                }
                fence_async_global();
            }
            fence_async_shared();
            const int s2 = (issued + ib) % PF_SLOTS;
            mbar_arrive_expect_tx(&full[s2], rowb);
            bulk_g2s(ring + (size_t)s2 * rowb, src_b(ib), rowb, &full[s2]);
            ++ib;
        };
        if (lead)
            while (ib < items_b && ib < PF_SLOTS) issue_b();
        for (int it = 0; it < items_b; it += per_row_b) {
            const int k = 1 + it / (rows * per_row_b), r = (it / per_row_b) % rows;
            const int srk = (me + k) % W;
            const size_t gr = (size_t)srk * R + lr0 + r;
            float x[VPT * 8];
            {   // the peer's reduced row
                const uint4 *sv = take(0xe00u);
                uint4 v[VPT];
#pragma unroll
                for (int j = 0; j < VPT; ++j) v[j] = sv[t + j * tpr];
                if (A.reduced) {
#pragma unroll
                    for (int j = 0; j < VPT; ++j) reinterpret_cast<uint4 *>(A.reduced + gr * N)[t + j * tpr] = v[j];
                }
                pf_unpack<T, VPT>(v, x);
                named_sync(bar, tpr);
                ++used;
                if (lead && ib < items_b) issue_b();
            }
            if (A.residual) {   // the residual row's slot is read inside the epilogue, then handed back
                const uint4 *rs = take(0xe00u);
                pf_row_epilogue<T, VPT>(A, gr, t, x, [&](int k) { return rs[t + k * tpr]; }, red, bar);
                named_sync(bar, tpr);
                ++used;
                if (lead && ib < items_b) issue_b();
            }
        }
    }
    comm_end(c, seq);
}

// Tail variant: rows staged through shared memory (tp_prefill_tail_bulk_kernel, the default; measured at TP1, M = 8192:
// 70 us against 89 us for the register version) or, with VLLM_TURING_PF_TAIL=reg, tp_prefill_tail_kernel.
inline bool pf_tail_bulk() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_PF_TAIL");
        v = (e && e[0] == 'r') ? 0 : 1;
    }
    return v != 0;
}

// VPT (16-byte vectors per thread) and threads per row of the row epilogue: the choice vt_rms_norm_quant makes
// (VPT from 8 down, threads = N / 8 / VPT a multiple of 32 in [64, 256]); false if none fits.
inline bool pf_row_shape(int N, int &vpt, int &tpr) {
    if (N <= 0 || (N & 7)) return false;
    const int nv = N / 8;
    for (int v = 8; v >= 1; --v) {
        if (nv % v) continue;
        const int t = nv / v;
        if ((t & 31) || t < 64 || t > 256) continue;
        vpt = v;
        tpr = t;
        return true;
    }
    return false;
}

template <typename T, int VPT>
static int launch_tail_bulk_v(const PfArgs<T> &A, dim3 g, dim3 b, size_t smem, cudaStream_t s) {
    static bool attr[VT_MAX_DEV] = {false};
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    if (!attr[dev]) {   // once, for the largest ring any N can ask for (launch_tail keeps smem within it)
        if (cudaFuncSetAttribute(tp_prefill_tail_bulk_kernel<T, VPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 max_smem_optin(dev) - 4096) != cudaSuccess)
            return (int)cudaGetLastError();
        attr[dev] = true;
    }
    return launch_k(tp_prefill_tail_bulk_kernel<T, VPT>, g, b, smem, s, true, A);
}

template <typename T>
static int launch_tail(const PfArgs<T> &A, int vpt, int grid, cudaStream_t s) {
    const dim3 g(grid), b((PF_TAIL_THREADS / A.tpr) * A.tpr);
    const size_t bulk_smem = (size_t)(PF_TAIL_THREADS / A.tpr) * PF_SLOTS * A.N * sizeof(T);
    if (pf_tail_bulk() && bulk_smem + 4096 <= (size_t)max_smem_optin(cur_device())) {
        switch (vpt) {
            case 8: return launch_tail_bulk_v<T, 8>(A, g, b, bulk_smem, s);
            case 7: return launch_tail_bulk_v<T, 7>(A, g, b, bulk_smem, s);
            case 6: return launch_tail_bulk_v<T, 6>(A, g, b, bulk_smem, s);
            case 5: return launch_tail_bulk_v<T, 5>(A, g, b, bulk_smem, s);
            case 4: return launch_tail_bulk_v<T, 4>(A, g, b, bulk_smem, s);
            case 3: return launch_tail_bulk_v<T, 3>(A, g, b, bulk_smem, s);
            case 2: return launch_tail_bulk_v<T, 2>(A, g, b, bulk_smem, s);
            default: return launch_tail_bulk_v<T, 1>(A, g, b, bulk_smem, s);
        }
    }
    switch (vpt) {
        case 8: return launch_k(tp_prefill_tail_kernel<T, 8>, g, b, 0, s, true, A);
        case 7: return launch_k(tp_prefill_tail_kernel<T, 7>, g, b, 0, s, true, A);
        case 6: return launch_k(tp_prefill_tail_kernel<T, 6>, g, b, 0, s, true, A);
        case 5: return launch_k(tp_prefill_tail_kernel<T, 5>, g, b, 0, s, true, A);
        case 4: return launch_k(tp_prefill_tail_kernel<T, 4>, g, b, 0, s, true, A);
        case 3: return launch_k(tp_prefill_tail_kernel<T, 3>, g, b, 0, s, true, A);
        case 2: return launch_k(tp_prefill_tail_kernel<T, 2>, g, b, 0, s, true, A);
        default: return launch_k(tp_prefill_tail_kernel<T, 1>, g, b, 0, s, true, A);
    }
}

template <typename T>
static int prefill_fused(Comm *ch, const void *a, const void *w, const float *sa, const float *sw, T *residual,
                         const T *norm_w, float eps, int8_t *q, float *scales, T *reduced, int M, int N, int K,
                         cudaStream_t s) {
    const CommView &v = ch->v;
    const int W = v.world, dev = ch->dev;
    int vpt = 0, tpr = 0;
    if (!pf_row_shape(N, vpt, tpr)) return VT_EARG;
    if (M % (TC_BM * W)) return VT_EARG;
    const int ntb = (N + PF_BN - 1) / PF_BN;
    // rows per rank in one piece: its partials fit a two-shot receive buffer and its tiles the flag table
    long long Rmax = (long long)(v.L.chunk_cap / ((size_t)N * sizeof(T)));
    const long long Rtiles = (long long)(PF_MAX_TILES / ntb) * TC_BM;
    if (Rmax > Rtiles) Rmax = Rtiles;
    Rmax = Rmax / TC_BM * TC_BM;
    if (Rmax < TC_BM) return VT_EARG;
    const bool wide = prefill_wide();
    const int stages = wide ? tc_wide_stages(dev, PfRsEpi<T>::kSmemFloats)
                            : tc_stages<PF_BN, 1>(dev, PfRsEpi<T>::kSmemFloats);
    if (stages < 2) return VT_EARG;
    const int smem = wide ? tc_wide_smem_bytes(stages, PfRsEpi<T>::kSmemFloats)
                          : tc_smem_bytes<PF_BN, 1>(stages, PfRsEpi<T>::kSmemFloats);
    auto gemm_kernel = wide ? tp_prefill_gemm_kernel<T, true> : tp_prefill_gemm_kernel<T, false>;
    static bool attr[2][2][VT_MAX_DEV] = {{{false}}};
    const int ti = std::is_same<T, __half>::value ? 0 : 1;
    if (!attr[wide][ti][dev]) {
        if (cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return (int)cudaGetLastError();
        attr[wide][ti][dev] = true;
    }
    CUtensorMap mb;
    if (!tc_make_map(&mb, w, N, K, PF_BN)) return VT_EARG;
    const int sms = num_sms(dev);
    const long long piece = Rmax * W;
    for (long long m0 = 0; m0 < M; m0 += piece) {
        const int Mp = (int)(M - m0 < piece ? M - m0 : piece);
        CUtensorMap ma;
        if (!tc_make_map(&ma, (const int8_t *)a + m0 * K, Mp, K, TC_BM)) return VT_EARG;
        TcArgs P{};
        P.n_tiles_a = wide ? (Mp + 2 * TC_BM - 1) / (2 * TC_BM) : Mp / TC_BM;
        P.n_tiles_b = ntb;
        P.nkb = (K + TC_BK - 1) / TC_BK;
        P.units = P.n_tiles_a * P.n_tiles_b;
        P.stream_k = 0;
        const int gm = wide ? 8 : 16;
        P.group_m = P.n_tiles_a < gm ? P.n_tiles_a : gm;
        P.split_tail = wide ? prefill_split_tail() : 0;
        P.sa = sa + m0;
        P.sw = sw;
        P.sa_rows = 1;
        P.sw_rows = 1;
        P.M = Mp;
        P.N = N;
        P.stages = stages;
        P.timeout_ns = pipe_timeout_ns();
        P.status = reinterpret_cast<unsigned *>(v.base[v.rank] + 128);
        PfArgs<T> A{};
        A.c = v;
        A.M = Mp;
        A.N = N;
        A.R = Mp / W;
        A.ntb = ntb;
        A.tpr = tpr;
        A.residual = residual ? residual + m0 * N : nullptr;
        A.norm_w = norm_w;
        A.eps = eps;
        A.q = q ? q + m0 * N : nullptr;
        A.scales = scales ? scales + m0 : nullptr;
        A.reduced = reduced ? reduced + m0 * N : nullptr;
        A.peer_timeout = peer_timeout_ns();
        A.stage_rs = pf_stage_rs(W);
        const int g1 = wide ? tc_wide_grid(sms, P) : (sms < P.units ? sms : P.units);
        if (int rc = launch_k(gemm_kernel, dim3(g1), dim3(wide ? TCW_THREADS : TC_THREADS), smem, s, true, ma, mb, P,
                              A))
            return rc;
        if (W == 1) {
            // one rank: nothing to reduce or gather, so the row epilogue is the standalone residual + RMSNorm + quant
            // kernel over the GEMM's rows (same arithmetic as the tail kernel's, at higher occupancy). The GEMM wrote
            // them to parity 0 (with one rank nothing is double-buffered) and published no flags.
            const T *part = reinterpret_cast<const T *>(v.base[v.rank] + v.L.rs_off);
            if (reduced) {
                if (cudaError_t e = cudaMemcpyAsync(reduced + m0 * N, part, (size_t)Mp * N * sizeof(T),
                                                    cudaMemcpyDeviceToDevice, s))
                    return (int)e;
            }
            if (residual) {
                const int dt = std::is_same<T, __half>::value ? 0 : 1;
                if (int rc = vt_rms_norm_quant(part, residual + m0 * N, norm_w, eps, q + m0 * N, scales + m0, nullptr,
                                               Mp, N, dt, s))
                    return rc;
            }
            continue;
        }
        int g2 = sms < PF_MAX_CTAS ? sms : PF_MAX_CTAS;
        if (int rc = launch_tail<T>(A, vpt, g2, s)) return rc;
    }
    return 0;
}

template <typename T>
static void preload_prefill() {
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, tp_prefill_gemm_kernel<T, false>);
    cudaFuncGetAttributes(&fa, tp_prefill_gemm_kernel<T, true>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 1>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 2>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 3>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 4>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 5>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 6>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 7>);
    cudaFuncGetAttributes(&fa, tp_prefill_tail_kernel<T, 8>);
}

}  // namespace vt

using namespace vt;

extern "C" {

// The fused row-parallel layer tail for prefill shapes: the arguments and results of vt_tp_row_linear for M > 32
// (M % (128 x world) == 0, N % 8 == 0 with a row shape pf_row_shape accepts, K % 16 == 0; a, w 16-byte aligned,
// residual / norm_w / reduced 16-byte aligned, q 8-byte aligned). Two launches per piece of rows (GEMM with the
// reduce-scatter in its epilogue, then reduce + all-gather + row epilogue), one call number each piece.
int vt_tp_row_linear_prefill(void *comm, const void *a, const void *w, const void *sa, const void *sw,
                             void *residual, const void *norm_w, float eps, void *q, void *scales, void *reduced,
                             int M, int N, int K, int dtype, void *stream) {
    Comm *ch = reinterpret_cast<Comm *>(comm);
    if (!ch || M < 1 || N < 8 || K < 16 || (K & 15) || ((uintptr_t)a & 15) || ((uintptr_t)w & 15)) return VT_EARG;
    if (!residual && !reduced) return VT_EARG;
    if (residual && (!norm_w || !q || !scales || ((uintptr_t)residual & 15) || ((uintptr_t)norm_w & 15) ||
                     ((uintptr_t)q & 7)))
        return VT_EARG;
    if (reduced && ((uintptr_t)reduced & 15)) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == 0)
        return prefill_fused<__half>(ch, a, w, (const float *)sa, (const float *)sw, (__half *)residual,
                                     (const __half *)norm_w, eps, (int8_t *)q, (float *)scales, (__half *)reduced, M,
                                     N, K, s);
    return prefill_fused<__nv_bfloat16>(ch, a, w, (const float *)sa, (const float *)sw, (__nv_bfloat16 *)residual,
                                        (const __nv_bfloat16 *)norm_w, eps, (int8_t *)q, (float *)scales,
                                        (__nv_bfloat16 *)reduced, M, N, K, s);
}

// Loads the prefill kernels' module now (a lazily loaded module may synchronise behind a kernel spinning on a peer).
int vt_tp_prefill_preload(void) {
    preload_prefill<__half>();
    preload_prefill<__nv_bfloat16>();
    return (int)cudaGetLastError();
}

}  // extern "C"

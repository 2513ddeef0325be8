// Row-wise epilogue kernels for B200 (sm_100a), HBM-bound; one CTA per token row, except silu_mul_quant for a few
// rows (decode), which splits each row over several CTAs so the whole GPU shares the work:
//   vt_scaled_int8_quant  per-token dynamic symmetric int8 quantisation   (vllm_turing/quantfuse.py:18-24)
//   vt_rms_norm_quant     residual add + RMSNorm + per-token int8 quant   (the call at vllm_turing/tailoverlap.py:200,
//                         arithmetic of tests/test_quantfuse.py:45-48 + quantfuse.py:18-24)
//   silu_mul_quant        SiLU(gate) * up + per-token int8 quant          (vllm_turing/csrc/silu_quant.cu:71-77 ABI)
// Reductions are deterministic (fixed shuffle tree, then warps in order), so every rank of a tensor-parallel group
// that feeds identical rows gets identical outputs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "host_util.h"

namespace vt {

constexpr int RQ_THREADS = 512;

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += red[i];   // warps in order: identical on every CTA and rank
    return t;
}

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
    return t;
}

// 4 consecutive 16-bit elements per thread-step (8 bytes); N % 4 == 0.
template <typename T>
__global__ void __launch_bounds__(RQ_THREADS) quant_kernel(const T *__restrict__ x, int8_t *__restrict__ q,
                                                           float *__restrict__ scales, int N) {
    __shared__ float red[32];
    const long long row = blockIdx.x;
    const uint2 *xr = reinterpret_cast<const uint2 *>(x + row * N);
    const int n4 = N >> 2;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const uint2 u = xr[i];
        const float2 a = unpack2<T>(u.x), b = unpack2<T>(u.y);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
    }
    amax = block_max(amax, red);
    const float inv = quant_inv(amax);
    if (threadIdx.x == 0) scales[row] = __fdiv_rn(amax, 127.0f);
    char4 *qr = reinterpret_cast<char4 *>(q + row * N);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const uint2 u = xr[i];
        const float2 a = unpack2<T>(u.x), b = unpack2<T>(u.y);
        qr[i] = make_char4(quant1(a.x, inv), quant1(a.y, inv), quant1(b.x, inv), quant1(b.y, inv));
    }
}

// residual := rnd(x + residual); y = rnd((h * rsqrt(mean(h^2) + eps)) * w); q, scale = quant(y); normed (opt) := y.
template <typename T>
__global__ void __launch_bounds__(RQ_THREADS)
    rms_norm_quant_kernel(const T *__restrict__ x, T *__restrict__ residual, const T *__restrict__ w, float eps,
                          int8_t *__restrict__ q, float *__restrict__ scales, T *__restrict__ normed, int N) {
    extern __shared__ float hbuf[];   // [N] the new residual as float
    __shared__ float red[32];
    const long long row = blockIdx.x;
    const uint2 *xr = reinterpret_cast<const uint2 *>(x + row * N);
    uint2 *rr = reinterpret_cast<uint2 *>(residual + row * N);
    const uint2 *wr = reinterpret_cast<const uint2 *>(w);
    const int n4 = N >> 2;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const uint2 xu = xr[i], ru = rr[i];
        const float2 xa = unpack2<T>(xu.x), xb = unpack2<T>(xu.y), ra = unpack2<T>(ru.x), rb = unpack2<T>(ru.y);
        const float h0 = rnd<T>(xa.x + ra.x), h1 = rnd<T>(xa.y + ra.y), h2 = rnd<T>(xb.x + rb.x),
                    h3 = rnd<T>(xb.y + rb.y);
        rr[i] = make_uint2(pack2<T>(h0, h1), pack2<T>(h2, h3));
        hbuf[4 * i] = h0;
        hbuf[4 * i + 1] = h1;
        hbuf[4 * i + 2] = h2;
        hbuf[4 * i + 3] = h3;
        ss += h0 * h0 + h1 * h1 + h2 * h2 + h3 * h3;
    }
    ss = block_sum(ss, red);
    const float rs = __frsqrt_rn(__fdiv_rn(ss, (float)N) + eps);
    float amax = 0.0f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const uint2 wu = wr[i];
        const float2 wa = unpack2<T>(wu.x), wb = unpack2<T>(wu.y);
        const float y0 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i], rs), wa.x));
        const float y1 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i + 1], rs), wa.y));
        const float y2 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i + 2], rs), wb.x));
        const float y3 = rnd<T>(__fmul_rn(__fmul_rn(hbuf[4 * i + 3], rs), wb.y));
        hbuf[4 * i] = y0;
        hbuf[4 * i + 1] = y1;
        hbuf[4 * i + 2] = y2;
        hbuf[4 * i + 3] = y3;
        if (normed)
            reinterpret_cast<uint2 *>(normed + row * N)[i] = make_uint2(pack2<T>(y0, y1), pack2<T>(y2, y3));
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(y0), fabsf(y1)), fmaxf(fabsf(y2), fabsf(y3))));
    }
    amax = block_max(amax, red);
    const float inv = quant_inv(amax);
    if (threadIdx.x == 0) scales[row] = __fdiv_rn(amax, 127.0f);
    char4 *qr = reinterpret_cast<char4 *>(q + row * N);
    for (int i = threadIdx.x; i < n4; i += blockDim.x)
        qr[i] = make_char4(quant1(hbuf[4 * i], inv), quant1(hbuf[4 * i + 1], inv), quant1(hbuf[4 * i + 2], inv),
                           quant1(hbuf[4 * i + 3], inv));
}

// Register-resident variant for rows of N % 8 == 0 (16-byte aligned, N <= 16384): one CTA of N / 8 / VPT threads
// (64..256) per row, each
// thread holding VPT 16-byte vectors of x, residual and weight, all loads issued before any arithmetic (one memory
// round trip per row, no shared-memory row buffer). Same arithmetic and rounding points as rms_norm_quant_kernel;
// only the float32 summation order of the mean of squares differs (per-thread partials, then warps in order).
template <typename T, int VPT>
__global__ void __launch_bounds__(256)
    rms_norm_quant_vec_kernel(const T *__restrict__ x, T *__restrict__ residual, const T *__restrict__ w, float eps,
                              int8_t *__restrict__ q, float *__restrict__ scales, T *__restrict__ normed, int N) {
    __shared__ float red[32];
    const size_t row = blockIdx.x;
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * N);
    uint4 *rr = reinterpret_cast<uint4 *>(residual + row * N);
    const uint4 *wr = reinterpret_cast<const uint4 *>(w);
    uint4 xv[VPT], rv[VPT], wv[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int i = threadIdx.x + k * blockDim.x;
        xv[k] = xr[i];
        rv[k] = rr[i];
        wv[k] = __ldg(wr + i);
    }
    float h[VPT * 8];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t xs[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
        const uint32_t rs_[4] = {rv[k].x, rv[k].y, rv[k].z, rv[k].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 a = unpack2<T>(xs[e]), b = unpack2<T>(rs_[e]);
            const float h0 = rnd<T>(a.x + b.x), h1 = rnd<T>(a.y + b.y);
            h[8 * k + 2 * e] = h0;
            h[8 * k + 2 * e + 1] = h1;
            ss += h0 * h0 + h1 * h1;
            o[e] = pack2<T>(h0, h1);
        }
        rr[threadIdx.x + k * blockDim.x] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    ss = block_sum(ss, red);
    const float rs = __frsqrt_rn(__fdiv_rn(ss, (float)N) + eps);
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t ws[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 wf = unpack2<T>(ws[e]);
            const float y0 = rnd<T>(__fmul_rn(__fmul_rn(h[8 * k + 2 * e], rs), wf.x));
            const float y1 = rnd<T>(__fmul_rn(__fmul_rn(h[8 * k + 2 * e + 1], rs), wf.y));
            h[8 * k + 2 * e] = y0;
            h[8 * k + 2 * e + 1] = y1;
            amax = fmaxf(amax, fmaxf(fabsf(y0), fabsf(y1)));
            o[e] = pack2<T>(y0, y1);
        }
        if (normed)
            reinterpret_cast<uint4 *>(normed + row * N)[threadIdx.x + k * blockDim.x] = make_uint4(o[0], o[1], o[2],
                                                                                                   o[3]);
    }
    amax = block_max(amax, red);
    const float inv = quant_inv(amax);
    if (threadIdx.x == 0) scales[row] = __fdiv_rn(amax, 127.0f);
    uint2 *qr = reinterpret_cast<uint2 *>(q + row * N);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        uint32_t b[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const float *v = &h[8 * k + 4 * hh];
            b[hh] = (uint32_t)(uint8_t)quant1(v[0], inv) | ((uint32_t)(uint8_t)quant1(v[1], inv) << 8) |
                    ((uint32_t)(uint8_t)quant1(v[2], inv) << 16) | ((uint32_t)(uint8_t)quant1(v[3], inv) << 24);
        }
        qr[threadIdx.x + k * blockDim.x] = make_uint2(b[0], b[1]);
    }
}

// SiLU(g) * u of elements [i0, i1) of one row into pbuf[0 ..), returning this thread's max |p|; same rounding points
// as below. When the range and rows are 16-byte aligned: 8-element vector loads, a thread's (up to 4) vectors of gate
// and up issued before any arithmetic -- the loop is latency-bound otherwise, one memory round trip per element.
template <typename T>
__device__ __forceinline__ float silu_range(const T *gr, const T *ur, int i0, int i1, float *pbuf) {
    float amax = 0.0f;
    if (((i0 | i1) & 7) == 0 && !((uintptr_t)gr & 15) && !((uintptr_t)ur & 15)) {
        const int nv = (i1 - i0) >> 3, nt = blockDim.x;
        const uint4 *gv = reinterpret_cast<const uint4 *>(gr + i0), *uv = reinterpret_cast<const uint4 *>(ur + i0);
        for (int b = threadIdx.x; b < nv; b += 4 * nt) {
            uint4 gq[4], uq[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (b + k * nt < nv) {
                    gq[k] = gv[b + k * nt];
                    uq[k] = uv[b + k * nt];
                }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int v = b + k * nt;
                if (v >= nv) continue;
                const uint32_t gw[4] = {gq[k].x, gq[k].y, gq[k].z, gq[k].w};
                const uint32_t uw[4] = {uq[k].x, uq[k].y, uq[k].z, uq[k].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 gf = unpack2<T>(gw[e]), uf = unpack2<T>(uw[e]);
                    const float p0 = rnd<T>(__fmul_rn(rnd<T>(__fdiv_rn(gf.x, 1.0f + expf(-gf.x))), uf.x));
                    const float p1 = rnd<T>(__fmul_rn(rnd<T>(__fdiv_rn(gf.y, 1.0f + expf(-gf.y))), uf.y));
                    pbuf[8 * v + 2 * e] = p0;
                    pbuf[8 * v + 2 * e + 1] = p1;
                    amax = fmaxf(amax, fmaxf(fabsf(p0), fabsf(p1)));
                }
            }
        }
        return amax;
    }
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float gf = t2f<T>(gr[i]);
        const float sg = rnd<T>(__fdiv_rn(gf, 1.0f + expf(-gf)));
        const float p = rnd<T>(__fmul_rn(sg, t2f<T>(ur[i])));
        pbuf[i - i0] = p;
        amax = fmaxf(amax, fabsf(p));
    }
    return amax;
}

// SiLU(g) rounded to the 16-bit type, times u rounded (vllm_turing/csrc/silu_quant.cu:11-14, 39), then quant.
template <typename T>
__global__ void __launch_bounds__(RQ_THREADS) silu_mul_quant_kernel(const T *__restrict__ gu, int8_t *__restrict__ q,
                                                                    float *__restrict__ scales, int I) {
    extern __shared__ float abuf[];
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();   // gate_up comes from the previous kernel
    const long long row = blockIdx.x;
    const T *g = gu + row * 2 * I;
    const T *u = g + I;
    float amax = silu_range<T>(g, u, 0, I, abuf);
    amax = block_max(amax, red);
    const float inv = quant_inv(amax);
    if (threadIdx.x == 0) scales[row] = __fdiv_rn(amax, 127.0f);
    for (int i = threadIdx.x; i < I; i += blockDim.x) q[row * I + i] = quant1(abuf[i], inv);
}

// Row-split variant for few rows: CTA (m, g) of an M x E grid computes the SiLU products of the g-th 1/E slice of
// row m; the row's absmax is combined across its E CTAs through one 8-byte word per CTA, {max |p| bits, tag}, tagged
// with the row's epoch + 1 (value and tag in one store: no atomics, no fence). Every CTA of the row polls the row's E
// words in parallel (one round trip once they are all in), takes the maximum (order-independent: deterministic) and
// quantises its own slice; CTA (m, 0) advances the row's epoch after it has seen all E words -- every CTA of the row
// has read the old epoch by then -- so an earlier call's words are never taken for this call's. Calls that overlap on
// the GPU would share the words: they must be stream-ordered (as every decode step is). The wait is bounded; a
// timeout lands in the library status word. Launched with programmatic dependent launch (it waits for the kernel
// that wrote gate_up before reading it).
constexpr int SQ_THREADS = 256;
constexpr int SQ_ROWS = 64;      // rows the split path serves
constexpr int SQ_MAX_E = 64;     // CTAs per row
static __device__ unsigned g_sq_epoch[SQ_ROWS];
static __device__ unsigned long long g_sq_word[SQ_ROWS][SQ_MAX_E];

template <typename T>
__global__ void __launch_bounds__(SQ_THREADS)
    silu_mul_quant_split_kernel(const T *__restrict__ gu, int8_t *__restrict__ q, float *__restrict__ scales, int I,
                                int E, uint64_t timeout_ns, unsigned *status) {
    extern __shared__ float pbuf[];
    __shared__ float red[32];
    __shared__ unsigned s_tag, s_max;
    pdl_launch_dependents();
    pdl_wait();   // gate_up comes from the previous kernel
    const int m = blockIdx.x / E, g = blockIdx.x - m * E;
    if (threadIdx.x == 0) {
        s_tag = *reinterpret_cast<volatile unsigned *>(&g_sq_epoch[m]) + 1u;
        s_max = 0u;
    }
    int i0, i1;
    if ((I & 7) == 0) {   // slices in whole 8-element vectors
        i0 = (int)((long long)(I >> 3) * g / E) * 8;
        i1 = (int)((long long)(I >> 3) * (g + 1) / E) * 8;
    } else {
        i0 = (int)((long long)I * g / E);
        i1 = (int)((long long)I * (g + 1) / E);
    }
    const T *gr = gu + (size_t)m * 2 * I;
    const T *ur = gr + I;
    float amax = silu_range<T>(gr, ur, i0, i1, pbuf);
    amax = block_max(amax, red);   // (its barriers also publish s_tag)
    const unsigned tag = s_tag;
    if (threadIdx.x == 0)
        st_volatile8(&g_sq_word[m][g], ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(amax));
    const uint64_t deadline = globaltimer() + timeout_ns;
    for (int k = threadIdx.x; k < E; k += blockDim.x) {
        unsigned long long x = ld_volatile8(&g_sq_word[m][k]);
        uint32_t it = 0;
        while ((unsigned)(x >> 32) != tag) {
            if ((++it & 63u) == 0 && globaltimer() > deadline) {
                report(status, ST_GROUP_TIMEOUT | 0x800000u | (unsigned)m);
                break;
            }
            x = ld_volatile8(&g_sq_word[m][k]);
        }
        atomicMax(&s_max, (unsigned)(x & 0xffffffffu));   // shared memory; |p| bits: order-independent
    }
    __syncthreads();
    amax = __uint_as_float(s_max);
    if (g == 0 && threadIdx.x == 0) g_sq_epoch[m] = tag;   // every CTA of the row has read the old epoch
    const float inv = quant_inv(amax);
    if (g == 0 && threadIdx.x == 0) scales[m] = __fdiv_rn(amax, 127.0f);
    int8_t *qr = q + (size_t)m * I;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) qr[i] = quant1(pbuf[i - i0], inv);
}

static int smem_attr(const void *fn, int bytes) {
    if (bytes <= 48 * 1024) return 0;
    return (int)cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace vt

using namespace vt;

namespace vt {

template <typename T>
static int launch_norm_vec(int vpt, int t, const void *x, void *residual, const void *weight, float eps, void *q,
                           void *scales, void *normed, int M, int N, cudaStream_t s) {
    const T *xp = (const T *)x;
    const T *wp = (const T *)weight;
    T *rp = (T *)residual, *np = (T *)normed;
    int8_t *qp = (int8_t *)q;
    float *sp = (float *)scales;
    switch (vpt) {
        case 8: rms_norm_quant_vec_kernel<T, 8><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        case 7: rms_norm_quant_vec_kernel<T, 7><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        case 6: rms_norm_quant_vec_kernel<T, 6><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        case 5: rms_norm_quant_vec_kernel<T, 5><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        case 4: rms_norm_quant_vec_kernel<T, 4><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        case 3: rms_norm_quant_vec_kernel<T, 3><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        case 2: rms_norm_quant_vec_kernel<T, 2><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
        default: rms_norm_quant_vec_kernel<T, 1><<<M, t, 0, s>>>(xp, rp, wp, eps, qp, sp, np, N); break;
    }
    return (int)cudaGetLastError();
}

// Few rows: the row-split kernel (about 2048 products per CTA, at most one CTA per SM); else a CTA per row.
template <typename T>
static int launch_silu(const void *gu, void *q, void *scales, int M, int I, cudaStream_t s) {
    const int dev = cur_device();
    const int sms = num_sms(dev);
    // About 1024 products per CTA, and no split into fewer than 4 (then one CTA per row: no cross-CTA step at all).
    // Measured (M = 5, graph replay, us per call; I = 17408 / 8704 / 4352 / 2176): 1024 per CTA 4.24 / 3.73 / 3.38 /
    // (E = 2) 3.30; 2048 per CTA 4.40 / 4.09 / (E = 2) 4.04 / 2.42; one CTA per row 7.48 / 4.61 / 3.33 / 2.47.
    static int per_cta = -1;   // VLLM_TURING_SILU_SPLIT: products per CTA of the row split
    if (per_cta < 0) {
        const char *e = getenv("VLLM_TURING_SILU_SPLIT");
        per_cta = e && atoi(e) > 0 ? atoi(e) : 1024;
    }
    int E = sms / M;
    int E_want = I / per_cta;
    if (E_want < 4) E_want = 1;
    if (E > E_want) E = E_want;
    if (E > SQ_MAX_E) E = SQ_MAX_E;
    if (M <= SQ_ROWS && E >= 2) {
        const int chunk = ((I + 7) / 8 + E - 1) / E * 8 + 8;   // the largest slice, vector-aligned slices included
        static bool attr[VT_MAX_DEV] = {false};
        if (dev >= 0 && dev < VT_MAX_DEV && !attr[dev]) {
            if (int rc = smem_attr((const void *)silu_mul_quant_split_kernel<T>, 100 * 1024)) return rc;
            attr[dev] = true;
        }
        void *scratch = nullptr;
        unsigned *status = nullptr;
        if (ws_acquire(0, s, &scratch, &status) != 0) status = nullptr;   // timeouts reported only with a workspace
        return launch_k(silu_mul_quant_split_kernel<T>, dim3(M * E), dim3(SQ_THREADS), (size_t)chunk * 4, s, true,
                        (const T *)gu, (int8_t *)q, (float *)scales, I, E, pipe_timeout_ns(), status);
    }
    if (int rc = smem_attr((const void *)silu_mul_quant_kernel<T>, I * 4)) return rc;
    return launch_k(silu_mul_quant_kernel<T>, dim3(M), dim3(RQ_THREADS), (size_t)I * 4, s, true, (const T *)gu,
                    (int8_t *)q, (float *)scales, I);
}

}  // namespace vt

using namespace vt;

extern "C" {

// x [M, N] fp16/bf16 (dtype 0/1) -> q int8 [M, N], scales float32 [M]. N % 4 == 0, 8-byte aligned rows.
int vt_scaled_int8_quant(const void *x, void *q, void *scales, int M, int N, int dtype, void *stream) {
    if (M < 0 || N <= 0 || (N & 3) || ((uintptr_t)x & 7) || ((uintptr_t)q & 3)) return VT_EARG;
    if (M == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == 0)
        quant_kernel<__half><<<M, RQ_THREADS, 0, s>>>((const __half *)x, (int8_t *)q, (float *)scales, N);
    else
        quant_kernel<__nv_bfloat16><<<M, RQ_THREADS, 0, s>>>((const __nv_bfloat16 *)x, (int8_t *)q, (float *)scales,
                                                             N);
    return (int)cudaGetLastError();
}

// residual [M, N] updated in place to x + residual; q int8 [M, N] and scales [M] of RMSNorm(x + residual) * weight;
// normed [M, N] (optional, NULL to skip) receives the normalised rows. N % 4 == 0, N <= 49152.
int vt_rms_norm_quant(const void *x, void *residual, const void *weight, float eps, void *q, void *scales,
                      void *normed, int M, int N, int dtype, void *stream) {
    if (M < 0 || N <= 0 || (N & 3) || N > 49152 || ((uintptr_t)x & 7) || ((uintptr_t)residual & 7) ||
        ((uintptr_t)weight & 7) || ((uintptr_t)q & 3) || ((uintptr_t)normed & 7))
        return VT_EARG;
    if (M == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    if ((N & 7) == 0 && !((uintptr_t)x & 15) && !((uintptr_t)residual & 15) && !((uintptr_t)weight & 15) &&
        !((uintptr_t)normed & 15) && !((uintptr_t)q & 7)) {
        const int nv = N / 8;
        for (int vpt = 8; vpt >= 1; --vpt) {   // threads = nv / vpt: a multiple of 32 in [64, 256]
            if (nv % vpt) continue;
            const int t = nv / vpt;
            if ((t & 31) || t < 64 || t > 256) continue;
            return dtype == 0 ? launch_norm_vec<__half>(vpt, t, x, residual, weight, eps, q, scales, normed, M, N, s)
                              : launch_norm_vec<__nv_bfloat16>(vpt, t, x, residual, weight, eps, q, scales, normed, M,
                                                               N, s);
        }
    }
    const int sm = N * 4;
    if (dtype == 0) {
        if (int rc = smem_attr((const void *)rms_norm_quant_kernel<__half>, sm)) return rc;
        rms_norm_quant_kernel<__half><<<M, RQ_THREADS, sm, s>>>((const __half *)x, (__half *)residual,
                                                                (const __half *)weight, eps, (int8_t *)q,
                                                                (float *)scales, (__half *)normed, N);
    } else {
        if (int rc = smem_attr((const void *)rms_norm_quant_kernel<__nv_bfloat16>, sm)) return rc;
        rms_norm_quant_kernel<__nv_bfloat16><<<M, RQ_THREADS, sm, s>>>(
            (const __nv_bfloat16 *)x, (__nv_bfloat16 *)residual, (const __nv_bfloat16 *)weight, eps, (int8_t *)q,
            (float *)scales, (__nv_bfloat16 *)normed, N);
    }
    return (int)cudaGetLastError();
}

// The reference's ABI (vllm_turing/csrc/silu_quant.cu:71-77): gate_up (M, 2I) fp16 -> q (M, I) int8, scales (M).
// Returns 1 on bad arguments, 2 on a launch error.
int silu_mul_quant(const void *gu, void *q, void *scales, int M, int I, void *stream) {
    if (I <= 0 || I > 49152 || M < 0) return 1;
    if (M == 0) return 0;
    return launch_silu<__half>(gu, q, scales, M, I, (cudaStream_t)stream) == 0 ? 0 : 2;
}

// bf16 variant of silu_mul_quant (dtype 0 fp16 / 1 bf16).
int vt_silu_mul_quant(const void *gu, void *q, void *scales, int M, int I, int dtype, void *stream) {
    if (dtype == 0) return silu_mul_quant(gu, q, scales, M, I, stream);
    if (I <= 0 || I > 49152 || M < 0) return VT_EARG;
    if (M == 0) return 0;
    return launch_silu<__nv_bfloat16>(gu, q, scales, M, I, (cudaStream_t)stream);
}

}  // extern "C"

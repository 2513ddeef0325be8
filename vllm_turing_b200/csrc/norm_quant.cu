// Row-wise epilogue kernels for B200 (sm_100a), one CTA per token row, HBM-bound:
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

// SiLU(g) rounded to the 16-bit type, times u rounded (vllm_turing/csrc/silu_quant.cu:11-14, 39), then quant.
template <typename T>
__global__ void __launch_bounds__(RQ_THREADS) silu_mul_quant_kernel(const T *__restrict__ gu, int8_t *__restrict__ q,
                                                                    float *__restrict__ scales, int I) {
    extern __shared__ float abuf[];
    __shared__ float red[32];
    const long long row = blockIdx.x;
    const T *g = gu + row * 2 * I;
    const T *u = g + I;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < I; i += blockDim.x) {
        const float gf = t2f<T>(g[i]);
        const float sg = rnd<T>(__fdiv_rn(gf, 1.0f + expf(-gf)));
        const float p = rnd<T>(__fmul_rn(sg, t2f<T>(u[i])));
        abuf[i] = p;
        amax = fmaxf(amax, fabsf(p));
    }
    amax = block_max(amax, red);
    const float inv = quant_inv(amax);
    if (threadIdx.x == 0) scales[row] = __fdiv_rn(amax, 127.0f);
    for (int i = threadIdx.x; i < I; i += blockDim.x) q[row * I + i] = quant1(abuf[i], inv);
}

static int smem_attr(const void *fn, int bytes) {
    if (bytes <= 48 * 1024) return 0;
    return (int)cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
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
    if (I <= 0 || I > 49152) return 1;
    if (M == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (smem_attr((const void *)silu_mul_quant_kernel<__half>, I * 4)) return 2;
    silu_mul_quant_kernel<__half><<<M, RQ_THREADS, I * 4, s>>>((const __half *)gu, (int8_t *)q, (float *)scales, I);
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// bf16 variant of silu_mul_quant (dtype 0 fp16 / 1 bf16).
int vt_silu_mul_quant(const void *gu, void *q, void *scales, int M, int I, int dtype, void *stream) {
    if (dtype == 0) return silu_mul_quant(gu, q, scales, M, I, stream);
    if (I <= 0 || I > 49152) return VT_EARG;
    if (M == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (int rc = smem_attr((const void *)silu_mul_quant_kernel<__nv_bfloat16>, I * 4)) return rc;
    silu_mul_quant_kernel<__nv_bfloat16><<<M, RQ_THREADS, I * 4, s>>>((const __nv_bfloat16 *)gu, (int8_t *)q,
                                                                      (float *)scales, I);
    return (int)cudaGetLastError();
}

}  // extern "C"

// The compressed all-reduce of the reference (AR8, vllm_turing/csrc/host_ar.cu:133-201, switched on by
// VLLM_TURING_AR8=1 in vllm_turing/hostar.py:40-44): each rank quantises its fp16 operand to int8 with one fp16 scale
// per 128-element group, the packed blocks are all-gathered, and every rank sums the dequantised blocks of all ranks
// (its own included) in rank order, so the result is identical on every rank. Lossy, and off unless asked for.
//
// Packed block of n elements (n % 128 == 0): n int8, then n / 128 fp16 scales (n + n / 64 bytes).
//   quant:   amax = max |x| over the group; sc = fp16(amax / 127); inv = sc > 0 ? 1 / fp32(sc) : 0;
//            q = clamp(rint(x * inv), -127, 127)                                        (host_ar.cu:138-160)
//   dequant: out = fp16(sum over ranks r in order of q_r * sc_r), fp32 additions      (host_ar.cu:163-180)
// Each product q * sc is exact in fp32 (8 and 11 significant bits), so with two ranks the single fp32 addition
// rounds exactly as the reference's `u * a0 + w * a1` does, contracted or not.
//
// Both kernels are HBM / NVLink-side elementwise passes: 16-byte loads (8 fp16 or 8 bytes of int8 per thread per
// rank), a grid of whole waves over the SMs, one 16-lane shuffle reduction per group for the maximum.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "host_util.h"

namespace vt {

constexpr int AR8_THREADS = 256;
constexpr int AR8_MAX_RANKS = 8;

// 16 threads per 128-element group, 8 elements per thread
__global__ void __launch_bounds__(AR8_THREADS) ar8_quant_kernel(const __half *__restrict__ x, int8_t *__restrict__ q,
                                                                __half *__restrict__ s, long long ngroups) {
    const long long stride = (long long)gridDim.x * blockDim.x;   // a multiple of 32
    const long long total = ngroups * 16;                           // a multiple of 16: half-warps are all in or out
    const int lane = threadIdx.x & 31;
    // warp-uniform loop (the shuffles below take the whole warp); a group is one half-warp
    for (long long tw = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31); tw < total; tw += stride) {
        const long long t = tw + lane;
        const bool act = t < total;
        const uint4 raw = act ? *reinterpret_cast<const uint4 *>(x + t * 8) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        float v[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[j]));
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
        }
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const __half sh = __float2half_rn(__fdiv_rn(amax, 127.0f));
        const float sc = __half2float(sh);
        const float inv = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float r = fmaxf(-127.0f, fminf(127.0f, rintf(__fmul_rn(v[j], inv))));
            packed[j >> 2] |= ((uint32_t)(int)r & 0xffu) << (8 * (j & 3));
        }
        if (!act) continue;
        *reinterpret_cast<uint2 *>(q + t * 8) = make_uint2(packed[0], packed[1]);
        if ((t & 15) == 0) s[t >> 4] = sh;
    }
}

// 8 elements per thread; gathered = world packed blocks of n + n / 64 bytes in rank order
__global__ void __launch_bounds__(AR8_THREADS) ar8_dequant_sum_kernel(const int8_t *__restrict__ gathered,
                                                                      __half *__restrict__ out, long long n,
                                                                      int world) {
    const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long blk = n + n / 64;
    for (long long t = t0; t < n / 8; t += stride) {
        const long long g = t >> 4;   // 16 eight-element units per group
        uint2 qv[AR8_MAX_RANKS];
        float sc[AR8_MAX_RANKS];
#pragma unroll
        for (int r = 0; r < AR8_MAX_RANKS; ++r) {   // every rank's loads in flight before the arithmetic
            if (r >= world) break;
            const int8_t *b = gathered + r * blk;
            qv[r] = *reinterpret_cast<const uint2 *>(b + t * 8);
            sc[r] = __half2float(reinterpret_cast<const __half *>(b + n)[g]);
        }
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t w0 = j < 4 ? qv[0].x : qv[0].y;
            acc[j] = __fmul_rn((float)(int8_t)(w0 >> (8 * (j & 3))), sc[0]);
        }
#pragma unroll
        for (int r = 1; r < AR8_MAX_RANKS; ++r) {
            if (r >= world) break;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t wr = j < 4 ? qv[r].x : qv[r].y;
                acc[j] = __fadd_rn(acc[j], __fmul_rn((float)(int8_t)(wr >> (8 * (j & 3))), sc[r]));
            }
        }
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
            o[j] = *reinterpret_cast<const uint32_t *>(&h);
        }
        *reinterpret_cast<uint4 *>(out + t * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// One element per thread, byte and 2-byte accesses: for n % 512 != 0, where rank r's block (n + n / 64 bytes) does
// not start 8-byte aligned. Same arithmetic and order as ar8_dequant_sum_kernel.
__global__ void __launch_bounds__(AR8_THREADS) ar8_dequant_sum_scalar_kernel(const int8_t *__restrict__ gathered,
                                                                             __half *__restrict__ out, long long n,
                                                                             int world) {
    const long long blk = n + n / 64;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float acc = 0.0f;
        for (int r = 0; r < world; ++r) {
            const int8_t *b = gathered + r * blk;
            const float v = __fmul_rn((float)b[i], __half2float(reinterpret_cast<const __half *>(b + n)[i >> 7]));
            acc = r == 0 ? v : __fadd_rn(acc, v);
        }
        out[i] = __float2half_rn(acc);
    }
}

static int ar8_grid(long long threads) {
    const int sms = num_sms(cur_device());
    long long g = (threads + AR8_THREADS - 1) / AR8_THREADS;
    const long long cap = (long long)sms * 8;   // whole waves: 8 resident CTAs of 256 threads per SM
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

}  // namespace vt

using namespace vt;

extern "C" {

// The reference's AR8 quantiser (host_ar.cu:182-188): x fp16 [n], n % 128 == 0; packed = n int8 then n / 128 fp16
// scales. x 16-byte aligned, packed 8-byte aligned with n / 128 scales at packed + n.
int ar8_quant(const void *x, void *packed, int n, void *stream) {
    if (!x || !packed || n <= 0 || (n % 128) || ((uintptr_t)x & 15) || ((uintptr_t)packed & 7)) return VT_EARG;
    const long long ng = n / 128;
    ar8_quant_kernel<<<ar8_grid(ng * 16), AR8_THREADS, 0, (cudaStream_t)stream>>>(
        (const __half *)x, (int8_t *)packed, (__half *)((int8_t *)packed + n), ng);
    return (int)cudaGetLastError();
}

// AR8 dequantise-and-sum over `world` packed blocks (n + n / 64 bytes each, rank order) into out fp16 [n]; 1..8 ranks,
// n % 128 == 0. With n % 512 == 0 (every block then starts 8-byte aligned; prefill messages M x 5120 always are),
// gathered 8-byte and out 16-byte aligned, the vectorised kernel; otherwise one element per thread. New entry (the
// reference's two-rank form is ar8_dequant_sum).
int vt_ar8_dequant_sum(const void *gathered, void *out, long long n, int world, void *stream) {
    if (!gathered || !out || n <= 0 || (n % 128) || world < 1 || world > AR8_MAX_RANKS || ((uintptr_t)out & 1) ||
        ((uintptr_t)gathered & 1))
        return VT_EARG;
    if ((n % 512) == 0 && !((uintptr_t)out & 15) && !((uintptr_t)gathered & 7)) {
        ar8_dequant_sum_kernel<<<ar8_grid(n / 8), AR8_THREADS, 0, (cudaStream_t)stream>>>((const int8_t *)gathered,
                                                                                        (__half *)out, n, world);
    } else {
        ar8_dequant_sum_scalar_kernel<<<ar8_grid(n), AR8_THREADS, 0, (cudaStream_t)stream>>>(
            (const int8_t *)gathered, (__half *)out, n, world);
    }
    return (int)cudaGetLastError();
}

// The reference's two-rank AR8 sum (host_ar.cu:190-201): n % 128 == 0, as there.
int ar8_dequant_sum(const void *gathered, void *out, int n, void *stream) {
    return vt_ar8_dequant_sum(gathered, out, n, 2, stream);
}

}  // extern "C"

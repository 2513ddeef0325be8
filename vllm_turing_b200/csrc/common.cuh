// Shared device helpers for the sm_100a kernels of vllm_turing_b200: shared-memory barriers (mbarrier) and 1-D bulk
// copies (cp.async.bulk, the TMA engine without a tensor map), LL words for cross-GPU signalling, bounded waits and the
// device status word every kernel reports a timeout into.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vt {

// ---- status codes written into the device status word (first error wins) -------------------------------------------
enum Status : unsigned {
    ST_OK = 0,
    ST_PIPE_TIMEOUT = 0x01000000u,      // a shared-memory pipeline wait (bulk copy / MMA completion) gave up
    ST_PEER_TIMEOUT = 0x02000000u,      // a peer rank's data (LL words) did not arrive in time
    ST_GROUP_TIMEOUT = 0x03000000u,     // a cooperating CTA of the same grid did not publish in time
    ST_TMEM_FAIL = 0x04000000u,         // tensor-memory allocation failed
};

__device__ __forceinline__ void report(unsigned *status, unsigned code) {
    if (status) atomicCAS(status, 0u, code);
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ---- mbarrier -------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of `parity` to complete; false once globaltimer passes `deadline` (ns). The timer is read only
// every 1024 polls: reading %globaltimer costs far more than a poll and would throttle the pipeline it bounds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    uint32_t it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++it & 1023u) == 0 && globaltimer() > deadline) return false;
    }
    return true;
}

// The same for a waiter off the critical path (e.g. an epilogue waiting out a whole tile's K range): it sleeps
// between polls, leaving the issue slots and the integer pipe of its SM sub-partition to the warps doing the work.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint64_t deadline, uint32_t ns) {
    uint32_t it = 0;
    while (!mbar_try_wait(bar, parity)) {
        __nanosleep(ns);
        if ((++it & 63u) == 0 && globaltimer() > deadline) return false;
    }
    return true;
}

// ---- 1-D bulk copy global -> shared (TMA engine), completion counted in bytes on an mbarrier -------------------------
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Same, with an L2 evict-first hint: streamed weights are read once per call.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---- 2-D TMA tensor load (no multicast): box at coordinates (x = innermost, bytes for int8; y = rows) ------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// L2 prefetch of one 2-D box (no shared memory, no completion to wait for; same coordinates as tma_load_2d)
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- programmatic dependent launch (griddepcontrol; no-ops when the grid was launched without the attribute) -------
// pdl_wait: returns once the preceding grid in the stream has completed and its memory is visible; every global access
// to data an earlier kernel produces or still reads comes after it. pdl_launch_dependents: lets the next grid in the
// stream be scheduled (onto SMs as they free up) before this one ends; its own pdl_wait keeps it correct.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- named barrier among a subset of warps ---------------------------------------------------------------------------
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- LL words: 16 bytes = {data0, flag, data1, flag}; each 8-byte half is written atomically, so a reader that sees
// both flags equal to the call's sequence number holds that call's 8 data bytes (no fences, one store per word) -------
__device__ __forceinline__ void ll_store(void *p, uint32_t d0, uint32_t d1, uint32_t seq) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(d0), "r"(seq), "r"(d1), "r"(seq)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_volatile16(const void *p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_volatile8(void *p, unsigned long long v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile8(const void *p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Polls an LL word until both flags carry `seq`; false on timeout.
__device__ __forceinline__ bool ll_wait(const void *p, uint32_t seq, uint64_t deadline, uint2 &data) {
    uint4 v = ld_volatile16(p);
    uint32_t it = 0;
    while (v.y != seq || v.w != seq) {
        if ((++it & 255u) == 0 && globaltimer() > deadline) return false;
        v = ld_volatile16(p);
    }
    data = make_uint2(v.x, v.z);
    return true;
}

// ---- 16-bit float conversions ----------------------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ T f2t(float x);
template <> __device__ __forceinline__ __half f2t<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 f2t<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <typename T> __device__ __forceinline__ float t2f(T x);
template <> __device__ __forceinline__ float t2f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float t2f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// two 16-bit values packed in a 32-bit word <-> floats (element 0 in the low half)
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t u) {
    const T *h = reinterpret_cast<const T *>(&u);
    return make_float2(t2f<T>(h[0]), t2f<T>(h[1]));
}
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b) {
    T h[2] = {f2t<T>(a), f2t<T>(b)};
    return *reinterpret_cast<uint32_t *>(h);
}
template <typename T> __device__ __forceinline__ float rnd(float x) { return t2f<T>(f2t<T>(x)); }

// ---- the reference's per-token quantisation of one value (vllm_turing/quantfuse.py:18-24) ----------------------------
// inv = (1 / absmax) * 127 in two float32 roundings: torch evaluates `127.0 / absmax` as absmax.reciprocal() * 127.
__device__ __forceinline__ float quant_inv(float amax) {
    return amax > 0.0f ? __fmul_rn(__frcp_rn(amax), 127.0f) : 0.0f;
}
__device__ __forceinline__ int8_t quant1(float y, float inv) {
    float r = rintf(__fmul_rn(y, inv));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return (int8_t)(int)r;
}

// per-token x per-channel dequant of one int32 accumulator, vllm_turing/csrc/w8a8_gemv.cu:91 order
__device__ __forceinline__ float dequant1(int acc, float sa, float sw) { return __fmul_rn(__fmul_rn((float)acc, sa), sw); }
__device__ __forceinline__ float dequant1b(int acc, float sa, float sw, float b) {
    return __fmaf_rn(__fmul_rn((float)acc, sa), sw, b);
}

}  // namespace vt

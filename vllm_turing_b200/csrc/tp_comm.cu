// Tensor-parallel collectives over NVLink 5 / NVSwitch peer memory for B200 (sm_100a), N = 1..8 ranks, one process
// per GPU. No NCCL on the path: kernels load and store peers' IPC-mapped regions directly.
//
//   one-shot (decode messages): every rank pushes its message as 16-byte LL words {4 data bytes, seq, 4 data bytes,
//     seq} into every rank's receive slot, then polls its own slot and sums the ranks in rank order (float32, one
//     rounding). The reference's two-rank LL kernel (vllm_turing/csrc/host_ar.cu:31-82) generalised to N ranks with
//     16-byte stores and bounded waits.
//   two-shot (prefill messages): reduce-scatter by chunk ownership (rank c owns chunk c; peers push their slice of it
//     into c's receive buffers, then a release flag), the owner sums in rank order and pushes the reduced chunk into
//     every peer's all-gather receive buffer as it goes (NVLink stores in flight with the reduction), then a flag;
//     every rank copies the peers' reduced chunks out locally. The N-rank SM version of the reference's copy-engine
//     all-reduce (vllm_turing/csrc/ce_ar.cu:103-146: push half, flag, wait, add, push, flag, wait). (Pulling the
//     reduced chunks after the reduction instead put an NVLink load latency on every unit of the all-gather.)
//   all-gather: each rank's slot of `gathered` is pre-written by the caller and the kernel fills the peers' slots
//     (the ABI idea of vllm_turing/csrc/dma_ag.cu:41-47, over P2P for N ranks instead of host staging for two).
//
// Exports (include/vllm_turing_b200.h): ce_alloc, ce_open, ce_close, ce_free, ce_enable_peer (the reference's IPC
// helpers, vllm_turing/csrc/ce_ar.cu:75-101), vt_comm_* (communicator objects), vt_all_reduce, vt_all_gather.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "comm.cuh"
#include "common.cuh"
#include "host_util.h"

namespace vt {

constexpr int AR_THREADS = 512;

// ---- one-shot LL all-reduce -------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(AR_THREADS) ar_oneshot_kernel(CommView c, const uint2 *in, uint2 *out,
                                                                long long nwords,
                                                                uint64_t timeout) {
    __shared__ unsigned s_seq;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t deadline = globaltimer() + timeout;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (long long i = i0; i < nwords; i += stride) {
        const uint2 d = in[i];
        for (int k = 0; k < c.world; ++k) {
            const int dst = (c.rank + k) % c.world;   // staggered: ranks do not all hit the same peer first
            ll_store(c.ll_slot(dst, p, c.rank) + i * 16, d.x, d.y, seq);
        }
    }
    bool dead = false;
    for (long long i = i0; i < nwords; i += stride) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int r = 0; r < c.world; ++r) {
            uint2 d = make_uint2(0u, 0u);
            if (!dead && !ll_wait(c.ll_slot(c.rank, p, r) + i * 16, seq, deadline, d)) {
                report(c.status(), ST_PEER_TIMEOUT | (unsigned)r);
                dead = true;
            }
            const float2 a = unpack2<T>(d.x), b = unpack2<T>(d.y);
            if (r == 0) {
                s0 = a.x; s1 = a.y; s2 = b.x; s3 = b.y;
            } else {
                s0 += a.x; s1 += a.y; s2 += b.x; s3 += b.y;
            }
        }
        out[i] = make_uint2(pack2<T>(s0, s1), pack2<T>(s2, s3));
    }
    comm_end(c, seq);
}

// ---- two-shot all-reduce (reduce-scatter + all-gather) -------------------------------------------------------------
// n elements in 16-byte units (8 elements); chunk k = units [k U / N, (k + 1) U / N); CTA j handles slice j of
// every chunk, so flags are per (source rank, CTA).
__device__ __forceinline__ void slice_of(long long U, int world, int k, int G, int j, long long &cs, long long &b,
                                         long long &e) {
    cs = U * k / world;
    const long long ce = U * (k + 1) / world, len = ce - cs;
    b = cs + len * j / G;
    e = cs + len * (j + 1) / G;
}

template <typename T>
__device__ __forceinline__ void acc8(float (&s)[8], const uint4 &v, bool first) {
    const float2 a = unpack2<T>(v.x), b = unpack2<T>(v.y), cc = unpack2<T>(v.z), d = unpack2<T>(v.w);
    const float f[8] = {a.x, a.y, b.x, b.y, cc.x, cc.y, d.x, d.y};
#pragma unroll
    for (int k = 0; k < 8; ++k) s[k] = first ? f[k] : s[k] + f[k];
}

// dst[u - off] = src[u] for u in [b, e), TS_UNROLL independent loads in flight per thread (NVLink and HBM latency)
constexpr int TS_UNROLL = 4;
__device__ __forceinline__ void copy_units(uint4 *dst, long long off, const uint4 *src, long long b, long long e) {
    const int nt = blockDim.x;
    for (long long u0 = b + threadIdx.x; u0 < e; u0 += (long long)TS_UNROLL * nt) {
        uint4 v[TS_UNROLL];
#pragma unroll
        for (int k = 0; k < TS_UNROLL; ++k)
            if (u0 + k * nt < e) v[k] = src[u0 + k * nt];
#pragma unroll
        for (int k = 0; k < TS_UNROLL; ++k)
            if (u0 + k * nt < e) dst[u0 + k * nt - off] = v[k];
    }
}

template <typename T>
__global__ void __launch_bounds__(AR_THREADS) ar_twoshot_kernel(CommView c, const uint4 *in, uint4 *out,
                                                                long long U,
                                                                uint64_t timeout) {
    __shared__ unsigned s_seq;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t deadline = globaltimer() + timeout;
    const int j = blockIdx.x, G = gridDim.x, tid = threadIdx.x, W = c.world, R = c.rank;
    long long cs, b, e;
    // 1. push my slice j of every peer's chunk into that peer's receive buffer for me
    for (int k = 1; k < W; ++k) {
        const int dst = (R + k) % W;
        slice_of(U, W, dst, G, j, cs, b, e);
        copy_units(reinterpret_cast<uint4 *>(c.rs_buf(dst, p, R)), cs, in, b, e);
    }
    __syncthreads();
    if (tid < W && tid != R) st_release_sys(c.flag(tid, p, 0, R, j), seq);
    // 2. wait for every peer's slice j of my chunk, reduce in rank order, publish
    bool ok = true;
    if (tid < W && tid != R && !flag_wait(c.flag(R, p, 0, tid, j), seq, deadline)) {
        report(c.status(), ST_PEER_TIMEOUT | 0x100u | (unsigned)tid);
        ok = false;
    }
    __syncthreads();
    (void)ok;
    slice_of(U, W, R, G, j, cs, b, e);
    const int nt = blockDim.x;
    for (long long u0 = b + tid; u0 < e; u0 += 2LL * nt) {   // two units per step: 2 x world loads in flight
        uint4 v[2][COMM_MAX_RANKS];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const long long u = u0 + k * nt;
            if (u >= e) continue;
#pragma unroll
            for (int r = 0; r < COMM_MAX_RANKS; ++r)
                if (r < W) v[k][r] = (r == R) ? in[u] : reinterpret_cast<const uint4 *>(c.rs_buf(R, p, r))[u - cs];
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const long long u = u0 + k * nt;
            if (u >= e) continue;
            float s[8];
#pragma unroll
            for (int r = 0; r < COMM_MAX_RANKS; ++r)
                if (r < W) acc8<T>(s, v[k][r], r == 0);   // rank order: identical bits on every rank
            const uint4 o = make_uint4(pack2<T>(s[0], s[1]), pack2<T>(s[2], s[3]), pack2<T>(s[4], s[5]),
                                       pack2<T>(s[6], s[7]));
            out[u] = o;
#pragma unroll
            for (int k2 = 1; k2 < COMM_MAX_RANKS; ++k2) {   // push the reduced slice into every peer (NVLink stores)
                if (k2 >= W) break;
                int dst = R + k2;
                if (dst >= W) dst -= W;
                reinterpret_cast<uint4 *>(c.agr_buf(dst, p, R))[u - cs] = o;
            }
        }
    }
    __syncthreads();
    if (tid < W && tid != R) st_release_sys(c.flag(tid, p, 1, R, j), seq);
    // 3. every peer pushed its reduced slice j into this rank's receive buffer: copy it out (local reads)
    if (tid < W && tid != R && !flag_wait(c.flag(R, p, 1, tid, j), seq, deadline))
        report(c.status(), ST_PEER_TIMEOUT | 0x200u | (unsigned)tid);
    __syncthreads();
    for (int k = 1; k < W; ++k) {
        const int src = (R + k) % W;
        slice_of(U, W, src, G, j, cs, b, e);
        copy_units(out + cs, 0, reinterpret_cast<const uint4 *>(c.agr_buf(R, p, src)), b - cs, e - cs);
    }
    comm_end(c, seq);
}

// ---- all-gather ------------------------------------------------------------------------------------------------------
// LL variant (small payloads). Rank r's payload is `rows` runs of row_bytes (% 8 == 0) at byte offset
// i * ld + r * row_bytes of `gathered` (rows = 1: the contiguous slots [r * m, (r + 1) * m)); its 8-byte words travel
// as LL words in payload order.
__global__ void __launch_bounds__(AR_THREADS) ag_ll_kernel(CommView c, char *__restrict__ gathered, long long rows,
                                                           long long row_bytes, long long ld, uint64_t timeout) {
    __shared__ unsigned s_seq;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t deadline = globaltimer() + timeout;
    const long long wpr = row_bytes >> 3, nw = rows * wpr, stride = (long long)gridDim.x * blockDim.x;
    const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (long long i = i0; i < nw; i += stride) {
        const long long r = i / wpr, j = i - r * wpr;
        const uint2 d = *reinterpret_cast<const uint2 *>(gathered + r * ld + (long long)c.rank * row_bytes + j * 8);
        for (int k = 1; k < c.world; ++k) {
            const int dst = (c.rank + k) % c.world;
            ll_store(c.ll_slot(dst, p, c.rank) + i * 16, d.x, d.y, seq);
        }
    }
    bool dead = false;
    for (long long i = i0; i < nw; i += stride) {
        const long long r = i / wpr, j = i - r * wpr;
        for (int k = 1; k < c.world; ++k) {
            const int src = (c.rank + k) % c.world;
            uint2 d = make_uint2(0u, 0u);
            if (!dead && !ll_wait(c.ll_slot(c.rank, p, src) + i * 16, seq, deadline, d)) {
                report(c.status(), ST_PEER_TIMEOUT | 0x300u | (unsigned)src);
                dead = true;
            }
            *reinterpret_cast<uint2 *>(gathered + r * ld + (long long)src * row_bytes + j * 8) = d;
        }
    }
    comm_end(c, seq);
}

// bulk variant: bytes [off, off + len) of every rank's m-byte slot (m, off, len % 16 == 0, len <= chunk_cap), pushed
// into the peers' receive buffers and flagged per CTA.
__global__ void __launch_bounds__(AR_THREADS) ag_bulk_kernel(CommView c, char *__restrict__ gathered, long long m,
                                                             long long off, long long len, uint64_t timeout) {
    __shared__ unsigned s_seq;
    const unsigned seq = comm_begin(c, &s_seq);
    const unsigned p = seq & 1u;
    const uint64_t deadline = globaltimer() + timeout;
    const int j = blockIdx.x, G = gridDim.x, tid = threadIdx.x, W = c.world, R = c.rank;
    const long long U = len >> 4, b = U * j / G, e = U * (j + 1) / G;
    gathered += off;
    const uint4 *mine = reinterpret_cast<const uint4 *>(gathered + (long long)R * m);
    for (int k = 1; k < W; ++k) {
        const int dst = (R + k) % W;
        uint4 *rb = reinterpret_cast<uint4 *>(c.rs_buf(dst, p, R));
        for (long long u = b + tid; u < e; u += blockDim.x) rb[u] = mine[u];
    }
    __syncthreads();
    if (tid < W && tid != R) st_release_sys(c.flag(tid, p, 0, R, j), seq);
    if (tid < W && tid != R && !flag_wait(c.flag(R, p, 0, tid, j), seq, deadline))
        report(c.status(), ST_PEER_TIMEOUT | 0x400u | (unsigned)tid);
    __syncthreads();
    for (int k = 1; k < W; ++k) {
        const int src = (R + k) % W;
        const uint4 *sb = reinterpret_cast<const uint4 *>(c.rs_buf(R, p, src));
        uint4 *dst = reinterpret_cast<uint4 *>(gathered + (long long)src * m);
        for (long long u = b + tid; u < e; u += blockDim.x) dst[u] = sb[u];
    }
    comm_end(c, seq);
}

// NVLink bandwidth probe: one of this rank's RS buffers -> a peer's RS buffer (the slot of this rank), 16-byte stores with
// TS_UNROLL loads in flight per thread over a grid-stride loop. Touches no flags and no call number.
__global__ void __launch_bounds__(AR_THREADS) peer_push_kernel(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                                               long long U) {
    const long long nt = (long long)gridDim.x * blockDim.x;
    for (long long u0 = (long long)blockIdx.x * blockDim.x + threadIdx.x; u0 < U; u0 += TS_UNROLL * nt) {
        uint4 v[TS_UNROLL];
#pragma unroll
        for (int k = 0; k < TS_UNROLL; ++k)
            if (u0 + k * nt < U) v[k] = src[u0 + k * nt];
#pragma unroll
        for (int k = 0; k < TS_UNROLL; ++k)
            if (u0 + k * nt < U) dst[u0 + k * nt] = v[k];
    }
}

template <typename K>
static void preload(K k) {
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, k);
}

}  // namespace vt

using namespace vt;

extern "C" {

// ---- IPC helpers (the reference's names and semantics, vllm_turing/csrc/ce_ar.cu:77-101) ----------------------------
// A zeroed device buffer and its 64-byte CUDA IPC handle. 0 ok; 1 cudaMalloc, 2 memset, 3 sync, 4 handle failed.
int har_preload(void);   // ref_abi.cu

int ce_alloc(size_t bytes, void **ptr, void *handle) {
    // load the two-rank kernels now (ce_ar.cu:79-81 preloads its add kernel for the same reason: a lazily loaded
    // module's first launch synchronises, behind a peer that may already be spinning)
    if (har_preload() != 0) return 5;
    if (cudaMalloc(ptr, bytes) != cudaSuccess) return 1;
    if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return 2;
    if (cudaDeviceSynchronize() != cudaSuccess) return 3;
    return cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(handle), *ptr) == cudaSuccess ? 0 : 4;
}

int ce_open(const void *handle, void **ptr) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : 1;
}

int ce_close(void *ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : 1; }

int ce_free(void *ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : 1; }

// Single-process multi-GPU use: peer access from the current device to `peer`.
int ce_enable_peer(int peer) {
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return 0;
    }
    return e == cudaSuccess ? 0 : 1;
}

// The bounds of the device-side waits for launches from now on (milliseconds; <= 0 keeps a bound): pipe = waits inside
// one CTA (bulk copies, MMA completion), peer = waits for other CTAs or GPUs. The environment variables
// VLLM_TURING_PIPE_TIMEOUT_MS / VLLM_TURING_AR_TIMEOUT_MS set the initial values. A CUDA graph keeps the bounds its
// kernels were captured with. Returns 0.
int vt_set_wait_bounds(double pipe_ms, double peer_ms) {
    if (pipe_ms > 0) pipe_timeout_slot().store((uint64_t)(pipe_ms * 1e6));
    if (peer_ms > 0) peer_timeout_slot().store((uint64_t)(peer_ms * 1e6));
    return 0;
}

// ---- communicator ------------------------------------------------------------------------------------------------------
size_t vt_comm_region_bytes(int world, size_t ll_data, size_t big_data, size_t scratch_ints) {
    if (world < 1 || world > COMM_MAX_RANKS) return 0;
    return comm_layout(world, ll_data, big_data, scratch_ints).total;
}

// bases[world]: every rank's region (this rank's own at bases[rank], peers' mapped with ce_open), each
// vt_comm_region_bytes(...) bytes and zeroed once. Returns an opaque handle or NULL.
void *vt_comm_create(int rank, int world, void *const *bases, size_t ll_data, size_t big_data, size_t scratch_ints) {
    if (world < 1 || world > COMM_MAX_RANKS || rank < 0 || rank >= world || !bases) return nullptr;
    Comm *c = new Comm();
    memset(&c->v, 0, sizeof(c->v));
    for (int r = 0; r < world; ++r) {
        if (!bases[r]) {
            delete c;
            return nullptr;
        }
        c->v.base[r] = reinterpret_cast<char *>(bases[r]);
    }
    c->v.rank = rank;
    c->v.world = world;
    c->v.L = comm_layout(world, ll_data, big_data, scratch_ints);
    c->dev = cur_device();
    // load every collective kernel now: a lazily loaded module's first launch may synchronise behind a kernel that is
    // already spinning on a peer (vllm_turing/csrc/host_ar.cu:84-92 preloads for the same reason)
    preload(ar_oneshot_kernel<__half>);
    preload(ar_oneshot_kernel<__nv_bfloat16>);
    preload(ar_twoshot_kernel<__half>);
    preload(ar_twoshot_kernel<__nv_bfloat16>);
    preload(ag_ll_kernel);
    preload(ag_bulk_kernel);
    cudaGetLastError();
    return c;
}

int vt_comm_destroy(void *comm) {
    delete reinterpret_cast<Comm *>(comm);
    return 0;
}

// Largest message of each algorithm (bytes).
long long vt_comm_ll_bytes(void *comm) { return (long long)(reinterpret_cast<Comm *>(comm)->v.L.ll_slot / 2); }
long long vt_comm_big_bytes(void *comm) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    return (long long)(c->v.L.chunk_cap * c->v.world);
}

// The communicator's status word (0 or the first timeout code a kernel reported); synchronises the device.
unsigned vt_comm_status(void *comm, int clear) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    unsigned v = 0;
    cudaDeviceSynchronize();
    cudaMemcpy(&v, c->v.base[c->v.rank] + 128, 4, cudaMemcpyDeviceToHost);
    if (clear) cudaMemset(c->v.base[c->v.rank] + 128, 0, 4);
    return v;
}

// The device-side call counter (number of completed collective calls on this communicator).
unsigned vt_comm_seq(void *comm) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    unsigned v = 0;
    cudaDeviceSynchronize();
    cudaMemcpy(&v, c->v.base[c->v.rank], 4, cudaMemcpyDeviceToHost);
    return v;
}

// out[n] = sum over ranks of in[n] (fp16 / bf16: dtype 0 / 1), float32 accumulation in rank order, one rounding.
// algo 0 auto (one-shot up to the LL slot, else two-shot), 1 one-shot, 2 two-shot. in may equal out. n % 4 == 0
// (one-shot) / n % 8 == 0 (two-shot); 16-byte aligned. Returns 0 or VT_EARG or a CUDA error.
int vt_all_reduce(void *comm, const void *in, void *out, long long n, int dtype, int algo, void *stream) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    if (!c || n < 0 || ((uintptr_t)in & 15) || ((uintptr_t)out & 15)) return VT_EARG;
    if (n == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    const long long bytes = n * 2;
    if (c->v.world == 1) {   // a sum over one rank: nothing to do in place, one copy otherwise (no call number used)
        if (in == out) return 0;
        return (int)cudaMemcpyAsync(out, in, (size_t)bytes, cudaMemcpyDeviceToDevice, s);
    }
    const int sms = num_sms(c->dev);
    if (algo == 0) algo = (bytes <= (long long)(c->v.L.ll_slot / 2) && (n & 3) == 0) ? 1 : 2;
    if (algo == 1) {
        if ((n & 3) || bytes > (long long)(c->v.L.ll_slot / 2)) return VT_EARG;
        const long long nwords = n >> 2;
        long long g = (nwords + AR_THREADS - 1) / AR_THREADS;
        if (g > sms) g = sms;
        if (dtype == 0)
            ar_oneshot_kernel<__half><<<(int)g, AR_THREADS, 0, s>>>(c->v, (const uint2 *)in, (uint2 *)out, nwords,
                                                                   peer_timeout_ns());
        else
            ar_oneshot_kernel<__nv_bfloat16><<<(int)g, AR_THREADS, 0, s>>>(c->v, (const uint2 *)in, (uint2 *)out,
                                                                          nwords, peer_timeout_ns());
        return (int)cudaGetLastError();
    }
    if (n & 7) return VT_EARG;
    // pieces of at most world * chunk_cap bytes (chunk boundaries in 16-byte units), one launch (one seq) each
    const long long cap_units = (long long)(c->v.L.chunk_cap / 16) * c->v.world;
    const long long U = n >> 3;
    for (long long u0 = 0; u0 < U; u0 += cap_units) {
        const long long u = (U - u0 < cap_units) ? U - u0 : cap_units;
        long long g = u / (c->v.world * 64);   // >= 64 units (1 KB) per CTA slice
        if (g < 1) g = 1;
        if (g > sms) g = sms;
        if (g > COMM_MAX_CTAS) g = COMM_MAX_CTAS;
        const uint4 *ip = reinterpret_cast<const uint4 *>(in) + u0;
        uint4 *op = reinterpret_cast<uint4 *>(out) + u0;
        if (dtype == 0)
            ar_twoshot_kernel<__half><<<(int)g, AR_THREADS, 0, s>>>(c->v, ip, op, u, peer_timeout_ns());
        else
            ar_twoshot_kernel<__nv_bfloat16><<<(int)g, AR_THREADS, 0, s>>>(c->v, ip, op, u, peer_timeout_ns());
        if (cudaError_t e = cudaGetLastError()) return (int)e;
    }
    return 0;
}

// gathered: world * m bytes, this rank's payload pre-written at [rank * m, (rank + 1) * m); the peers' slots are
// filled. m % 8 == 0 (LL, up to the LL slot and 1 MiB) or m % 16 == 0 (bulk, in pieces of the two-shot chunk
// capacity, one launch each).
int vt_all_gather(void *comm, void *gathered, long long m, void *stream) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    if (!c || m < 0 || ((uintptr_t)gathered & 15)) return VT_EARG;
    if (m == 0 || c->v.world == 1) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    const int sms = num_sms(c->dev);
    if ((m & 7) == 0 && m <= (long long)(c->v.L.ll_slot / 2) && m <= (1 << 20)) {
        const long long nw = m >> 3;
        long long g = (nw + AR_THREADS - 1) / AR_THREADS;
        if (g > sms) g = sms;
        ag_ll_kernel<<<(int)g, AR_THREADS, 0, s>>>(c->v, (char *)gathered, 1, m, m * c->v.world, peer_timeout_ns());
        return (int)cudaGetLastError();
    }
    if (m & 15) return VT_EARG;
    const long long cap = (long long)c->v.L.chunk_cap;
    for (long long off = 0; off < m; off += cap) {
        const long long len = (m - off < cap) ? m - off : cap;
        long long g = (len >> 4) / 64;
        if (g < 1) g = 1;
        if (g > sms) g = sms;
        if (g > COMM_MAX_CTAS) g = COMM_MAX_CTAS;
        ag_bulk_kernel<<<(int)g, AR_THREADS, 0, s>>>(c->v, (char *)gathered, m, off, len, peer_timeout_ns());
        if (cudaError_t e = cudaGetLastError()) return (int)e;
    }
    return 0;
}

// NVLink bandwidth probe (bench.py --mode p2p): copies `bytes` (% 16 == 0, <= the two-shot chunk capacity) from one
// of this rank's RS buffers (parity 1) into one of rank `peer`'s (parity 0), with SM stores (engine 0: grid of `ctas` CTAs, 0 = 4 per SM) or the
// copy engines (engine 1: cudaMemcpyAsync to the IPC-mapped peer address). Not a collective: the caller brackets it
// with barriers and runs no other call on the communicator meanwhile. The copied bytes are meaningless.
int vt_comm_peer_copy(void *comm, int peer, long long bytes, int engine, int ctas, void *stream) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    if (!c || peer < 0 || peer >= c->v.world || bytes <= 0 || (bytes & 15) ||
        bytes > (long long)c->v.L.chunk_cap)
        return VT_EARG;
    const char *src = c->v.base[c->v.rank] + c->v.L.rs_off + ((size_t)c->v.world + c->v.rank) * c->v.L.chunk_cap;
    char *dst = c->v.base[peer] + c->v.L.rs_off + (size_t)c->v.rank * c->v.L.chunk_cap;
    cudaStream_t s = (cudaStream_t)stream;
    if (engine == 1) return (int)cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice, s);
    const int g = ctas > 0 ? ctas : 4 * num_sms(c->dev);
    peer_push_kernel<<<g, AR_THREADS, 0, s>>>((uint4 *)dst, (const uint4 *)src, bytes >> 4);
    return (int)cudaGetLastError();
}

// Row-strided all-gather: gathered [rows, ld_bytes] holds world column blocks of row_bytes per row; this rank's block
// (byte offset rank * row_bytes of every row) is pre-written, the call fills the peers' blocks. The concatenation
// along the last dimension that vLLM's all_gather(dim=-1) builds (logits [M, world * V / world]) without a separate
// transpose. row_bytes % 8 == 0, ld_bytes % 8 == 0, ld_bytes >= world * row_bytes, rows * row_bytes at most the LL
// capacity of the communicator (one-shot LL words; size it with ll_data at creation); larger payloads: VT_EARG (use
// vt_all_gather on contiguous slots).
int vt_all_gather_rows(void *comm, void *gathered, long long rows, long long row_bytes, long long ld_bytes,
                       void *stream) {
    Comm *c = reinterpret_cast<Comm *>(comm);
    if (!c || rows < 0 || row_bytes < 0 || ((uintptr_t)gathered & 7) || (row_bytes & 7) || (ld_bytes & 7) ||
        ld_bytes < (long long)c->v.world * row_bytes)
        return VT_EARG;
    if (rows == 0 || row_bytes == 0 || c->v.world == 1) return 0;
    const long long m = rows * row_bytes;
    if (m > (long long)(c->v.L.ll_slot / 2)) return VT_EARG;
    const long long nw = m >> 3;
    long long g = (nw + AR_THREADS - 1) / AR_THREADS;
    const int sms = num_sms(c->dev);
    if (g > sms) g = sms;
    ag_ll_kernel<<<(int)g, AR_THREADS, 0, (cudaStream_t)stream>>>(c->v, (char *)gathered, rows, row_bytes, ld_bytes,
                                                                   peer_timeout_ns());
    return (int)cudaGetLastError();
}

}  // extern "C"

// The reference's two-rank transport entry points, kept by name, signature and return convention so that its Python
// (vllm_turing/hostar.py, cear.py, dmaag.py) can bind this library unchanged, re-implemented for B200:
//
//   har_preload / har_blocks / har_register / har_unregister / har_all_reduce   (vllm_turing/csrc/host_ar.cu:86-131)
//     the two-rank LL all-reduce over caller-owned regions: this rank's LL words are written to `my_ll` (the peer's
//     receive region over NVLink, or a host-mapped segment), the peer's are polled in `peer_ll`. The region format is
//     the reference's contract (two parity slots of slot_words 8-byte words, each {data word, call number}; one call
//     counter per block in `counters`), which is why it is the reference's; here each thread moves two words per
//     16-byte access where the alignment allows it, and every wait is bounded.
//   ce_driver_ok / ce_all_reduce                                               (vllm_turing/csrc/ce_ar.cu:101-146)
//     the two-rank fp16 all-reduce over two IPC-shared buffers (256 bytes of flags, then receive buffers R1 and R2 of
//     `cap` bytes). The reference drives copy engines and makes the stream wait on the peer's flag in the front end
//     (unbounded); here one kernel does the two-shot over NVLink stores with a flag pair per CTA slice (32 slices) and
//     bounded waits, so a missing peer ends the call with a status instead of a hung stream.
//   dag_register / dag_all_gather                                              (vllm_turing/csrc/dma_ag.cu:28-74)
//     the two-rank all-gather through pinned, host-mapped staging memory (for GPUs without peer access): one kernel on
//     the `main` stream writes this rank's payload into its staging region piece by piece, publishing a flag per
//     piece, while its other CTAs wait (bounded) for the peer's flags and copy the peer's pieces in. The d2h / h2d
//     streams and the events of the reference's copy-engine version are accepted and unused.
//
// A wait that runs out (VLLM_TURING_AR_TIMEOUT_MS) writes ST_PEER_TIMEOUT into the library workspace's status word
// (vt_status); the reference's ABI has no status argument. Results are identical on both ranks: the sum of two values
// in float32 rounded once is the same in either order (and equals fp16 __hadd2).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.cuh"
#include "common.cuh"
#include "host_util.h"

namespace vt {

// ---- har: two-rank LL all-reduce ---------------------------------------------------------------------------------------
constexpr int HAR_T = 256;            // threads per block
constexpr int HAR_PAIRS = 8;          // word pairs per thread
constexpr int HAR_WORDS = HAR_T * HAR_PAIRS * 2;   // 32-bit data words per block

template <typename T>
__device__ __forceinline__ uint32_t add_words(uint32_t a, uint32_t b) {
    const float2 x = unpack2<T>(a), y = unpack2<T>(b);
    return pack2<T>(x.x + y.x, x.y + y.y);
}

// Block b covers words [b HAR_WORDS, (b + 1) HAR_WORDS); thread t its pairs t, t + HAR_T, ... (words 2p, 2p + 1).
template <typename T>
__global__ void __launch_bounds__(HAR_T) har_ll_kernel(const uint32_t *__restrict__ in, uint32_t *__restrict__ out,
                                                       int nwords, unsigned long long *dst_ll,
                                                       const unsigned long long *src_ll, int *counters,
                                                       int slot_words, uint64_t timeout, unsigned *status) {
    __shared__ unsigned s_seq;
    if (threadIdx.x == 0) s_seq = (unsigned)*reinterpret_cast<volatile int *>(counters + blockIdx.x) + 1u;
    __syncthreads();
    const unsigned seq = s_seq;
    const size_t slot = (size_t)(seq & 1u) * slot_words;
    unsigned long long *dst = dst_ll + slot;
    const unsigned long long *src = src_ll + slot;
    const int w0 = blockIdx.x * HAR_WORDS;
    // 16-byte accesses when every address involved is 16-byte aligned (slot_words even, regions 16-byte aligned)
    const bool vec = ((((uintptr_t)dst | (uintptr_t)src) & 15) == 0);
    const unsigned long long tag = (unsigned long long)seq << 32;
    uint32_t v[HAR_PAIRS][2];
#pragma unroll
    for (int j = 0; j < HAR_PAIRS; ++j) {
        const int i = w0 + 2 * (threadIdx.x + j * HAR_T);
        v[j][0] = i < nwords ? in[i] : 0u;
        v[j][1] = i + 1 < nwords ? in[i + 1] : 0u;
        if (i + 1 < nwords && vec) {
            asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + i), "l"(tag | v[j][0]),
                         "l"(tag | v[j][1])
                         : "memory");
        } else {
            if (i < nwords) st_volatile8(dst + i, tag | v[j][0]);
            if (i + 1 < nwords) st_volatile8(dst + i + 1, tag | v[j][1]);
        }
    }
    const uint64_t deadline = globaltimer() + timeout;
    bool dead = false;
#pragma unroll 1
    for (int j = 0; j < HAR_PAIRS; ++j) {
        const int i = w0 + 2 * (threadIdx.x + j * HAR_T);
        if (i >= nwords) break;
        const bool two = i + 1 < nwords;
        unsigned long long a = 0, b = 0;
        uint32_t it = 0;
        for (;;) {
            if (two && vec) {
                asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src + i) : "memory");
            } else {
                a = ld_volatile8(src + i);
                b = two ? ld_volatile8(src + i + 1) : tag;
            }
            if ((unsigned)(a >> 32) == seq && (unsigned)(b >> 32) == seq) break;
            if (dead || ((++it & 255u) == 0 && globaltimer() > deadline)) {
                if (!dead) report(status, ST_PEER_TIMEOUT | 0x700u);
                dead = true;
                break;
            }
        }
        out[i] = add_words<T>(v[j][0], (uint32_t)a);
        if (two) out[i + 1] = add_words<T>(v[j][1], (uint32_t)b);
    }
    __syncthreads();
    if (threadIdx.x == 0) counters[blockIdx.x] = (int)seq;
}

// ---- ce: two-rank fp16 two-shot over the IPC buffers -------------------------------------------------------------------
constexpr int CE_SLICES = 32;         // CTAs; flag pair per slice in the 256-byte header
constexpr int CE_THREADS = 512;

__device__ __forceinline__ unsigned *ce_flag(char *buf, int which, int j) {
    return reinterpret_cast<unsigned *>(buf) + which * CE_SLICES + j;
}

// out[u] = a[u] + b[u] over 16-byte units [u0, u1) (8 halves each, float32 sum rounded once)
__device__ __forceinline__ void ce_add_units(const uint4 *a, const uint4 *b, uint4 *o, long long u0, long long u1) {
    for (long long u = u0 + threadIdx.x; u < u1; u += 2LL * CE_THREADS) {
        const bool two = u + CE_THREADS < u1;
        const uint4 x0 = a[u], y0 = __ldcg(b + u);
        uint4 x1 = x0, y1 = y0;
        if (two) {
            x1 = a[u + CE_THREADS];
            y1 = __ldcg(b + u + CE_THREADS);
        }
        o[u] = make_uint4(add_words<__half>(x0.x, y0.x), add_words<__half>(x0.y, y0.y), add_words<__half>(x0.z, y0.z),
                          add_words<__half>(x0.w, y0.w));
        if (two)
            o[u + CE_THREADS] = make_uint4(add_words<__half>(x1.x, y1.x), add_words<__half>(x1.y, y1.y),
                                           add_words<__half>(x1.z, y1.z), add_words<__half>(x1.w, y1.w));
    }
}
__device__ __forceinline__ void ce_copy_units(const uint4 *s, uint4 *d, long long u0, long long u1, bool ldcg) {
    for (long long u = u0 + threadIdx.x; u < u1; u += CE_THREADS) d[u] = ldcg ? __ldcg(s + u) : s[u];
}

// Rank r owns half r (elements [0, h) or [h, n), h = n / 2): (1) push the peer's half of x into the peer's R1, flag;
// (2) wait for the own flag, own half of out = x + R1, push it into the peer's R2, flag; (3) wait, copy R2 into the
// peer's half of out. Slice j of each half belongs to CTA j on both ranks.
__global__ void __launch_bounds__(CE_THREADS) ce_two_rank_kernel(const __half *x, __half *out, long long n, int rank,
                                                                 char *my, char *peer, long long cap, unsigned seq,
                                                                 uint64_t timeout, unsigned *status) {
    const long long h = n / 2;
    const long long own_off = rank == 0 ? 0 : h, own_len = rank == 0 ? h : n - h;
    const long long oth_off = rank == 0 ? h : 0, oth_len = rank == 0 ? n - h : h;
    const int j = blockIdx.x;
    const uint64_t deadline = globaltimer() + timeout;
    // this CTA's slices (16-byte units) of the peer's half and of the own half
    const long long ou = oth_len / 8, mu = own_len / 8;
    const long long o0 = ou * j / CE_SLICES, o1 = ou * (j + 1) / CE_SLICES;
    const long long m0 = mu * j / CE_SLICES, m1 = mu * (j + 1) / CE_SLICES;
    uint4 *peer_r1 = reinterpret_cast<uint4 *>(peer + 256), *peer_r2 = reinterpret_cast<uint4 *>(peer + 256 + cap);
    const uint4 *my_r1 = reinterpret_cast<const uint4 *>(my + 256);
    const uint4 *my_r2 = reinterpret_cast<const uint4 *>(my + 256 + cap);
    // (1)
    ce_copy_units(reinterpret_cast<const uint4 *>(x + oth_off), peer_r1, o0, o1, false);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) st_release_sys(ce_flag(peer, 0, j), seq);
    // (2)
    if (threadIdx.x == 0 && !flag_wait(ce_flag(my, 0, j), seq, deadline)) report(status, ST_PEER_TIMEOUT | 0x800u);
    __syncthreads();
    ce_add_units(reinterpret_cast<const uint4 *>(x + own_off), my_r1, reinterpret_cast<uint4 *>(out + own_off), m0,
                 m1);
    __syncthreads();
    ce_copy_units(reinterpret_cast<const uint4 *>(out + own_off), peer_r2, m0, m1, false);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) st_release_sys(ce_flag(peer, 1, j), seq);
    // (3)
    if (threadIdx.x == 0 && !flag_wait(ce_flag(my, 1, j), seq, deadline)) report(status, ST_PEER_TIMEOUT | 0x900u);
    __syncthreads();
    ce_copy_units(my_r2, reinterpret_cast<uint4 *>(out + oth_off), o0, o1, true);
}

// ---- dag: two-rank all-gather through host-mapped staging ---------------------------------------------------------------
constexpr int DAG_THREADS = 256;

// bytes [b, e) from s to d: 16-byte units where both sides allow it, then single bytes
__device__ __forceinline__ void dag_copy(const char *s, char *d, long long b, long long e) {
    if ((((uintptr_t)(s + b) | (uintptr_t)(d + b)) & 15) == 0) {
        const long long nu = (e - b) >> 4;
        const uint4 *su = reinterpret_cast<const uint4 *>(s + b);
        uint4 *du = reinterpret_cast<uint4 *>(d + b);
        for (long long u = threadIdx.x; u < nu; u += DAG_THREADS) du[u] = __ldcg(su + u);
        b += nu << 4;
    }
    for (long long i = b + threadIdx.x; i < e; i += DAG_THREADS) d[i] = s[i];
}

// CTAs [0, G): pieces p = j, j + G, ... of this rank's payload -> my_stage, then my_flag[p] = seq.
// CTAs [G, 2G): pieces of the peer's payload, after peer_flag[p] >= seq, peer_stage -> theirs.
__global__ void __launch_bounds__(DAG_THREADS) dag_kernel(const char *mine, char *theirs, long long m, char *my_stage,
                                                          const char *peer_stage, int *my_flag, const int *peer_flag,
                                                          int seq, int P, long long piece, uint64_t timeout,
                                                          unsigned *status) {
    const int G = gridDim.x / 2;
    const bool push = (int)blockIdx.x < G;
    const int j = push ? blockIdx.x : blockIdx.x - G;
    const uint64_t deadline = globaltimer() + timeout;
    bool dead = false;
    for (int p = j; p < P; p += G) {
        const long long b = (long long)p * piece, e = b + piece < m ? b + piece : m;
        if (b >= e) break;
        if (push) {
            dag_copy(mine, my_stage, b, e);
            __threadfence_system();
            __syncthreads();
            if (threadIdx.x == 0) st_release_sys(reinterpret_cast<unsigned *>(my_flag + p), (unsigned)seq);
        } else {
            if (threadIdx.x == 0 && !dead) {
                uint32_t it = 0;
                while ((int)ld_acquire_sys(reinterpret_cast<const unsigned *>(peer_flag + p)) < seq) {
                    __nanosleep(200);
                    if ((++it & 63u) == 0 && globaltimer() > deadline) {
                        report(status, ST_PEER_TIMEOUT | 0xa00u);
                        dead = true;
                        break;
                    }
                }
            }
            __syncthreads();
            dag_copy(peer_stage, theirs, b, e);
        }
    }
}

static unsigned *lib_status(cudaStream_t s) {
    void *scratch = nullptr;
    unsigned *status = nullptr;
    if (ws_acquire(0, s, &scratch, &status) != 0) return nullptr;   // timeouts then go unreported
    return status;
}

}  // namespace vt

using namespace vt;

extern "C" {

// Loads the kernels of this file now (a lazily loaded module may synchronise behind a kernel spinning on a peer) and
// creates the library workspace whose status word the waits report into. 0 ok; 1, 2 the fp16 / bf16 LL kernels.
int har_preload(void) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, har_ll_kernel<__half>) != cudaSuccess) return 1;
    if (cudaFuncGetAttributes(&fa, har_ll_kernel<__nv_bfloat16>) != cudaSuccess) return 2;
    cudaFuncGetAttributes(&fa, ce_two_rank_kernel);
    cudaFuncGetAttributes(&fa, dag_kernel);
    lib_status(0);
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// Blocks (and per-block call counters the caller allocates, zeroed) for nwords data words.
int har_blocks(int nwords) { return nwords <= 0 ? 0 : (nwords + HAR_WORDS - 1) / HAR_WORDS; }

// Registers a host range (e.g. a shared-memory mapping) for device access; returns its device pointer, NULL on failure.
void *har_register(void *ptr, size_t size) {
    if (cudaHostRegister(ptr, size, cudaHostRegisterMapped | cudaHostRegisterPortable) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    void *d = nullptr;
    if (cudaHostGetDevicePointer(&d, ptr, 0) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return d;
}

int har_unregister(void *ptr) { return (int)cudaHostUnregister(ptr); }

// out[nwords] = in + the peer's in (32-bit words of two fp16 / bf16 values; dtype 0 / 1). my_ll: where this rank's LL
// words go (the peer's receive region), peer_ll: where the peer's arrive (polled); each 2 * slot_words 8-byte words.
// counters: har_blocks(slot_words) zeroed ints, this rank's own. Returns -1 if nwords > slot_words, else the launch's
// cudaError.
int har_all_reduce(const void *in, void *out, int nwords, int dtype, void *my_ll, const void *peer_ll, void *counters,
                   int slot_words, void *stream) {
    if (nwords > slot_words) return -1;
    if (nwords <= 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    const int nb = har_blocks(nwords);
    unsigned *st = lib_status(s);
    if (dtype == 0)
        har_ll_kernel<__half><<<nb, HAR_T, 0, s>>>((const uint32_t *)in, (uint32_t *)out, nwords,
                                                   (unsigned long long *)my_ll, (const unsigned long long *)peer_ll,
                                                   (int *)counters, slot_words, peer_timeout_ns(), st);
    else
        har_ll_kernel<__nv_bfloat16><<<nb, HAR_T, 0, s>>>((const uint32_t *)in, (uint32_t *)out, nwords,
                                                          (unsigned long long *)my_ll,
                                                          (const unsigned long long *)peer_ll, (int *)counters,
                                                          slot_words, peer_timeout_ns(), st);
    return (int)cudaGetLastError();
}

// 0: ce_all_reduce can run (it needs no driver entry points here: its cross-GPU ordering is done by its kernel).
int ce_driver_ok(void) { return 0; }

// x, out: n fp16 values (n % 16 == 0, 16-byte aligned); my / peer: this rank's and the peer's buffer (256 bytes of
// flags, then R1 and R2 of cap bytes each); seq: 1, 2, ... in the same order on both ranks; blocks: accepted, unused
// (the kernel always cuts each half into the same 32 slices, so the two ranks cannot disagree). Returns 0, 2 bad
// arguments, 3 cap too small, 7 launch failed (the reference's step codes).
int ce_all_reduce(const void *x, void *out, long n, int rank, void *my, void *peer, long cap, unsigned seq, int blocks,
                  cudaStream_t st) {
    (void)blocks;
    if (n % 16 != 0 || n <= 0 || (((uintptr_t)x | (uintptr_t)out) & 15) || rank < 0 || rank > 1 || !my || !peer)
        return 2;
    const long h = n / 2;
    if ((n - h) * 2 > cap) return 3;
    unsigned *status = lib_status(st);
    ce_two_rank_kernel<<<CE_SLICES, CE_THREADS, 0, st>>>((const __half *)x, (__half *)out, n, rank, (char *)my,
                                                         (char *)peer, cap, seq, peer_timeout_ns(), status);
    return cudaGetLastError() == cudaSuccess ? 0 : 7;
}

// Registers the staging segment (host pointer, bytes); returns the device pointer of its start, NULL on failure.
void *dag_register(void *host, size_t bytes) { return har_register(host, bytes); }

// gathered (device, 2 m bytes) holds this rank's payload in half `rank` (written on `main`); the peer's lands in the
// other half. my_stage / peer_stage: host staging of m bytes (registered); my_flag_dev / peer_flag_dev: device pointers
// of the P int32 piece flags of each rank; seq: the call number (flags are compared with >=). One kernel on `main`;
// d2h_, h2d_ and the events are accepted and unused. 0 ok, 1 failure.
int dag_all_gather(void *gathered, long long m, int rank, void *my_stage, const void *peer_stage, int *my_flag_dev,
                   const int *peer_flag_dev, int seq, int P, void *main_, void *d2h_, void *h2d_, void *ev0, void *ev1,
                   void *ev2) {
    (void)d2h_, (void)h2d_, (void)ev0, (void)ev1, (void)ev2;
    if (!gathered || m < 0 || rank < 0 || rank > 1 || P < 1 || !my_flag_dev || !peer_flag_dev) return 1;
    if (m == 0) return 0;
    void *my_dev = nullptr, *peer_dev = nullptr;
    if (cudaHostGetDevicePointer(&my_dev, my_stage, 0) != cudaSuccess ||
        cudaHostGetDevicePointer(&peer_dev, const_cast<void *>(peer_stage), 0) != cudaSuccess) {
        cudaGetLastError();
        return 1;
    }
    cudaStream_t s = (cudaStream_t)main_;
    const long long piece = ((m + P - 1) / P + 255) / 256 * 256;
    const int np = (int)((m + piece - 1) / piece);
    const int G = np < 32 ? np : 32;
    char *g = (char *)gathered;
    dag_kernel<<<2 * G, DAG_THREADS, 0, s>>>(g + (long long)rank * m, g + (long long)(1 - rank) * m, m,
                                             (char *)my_dev, (const char *)peer_dev, my_flag_dev, peer_flag_dev, seq,
                                             np, piece, peer_timeout_ns(), lib_status(s));
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

}  // extern "C"

// Decode-shape W8A8 GEMV for B200 (sm_100a): the streamed, HBM-bound kernel of gemv_core.cuh with the reference's
// per-token x per-channel dequant epilogue, and an int32-accumulator variant for bit-exact parity checks.
//
// C ABI (declared in include/vllm_turing_b200.h):
//   w8a8_gemv     -- the reference's signature (vllm_turing/csrc/w8a8_gemv.cu:347-361), M 1..16
//   w8a8_gemv_ws  -- the same with a caller-owned zeroed workspace (graph capture safe)
//   vt_gemv_s32   -- int32 accumulators out[M, N] (no dequant)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv_core.cuh"
#include "host_util.h"
#include "tma_host.h"

namespace vt {

template <typename T>
struct DequantEpi {
    T *out;
    const float *sa, *sw;
    const T *bias;
    int M, N, sa_rows, sw_rows;
    __device__ __forceinline__ void operator()(int rb, const int *tile, int tid) const {
        for (int idx = tid; idx < M * 32; idx += GV_CTHREADS) {
            const int m = idx >> 5, n = rb * GV_RB + (idx & 31);
            if (n >= N) continue;
            const float sam = sa[sa_rows ? m : 0], swn = sw[sw_rows ? n : 0];
            const float v = bias ? dequant1b(tile[idx], sam, swn, t2f<T>(bias[n])) : dequant1(tile[idx], sam, swn);
            out[(long long)m * N + n] = f2t<T>(v);
        }
    }
};

struct S32Epi {
    int *out;
    int M, N;
    __device__ __forceinline__ void operator()(int rb, const int *tile, int tid) const {
        for (int idx = tid; idx < M * 32; idx += GV_CTHREADS) {
            const int m = idx >> 5, n = rb * GV_RB + (idx & 31);
            if (n < N) out[(long long)m * N + n] = tile[idx];
        }
    }
};

template <int MT, class Epi>
__global__ void __launch_bounds__(GV_THREADS, 1)
    gemv_kernel(const int8_t *__restrict__ a, const __grid_constant__ CUtensorMap wmap, int M, int N, int K,
                int *scratch, int *tickets, int stages, uint64_t timeout_ns, unsigned *status, Epi epi) {
    extern __shared__ __align__(128) unsigned char smem[];
    const uint64_t deadline = globaltimer() + timeout_ns;
    gemv_phase<MT>(a, &wmap, M, N, K, scratch, tickets, smem, stages, deadline, status, epi);
}

// TMA map of the weight [N, K] for the GEMV stages: box 256 bytes x 32 rows, no swizzle.
inline bool gemv_wmap(CUtensorMap *m, const void *w, int N, int K) {
    return make_map_i8(m, w, N, K, GV_SEGB / 2, GV_RB, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Scratch the GEMV needs: int32 partial sums [M, N] + one ticket per 32-column row-block.
inline size_t gemv_scratch_bytes(int M, int N) {
    const size_t nrb = (size_t)(N + GV_RB - 1) / GV_RB;
    return ((size_t)M * N * 4 + nrb * 4 + 255) & ~(size_t)255;
}

inline int gemv_mt(int M) {
    if (M <= 6) return M;
    if (M <= 8) return 8;
    if (M <= 12) return 12;
    return 16;
}

template <int MT, class Epi>
static int launch_mt(const int8_t *a, const int8_t *w, int M, int N, int K, void *scratch, unsigned *status,
                     const Epi &epi, cudaStream_t s) {
    const int dev = cur_device();
    const int avail = gv_smem_budget(dev);
    int stages = (avail - GV_HDR - gv_align128((long long)MT * K)) / GV_STAGE;
    if (stages > GV_MAXSTAGES) stages = GV_MAXSTAGES;
    if (stages < 2) return VT_EARG;   // the activations do not fit next to a ring: the tensor-core path takes it
    const int smem = gv_smem_bytes(MT, K, stages);
    static bool attr_set[VT_MAX_DEV] = {false};
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(gemv_kernel<MT, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, avail) !=
            cudaSuccess)
            return (int)cudaGetLastError();
        attr_set[dev] = true;
    }
    const int nrb = (N + GV_RB - 1) / GV_RB;
    const long long T = (long long)nrb * (K >> 4);
    long long g = T / 64;   // at least 64 chunks (1 KB per row) per CTA
    if (g < 1) g = 1;
    if (g > num_sms(dev)) g = num_sms(dev);
    int *sc = reinterpret_cast<int *>(scratch);
    int *tickets = sc + (size_t)M * N;
    CUtensorMap wmap;
    if (!gemv_wmap(&wmap, w, N, K)) return VT_EARG;
    gemv_kernel<MT, Epi><<<(int)g, GV_THREADS, smem, s>>>(a, wmap, M, N, K, sc, tickets, stages, pipe_timeout_ns(),
                                                          status, epi);
    return (int)cudaGetLastError();
}

template <class Epi>
static int launch(const int8_t *a, const int8_t *w, int M, int N, int K, void *scratch, unsigned *status,
                  const Epi &epi, cudaStream_t s) {
    switch (gemv_mt(M)) {
        case 1: return launch_mt<1>(a, w, M, N, K, scratch, status, epi, s);
        case 2: return launch_mt<2>(a, w, M, N, K, scratch, status, epi, s);
        case 3: return launch_mt<3>(a, w, M, N, K, scratch, status, epi, s);
        case 4: return launch_mt<4>(a, w, M, N, K, scratch, status, epi, s);
        case 5: return launch_mt<5>(a, w, M, N, K, scratch, status, epi, s);
        case 6: return launch_mt<6>(a, w, M, N, K, scratch, status, epi, s);
        case 8: return launch_mt<8>(a, w, M, N, K, scratch, status, epi, s);
        case 12: return launch_mt<12>(a, w, M, N, K, scratch, status, epi, s);
        default: return launch_mt<16>(a, w, M, N, K, scratch, status, epi, s);
    }
}

static bool gemv_args_ok(const void *a, const void *w, int M, int N, int K) {
    return M >= 1 && M <= 16 && N >= 1 && K >= 16 && (K & 15) == 0 && ((uintptr_t)a & 15) == 0 &&
           ((uintptr_t)w & 15) == 0;
}

template <typename T>
static int gemv_dequant(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out,
                        int M, int N, int K, int sa_rows, int sw_rows, void *scratch, unsigned *status,
                        cudaStream_t s) {
    DequantEpi<T> epi{(T *)out, (const float *)sa, (const float *)sw, (const T *)bias, M, N, sa_rows, sw_rows};
    return launch((const int8_t *)a, (const int8_t *)w, M, N, K, scratch, status, epi, s);
}

}  // namespace vt

using namespace vt;

extern "C" {

// Bytes of zeroed workspace w8a8_gemv_ws needs for these shapes (status word included).
size_t w8a8_gemv_ws_bytes(int M, int N) { return 256 + gemv_scratch_bytes(M, N); }

// The reference's ABI: a [M, K] int8, w [N, K] int8 (row-major), sa [M] or [1], sw [N] or [1] float32, bias [N] or
// NULL (out dtype), out [M, N]; dtype 0 fp16 / 1 bf16. Returns 0, -1 on bad arguments, else a CUDA error code. The
// split-K scratch comes from the library's per-device workspace (allocated at the first call for a shape class; that
// first call must not be inside stream capture).
int w8a8_gemv(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M, int N,
              int K, int sa_rows, int sw_rows, int dtype, void *stream) {
    if (!gemv_args_ok(a, w, M, N, K)) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    int rc = ws_acquire(gemv_scratch_bytes(M, N), s, &scratch, &status);
    if (rc) return rc;
    if (dtype == 0)
        return gemv_dequant<__half>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
    return gemv_dequant<__nv_bfloat16>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
}

// Same with a caller-owned workspace of w8a8_gemv_ws_bytes(M, N) bytes, zeroed once before its first use (the kernel
// leaves it zeroed); calls sharing a workspace must be stream-ordered. The first 256 bytes hold the status word.
int w8a8_gemv_ws(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out, int M,
                 int N, int K, int sa_rows, int sw_rows, int dtype, void *workspace, size_t ws_bytes, void *stream) {
    if (!gemv_args_ok(a, w, M, N, K) || !workspace || ws_bytes < w8a8_gemv_ws_bytes(M, N)) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned *status = (unsigned *)workspace;
    void *scratch = (char *)workspace + 256;
    if (dtype == 0)
        return gemv_dequant<__half>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
    return gemv_dequant<__nv_bfloat16>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, scratch, status, s);
}

// int32 accumulators: acc[M, N] = a . w^T exactly.
int vt_gemv_s32(const void *a, const void *w, void *acc, int M, int N, int K, void *stream) {
    if (!gemv_args_ok(a, w, M, N, K)) return VT_EARG;
    cudaStream_t s = (cudaStream_t)stream;
    void *scratch;
    unsigned *status;
    int rc = ws_acquire(gemv_scratch_bytes(M, N), s, &scratch, &status);
    if (rc) return rc;
    S32Epi epi{(int *)acc, M, N};
    return launch((const int8_t *)a, (const int8_t *)w, M, N, K, scratch, status, epi, s);
}

}  // extern "C"

// ---- allocation-free GEMV ------------------------------------------------------------------------------------------
// Some callers cannot allocate device memory at the moment they run a GEMV: code inside a custom allocator or memory
// profiler (vLLM's memory profiling measures every allocation, so the kernel must not add any), processes that hand
// all device memory to a pool before the first call, and code paths that run while another thread holds the
// allocator. For them w8a8_gemv_noalloc takes its split-K scratch from a fixed array compiled into the library
// instead of cudaMalloc: NOALLOC_INTS int32 words (1 MiB + 33 KiB), which every GPU that loads the library keeps
// until the process exits. Its first call on a device resolves the array's device address (cudaGetSymbolAddress, with
// that device current); make that first call before any stream capture. All calls on a device share the one array,
// so calls that overlap on the GPU (different streams, or different host threads without ordering) race and produce
// wrong results; order them on one stream.
namespace vt {

constexpr int NOALLOC_PARTIAL_INTS = 1 << 18;                     // int32 partial sums: M * N <= 262144
constexpr int NOALLOC_TICKET_INTS = 8192;                         // one per 32-column row-block: N <= 262144
constexpr int NOALLOC_INTS = 64 + NOALLOC_PARTIAL_INTS + NOALLOC_TICKET_INTS;   // 256-byte status header first
static __device__ __align__(256) int g_noalloc_scratch[NOALLOC_INTS];

static int *noalloc_scratch_ptr(int dev) {
    static int *ptrs[VT_MAX_DEV] = {nullptr};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        ptrs[dev] = reinterpret_cast<int *>(p);
    }
    return ptrs[dev];
}

}  // namespace vt

extern "C" {

// The w8a8_gemv contract (same arguments, same results) without any device allocation: scratch comes from the
// library's fixed array. Rejects, with VT_EARG and before launching anything, M * N > 262144 or N > 262144 (the
// array's capacity) as well as every shape w8a8_gemv rejects. The partial-sum region and tickets it uses are cleared
// on the stream before the kernel runs (cudaMemsetAsync, no allocation), so a call never depends on the contents a
// previous call left. The first call on each device must come before any stream capture (see above).
int w8a8_gemv_noalloc(const void *a, const void *w, const void *sa, const void *sw, const void *bias, void *out,
                      int M, int N, int K, int sa_rows, int sw_rows, int dtype, void *stream) {
    if (!gemv_args_ok(a, w, M, N, K)) return VT_EARG;
    const long long nrb = (N + GV_RB - 1) / GV_RB;
    if ((long long)M * N > NOALLOC_PARTIAL_INTS || nrb > NOALLOC_TICKET_INTS) return VT_EARG;
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    int *base = noalloc_scratch_ptr(dev);
    if (!base) return (int)cudaErrorInvalidSymbol;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned *status = reinterpret_cast<unsigned *>(base);
    int *partials = base + 64;
    int *tickets = partials + (size_t)M * N;   // the layout the GEMV launcher expects: partials, then tickets
    cudaError_t e = cudaMemsetAsync(partials, 0, ((size_t)M * N + (size_t)nrb) * sizeof(int), s);
    if (e != cudaSuccess) return (int)e;
    (void)tickets;
    if (dtype == 0)
        return gemv_dequant<__half>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, partials, status, s);
    return gemv_dequant<__nv_bfloat16>(a, w, sa, sw, bias, out, M, N, K, sa_rows, sw_rows, partials, status, s);
}

// The status word of w8a8_gemv_noalloc on the current device (the first word of its fixed array): 0, or the first
// timeout code one of its kernels reported (a pipeline wait that gave up leaves `out` wrong while the call itself
// returned 0). clear != 0 resets it. Synchronises the device; allocates nothing. 0xffffffff if the array's address
// cannot be resolved.
unsigned vt_noalloc_status(int clear) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return 0xffffffffu;
    int *base = noalloc_scratch_ptr(dev);
    if (!base) return 0xffffffffu;
    unsigned v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&v, base, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return 0xffffffffu;
    }
    if (clear && cudaMemset(base, 0, 4) != cudaSuccess) cudaGetLastError();
    return v;
}

// Number of non-zero 32-bit words in the first `bytes` of the current device's library workspace scratch (every
// kernel that uses it leaves it zeroed; tests check that invariant). Synchronises the device; -1 on error.
long long vt_workspace_nonzero(long long bytes) {
    void *scratch;
    unsigned *status;
    if (bytes <= 0 || ws_acquire(0, 0, &scratch, &status) != 0) return -1;
    const int dev = cur_device();
    const size_t have = ws_table()[dev].bytes - 256;
    if ((size_t)bytes > have) bytes = (long long)have;
    const size_t n = (size_t)bytes / 4;
    int *h = (int *)malloc(n * 4);
    if (!h) return -1;
    cudaDeviceSynchronize();
    if (cudaMemcpy(h, scratch, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        free(h);
        cudaGetLastError();
        return -1;
    }
    long long c = 0;
    for (size_t i = 0; i < n; ++i) c += h[i] != 0;
    free(h);
    return c;
}

// Reads (and with clear != 0 resets) the library workspace status word of the current device: 0, or the first
// timeout code a kernel reported (see common.cuh). Synchronises the device.
unsigned vt_status(int clear) {
    void *scratch;
    unsigned *status;
    if (ws_acquire(0, 0, &scratch, &status) != 0) return 0xffffffffu;
    unsigned v = 0;
    cudaDeviceSynchronize();
    cudaMemcpy(&v, status, 4, cudaMemcpyDeviceToHost);
    if (clear) cudaMemset(status, 0, 4);
    return v;
}

}  // extern "C"

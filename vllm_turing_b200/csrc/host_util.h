// Host-side helpers shared by the .cu files of libvllm_turing_b200.so: cached device attributes, the per-device
// library workspace (zeroed scratch for split-K tickets and partial sums, plus the device status word) and the
// timeouts of the bounded device waits.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>
#include <mutex>
#include <utility>

namespace vt {

constexpr int VT_MAX_DEV = 64;

// error codes returned by the C ABI (in addition to positive cudaError_t values)
enum : int {
    VT_EARG = -1,        // unsupported shape / alignment / argument
    VT_ECAPTURE = -2,    // the call needs a workspace allocation while the stream is capturing
    VT_ENOMEM = -3,      // workspace allocation failed
};

inline int cur_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

inline int num_sms(int dev) {
    static int cache[VT_MAX_DEV] = {0};
    if (dev < 0 || dev >= VT_MAX_DEV) return 148;
    if (!cache[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v > 0 ? v : 148;
    }
    return cache[dev];
}

inline int max_smem_optin(int dev) {
    static int cache[VT_MAX_DEV] = {0};
    if (dev < 0 || dev >= VT_MAX_DEV) return 232448;
    if (!cache[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cache[dev] = v > 0 ? v : 232448;
    }
    return cache[dev];
}

// Dynamic shared memory the streamed kernels may take: the opt-in limit minus 1 KB for static shared variables.
inline int gv_smem_budget(int dev) { return max_smem_optin(dev) - 1024; }

inline uint64_t env_ns(const char *name, double default_ms) {
    const char *v = getenv(name);
    double ms = v ? atof(v) : default_ms;
    if (ms <= 0) ms = default_ms;
    return (uint64_t)(ms * 1e6);
}

// Bound on waits inside one CTA (bulk copies, MMA completion): a healthy kernel waits microseconds.
inline std::atomic<uint64_t> &pipe_timeout_slot() {
    static std::atomic<uint64_t> v{env_ns("VLLM_TURING_PIPE_TIMEOUT_MS", 2000.0)};
    return v;
}
inline uint64_t pipe_timeout_ns() { return pipe_timeout_slot().load(std::memory_order_relaxed); }
// Bound on waits for other CTAs or other GPUs (LL words of peers): ranks may enter a call far apart in time.
inline std::atomic<uint64_t> &peer_timeout_slot() {
    static std::atomic<uint64_t> v{env_ns("VLLM_TURING_AR_TIMEOUT_MS", 10000.0)};
    return v;
}
inline uint64_t peer_timeout_ns() { return peer_timeout_slot().load(std::memory_order_relaxed); }

// Programmatic dependent launch for the decode-chain kernels (tcgen05 GEMMs, fused row-linear, row-split SiLU-quant):
// VLLM_TURING_PDL=0 turns it off.
inline bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("VLLM_TURING_PDL");
        v = (e && atoi(e) == 0) ? 0 : 1;
    }
    return v != 0;
}

// kernel<<<grid, block, smem, s>>>(args...) with the programmatic-stream-serialization attribute when pdl is set (the
// kernel may start while its predecessor in the stream finishes; it must call pdl_wait before using that one's data).
template <typename... KArgs, typename... Args>
inline int launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                    Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

inline bool stream_capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return st != cudaStreamCaptureStatusNone;
}

// Per-device library workspace: [0, 256) status word(s), then zero-initialised scratch that kernels return to zero.
struct Workspace {
    void *base = nullptr;
    size_t bytes = 0;
};

inline std::mutex &ws_mutex() {
    static std::mutex m;
    return m;
}
inline Workspace *ws_table() {
    static Workspace t[VT_MAX_DEV];
    return t;
}

// Per-device auxiliary buffer for data a kernel rewrites in full on every call before reading it (never assumed to be
// zero, so it is kept apart from the zeroed workspace). Grows outside stream capture only.
inline Workspace *aux_table() {
    static Workspace t[VT_MAX_DEV];
    return t;
}
inline int aux_acquire(size_t need, cudaStream_t s, void **buf) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    std::lock_guard<std::mutex> lk(ws_mutex());
    Workspace &w = aux_table()[dev];
    if (w.bytes < need) {
        if (stream_capturing(s)) return VT_ECAPTURE;
        const size_t nb = (need + ((size_t)1 << 20) - 1) & ~(((size_t)1 << 20) - 1);
        if (w.base) {
            cudaStreamSynchronize(s);
            cudaDeviceSynchronize();
            cudaFree(w.base);
            w.base = nullptr;
            w.bytes = 0;
        }
        void *p = nullptr;
        if (cudaMalloc(&p, nb) != cudaSuccess) {
            cudaGetLastError();
            return VT_ENOMEM;
        }
        w.base = p;
        w.bytes = nb;
    }
    *buf = w.base;
    return 0;
}

// Returns a zeroed device buffer of at least `need` bytes past the 256-byte status header of the current device (the
// pointer returned points at the scratch; status = scratch - 256). Grows outside stream capture only.
inline int ws_acquire(size_t need, cudaStream_t s, void **scratch, unsigned **status) {
    const int dev = cur_device();
    if (dev < 0 || dev >= VT_MAX_DEV) return VT_EARG;
    std::lock_guard<std::mutex> lk(ws_mutex());
    Workspace &w = ws_table()[dev];
    need = (need + 255) & ~(size_t)255;
    if (w.bytes < need + 256) {
        if (stream_capturing(s)) return VT_ECAPTURE;
        size_t nb = need + 256;
        if (nb < ((size_t)8 << 20)) nb = (size_t)8 << 20;
        void *p = nullptr;
        if (w.base) {
            cudaStreamSynchronize(s);
            cudaDeviceSynchronize();
            cudaFree(w.base);
            w.base = nullptr;
            w.bytes = 0;
        }
        if (cudaMalloc(&p, nb) != cudaSuccess) {
            cudaGetLastError();
            return VT_ENOMEM;
        }
        if (cudaMemset(p, 0, nb) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            cudaGetLastError();
            cudaFree(p);
            return VT_ENOMEM;
        }
        w.base = p;
        w.bytes = nb;
    }
    *status = reinterpret_cast<unsigned *>(w.base);
    *scratch = reinterpret_cast<char *>(w.base) + 256;
    return 0;
}

}  // namespace vt

// The tensor-parallel communicator shared by the all-reduce, all-gather and fused row-linear kernels.
//
// Every rank owns one device region (cudaMalloc'd, exported with a CUDA IPC handle, zeroed once); every rank maps every
// peer's region (ce_open). All ranks use the identical layout:
//
//   [0, CTRL)            control: seq (u32 @0, the last completed call), done ticket (u32 @64), status (u32 @128),
//                        group mailbox (u64 [32 rows][16 groups][2] @4096), split-K tickets of the fused
//                        GEMM (int [4096] @16384: GEMV row-blocks or tcgen05 tiles), tile mailbox of the fused
//                        decode tail (@65536: 16-byte statistics words [64 tiles][32 rows], then 8-byte absmax
//                        words [64 tiles][32 rows])
//   LL                   LL receive slots [parity 2][src rank][ll_slot bytes]: peers push 16-byte LL words here
//   SCRATCH              int32 split-K partial sums of the fused GEMV [ll rows][N] (local use only)
//   RS                   two-shot reduce-scatter receive buffers [parity 2][src rank][chunk_cap bytes]
//   AGR                  all-gather receive buffers of the two-shot and the fused prefill tail: the peers' reduced
//                        chunks / rows, pushed by their owners [parity 2][src rank][chunk_cap] (world > 1)
//   FLAGS                u32 flags [parity 2][kind 2][src rank][256 CTAs] (kind 0: RS data landed, 1: reduced chunk pushed)
//   PF                   fused prefill row-linear: tile flags [parity 2][src rank][PF_MAX_TILES] (a source's GEMM
//                        tile of this rank's rows landed in RS) and reduced-rows flags [parity 2][src rank][PF_MAX_CTAS]
//                        (CTA j of rank src pushed its reduced rows into this rank's AGR buffer)
//
// Call protocol (the same call order on every rank, stream-ordered calls on each rank; cf. vllm_turing/cear.py:79):
//   each launch reads seq = ctrl.seq + 1 at its start; the last of its CTAs to finish stores ctrl.seq = seq, so seq
//   lives on the device and CUDA-graph replays keep counting (vllm_turing/csrc/host_ar.cu:36-38, 78-81 keep per-block
//   counters for the same reason). Buffers are double-buffered by seq parity: a rank can be at most one call ahead of a
//   peer (finishing call s needs the peer's call-s data, which the peer writes only after its call s - 1 finished
//   reading), so call s + 2 may reuse the buffers of call s. Readers test flags for equality with seq.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace vt {

constexpr int COMM_MAX_RANKS = 8;
constexpr int COMM_MAX_CTAS = 256;
constexpr size_t COMM_CTRL = 131072;
constexpr size_t COMM_MBOX_OFF = 4096;
constexpr size_t COMM_TICKET_OFF = 16384;
constexpr int COMM_TICKETS = 4096;
constexpr int COMM_MBOX_ROWS = 32, COMM_MBOX_GROUPS = 16;
constexpr int PF_MAX_TILES = 4096, PF_MAX_CTAS = 1024;
constexpr size_t COMM_TMBOX_OFF = 65536;   // tile mailbox: 32 KB of statistics words, 16 KB of absmax words
constexpr int COMM_TMBOX_TILES = 64;

struct CommLayout {
    size_t ll_slot;       // bytes of one LL slot (= 2 x the data bytes it carries)
    size_t ll_off, scratch_off, scratch_bytes, rs_off, agr_off, flags_off, pf_off, total;
    size_t chunk_cap;     // two-shot: bytes of one rank's chunk per call
};

__host__ __device__ inline size_t comm_align(size_t x) { return (x + 4095) & ~(size_t)4095; }

// ll_data: largest one-shot / fused message in bytes; big_data: largest two-shot message per launch in bytes;
// scratch_ints: int32 split-K scratch of the fused GEMV.
__host__ __device__ inline CommLayout comm_layout(int world, size_t ll_data, size_t big_data, size_t scratch_ints) {
    CommLayout L;
    L.ll_slot = comm_align(ll_data * 2);
    L.ll_off = COMM_CTRL;
    L.scratch_off = L.ll_off + 2 * (size_t)world * L.ll_slot;
    L.scratch_bytes = comm_align(scratch_ints * 4);
    L.chunk_cap = comm_align((big_data + world - 1) / world);
    L.rs_off = L.scratch_off + L.scratch_bytes;
    L.agr_off = L.rs_off + 2 * (size_t)world * L.chunk_cap;
    L.flags_off = L.agr_off + (world > 1 ? 2 * (size_t)world * L.chunk_cap : 0);
    L.pf_off = L.flags_off + comm_align(2 * 2 * (size_t)COMM_MAX_RANKS * COMM_MAX_CTAS * 4);
    L.total = L.pf_off + comm_align(2 * (size_t)COMM_MAX_RANKS * PF_MAX_TILES * 4 +
                                    2 * (size_t)COMM_MAX_RANKS * PF_MAX_CTAS * 4);
    return L;
}

// Kernel-side view of a communicator (passed by value).
struct CommView {
    char *base[COMM_MAX_RANKS];   // every rank's region, base[rank] local
    int rank, world;
    CommLayout L;
    __device__ __forceinline__ char *local() const { return base[rank]; }
    __device__ __forceinline__ unsigned *seq_ptr() const { return reinterpret_cast<unsigned *>(local()); }
    __device__ __forceinline__ unsigned *done_ptr() const { return reinterpret_cast<unsigned *>(local() + 64); }
    __device__ __forceinline__ unsigned *status() const { return reinterpret_cast<unsigned *>(local() + 128); }
    __device__ __forceinline__ unsigned long long *mbox() const {
        return reinterpret_cast<unsigned long long *>(local() + COMM_MBOX_OFF);
    }
    // fused decode tail, 128-feature tile `tile`, token row m: the tile's statistics as one 16-byte LL word (sum of
    // squares of the new residual; the |residual|, |norm weight| pair of its largest product and a near-tie flag), and
    // its absmax of the normalised values as a seq-tagged 8-byte word
    __device__ __forceinline__ uint4 *tm_stat(int tile, int m) const {
        return reinterpret_cast<uint4 *>(local() + COMM_TMBOX_OFF) + (size_t)tile * COMM_MBOX_ROWS + m;
    }
    __device__ __forceinline__ unsigned long long *tm_amax(int tile, int m) const {
        return reinterpret_cast<unsigned long long *>(local() + COMM_TMBOX_OFF + 32768) +
               (size_t)tile * COMM_MBOX_ROWS + m;
    }
    __device__ __forceinline__ int *tickets() const { return reinterpret_cast<int *>(local() + COMM_TICKET_OFF); }
    __device__ __forceinline__ int *scratch() const { return reinterpret_cast<int *>(local() + L.scratch_off); }
    // LL slot of `src` for parity p in rank `dst`'s region
    __device__ __forceinline__ char *ll_slot(int dst, unsigned p, int src) const {
        return base[dst] + L.ll_off + ((size_t)p * world + src) * L.ll_slot;
    }
    __device__ __forceinline__ char *rs_buf(int dst, unsigned p, int src) const {
        return base[dst] + L.rs_off + ((size_t)p * world + src) * L.chunk_cap;
    }
    __device__ __forceinline__ unsigned *flag(int dst, unsigned p, int kind, int src, int cta) const {
        return reinterpret_cast<unsigned *>(base[dst] + L.flags_off) +
               (((size_t)p * 2 + kind) * COMM_MAX_RANKS + src) * COMM_MAX_CTAS + cta;
    }
    // fused prefill: tile `tile` (numbered within the owner's rows) from `src` landed in rank `dst`'s RS buffer
    __device__ __forceinline__ unsigned *pf_tile_flag(int dst, unsigned p, int src, int tile) const {
        return reinterpret_cast<unsigned *>(base[dst] + L.pf_off) + ((size_t)p * COMM_MAX_RANKS + src) * PF_MAX_TILES +
               tile;
    }
    // two-shot and fused prefill: rank `src`'s reduced chunk / rows in rank `dst`'s receive buffer (pushed by src)
    __device__ __forceinline__ char *agr_buf(int dst, unsigned p, int src) const {
        return base[dst] + L.agr_off + ((size_t)p * world + src) * L.chunk_cap;
    }
    // fused prefill: CTA `cta` of rank `src` pushed its reduced rows into rank `dst`'s receive buffer
    __device__ __forceinline__ unsigned *pf_ag_flag(int dst, unsigned p, int src, int cta) const {
        return reinterpret_cast<unsigned *>(base[dst] + L.pf_off) + 2 * (size_t)COMM_MAX_RANKS * PF_MAX_TILES +
               ((size_t)p * COMM_MAX_RANKS + src) * PF_MAX_CTAS + cta;
    }
};

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool flag_wait(const unsigned *p, unsigned seq, uint64_t deadline) {
    uint32_t it = 0;
    while (ld_acquire_sys(p) != seq) {
        if ((++it & 63u) == 0 && globaltimer() > deadline) return false;
    }
    return true;
}

// Start of a call: every CTA reads the call's sequence number (thread 0, broadcast through shared memory).
__device__ __forceinline__ unsigned comm_begin(const CommView &c, unsigned *s_seq) {
    if (threadIdx.x == 0) *s_seq = *reinterpret_cast<volatile unsigned *>(c.seq_ptr()) + 1u;
    __syncthreads();
    return *s_seq;
}
// End of a call: the last CTA to finish publishes seq (all CTAs have read the old value by then).
__device__ __forceinline__ void comm_end(const CommView &c, unsigned seq) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned t = atomicAdd(c.done_ptr(), 1u);
        if (t == gridDim.x - 1) {
            *reinterpret_cast<volatile unsigned *>(c.done_ptr()) = 0u;
            __threadfence();
            *reinterpret_cast<volatile unsigned *>(c.seq_ptr()) = seq;
        }
    }
}

// Host-side communicator object (the opaque handle of the C ABI).
struct Comm {
    CommView v;
    int dev;
};

}  // namespace vt

// common.cuh — shared device helpers and host error plumbing of libocrcuda.so (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "ocr_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libocrcuda is written for sm_100a (B200) only"
#endif

namespace ocr {

// ---- host: the per-thread last error (ocr_last_error) -----------------------------------------------------------
void set_error(const std::string& msg);
ocr_status fail(ocr_status code, const std::string& msg);
ocr_status cuda_fail(cudaError_t e, const char* what);

#define OCR_CUDA(call)                                                                                                 \
    do {                                                                                                               \
        cudaError_t e_ = (call);                                                                                       \
        if (e_ != cudaSuccess) return ::ocr::cuda_fail(e_, #call);                                                     \
    } while (0)
#define OCR_TRY(call)                                                                                                  \
    do {                                                                                                               \
        ocr_status s_ = (call);                                                                                        \
        if (s_ != OCR_OK) return s_;                                                                                   \
    } while (0)

// Kernel attributes (the opt-in shared memory limit, non-portable cluster sizes) belong to the current device's
// context, and occupancy answers are per device: a process may drive contexts on several GPUs, so every such setup
// and cache is kept per device. MAX_DEVICES bounds the tables.
constexpr int MAX_DEVICES = 64;
inline int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        d = 0;
    }
    return d;
}
// runs f() once per device (the current one), serialised across host threads
struct PerDeviceOnce {
    std::mutex mu;
    bool done[MAX_DEVICES] = {};
    template <class F>
    void operator()(F&& f) {
        const int d = current_device();
        std::lock_guard<std::mutex> lock(mu);
        if (d < 0 || d >= MAX_DEVICES) {
            f();
            return;
        }
        if (!done[d]) {
            f();
            done[d] = true;
        }
    }
};

// ---- device -----------------------------------------------------------------------------------------------------
constexpr unsigned FULL = 0xffffffffu;
constexpr uint32_t NO_INDEX = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

// the argmax order of the sampler: a larger value wins, equal values → the lower index (ocr-decode's argmax keeps the
// first maximum); NaN never wins (every comparison with it is false)
__device__ __forceinline__ bool better(float v, uint32_t i, float w, uint32_t j) {
    return v > w || (v == w && i < j);
}

__device__ __forceinline__ void warp_argmax(float& v, uint32_t& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float w = __shfl_xor_sync(FULL, v, o);
        uint32_t j = __shfl_xor_sync(FULL, i, o);
        if (better(w, j, v, i)) {
            v = w;
            i = j;
        }
    }
}

// 16-byte streaming load of read-once data (weights): no L1 allocation
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// four signed bytes of a word → four exact floats: the biased byte (q + 128) is placed in the mantissa of 2^23
// (0x4B0000bb = 8388608 + byte) by one byte permute, then 2^23 + 128 is subtracted (exact: all values are integers
// below 2^24)
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* out) {
    const uint32_t u = w ^ 0x80808080u;
    out[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
    out[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
    out[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
    out[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}

// programmatic dependent launch: wait for the grids this one depends on (their memory visible); let dependents start
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- the in-chain timeline ----
// A launch given a slot records, from thread 0 of each of its CTAs, the latest CTA start, the latest release of its
// dependency wait (griddepcontrol.wait) and the latest CTA end, in %globaltimer nanoseconds. Slots keep maxima, so a
// slot written by several replays of one graph holds the last replay's times. A launch's in-chain time is the end of
// its latest CTA less the end of the launch before it: what it adds to the chained step, overlap included.
struct TlSlot {
    unsigned long long start, dep, end, pad;
};
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void tl_record(TlSlot* s, unsigned long long t_start, unsigned long long t_dep) {
    if (!s) return;
    atomicMax(&s->start, t_start);
    atomicMax(&s->dep, t_dep);
    atomicMax(&s->end, gtimer());
}

// device-side error flag (ocr_ctx_sync reports it): the first code wins
enum DevErr : int { DEV_OK = 0, DEV_BAD_INDEX = 1, DEV_BAD_POS = 2, DEV_TIMEOUT = 3 };

__device__ __forceinline__ void dev_error(int* flag, int code) {
    if (flag) atomicCAS(flag, 0, code);
}

// ---- bulk-async copies (the copy engine, no tensor map: contiguous 16-B multiples) and mbarriers ----------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// make the initialised barriers visible to the copy engine (async proxy)
// orders this thread's shared-memory accesses through the generic proxy before later async-proxy (bulk copy) ones
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// one poll that suspends the thread until the phase completes or `hint_ns` nanoseconds pass
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity, uint32_t hint_ns = 100000) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// a bounded wait: gives up after MBAR_TRIES polls of at most 100 µs each (≈ 2 s), flags DEV_TIMEOUT, returns false
constexpr uint32_t MBAR_TRIES = 20000;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, uint32_t tries = MBAR_TRIES,
                                          uint32_t hint_ns = 100000) {
    for (uint32_t i = 0; i < tries; i++)
        if (mbar_try_wait(bar, parity, hint_ns)) return true;
    dev_error(err, DEV_TIMEOUT);
    return false;
}

// ---- pushes into another CTA's shared memory (thread-block clusters) ----
// the cluster address of this CTA's shared variable `p` in the CTA of cluster rank `rank`
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// stores into a cluster peer's shared memory (addresses from cluster_addr), each counting its bytes as complete-tx on
// the peer's mbarrier `rbar`: the peer waits on its own barrier for everything pushed to it
__device__ __forceinline__ void st_async(uint32_t raddr, float v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
                 "r"(__float_as_uint(v)), "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void st_async(uint32_t raddr, float2 v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(raddr),
                 "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(rbar)
                 : "memory");
}
// the split cluster barrier (every thread of every CTA, in the same order): arrive, later wait
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// a bounded wait for a phase whose bytes other CTAs of the cluster pushed (acquire at cluster scope)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < MBAR_TRIES; i++) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
            : "memory");
        if (ok) return true;
    }
    dev_error(err, DEV_TIMEOUT);
    return false;
}

// bounded wait on bars[0 … n) (n ≤ N) for the same phase, their polls issued side by side
template <int N>
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bars, int n, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < MBAR_TRIES; i++) {
        bool ok = true;
#pragma unroll
        for (int k = 0; k < N; k++)
            if (k < n) ok &= mbar_try_wait(&bars[k], parity);
        if (ok) return true;
    }
    dev_error(err, DEV_TIMEOUT);
    return false;
}

// global → shared, `bytes` (multiple of 16, both addresses 16-B aligned), completion counted on `bar`
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// pulls [src, src + bytes) into L2: no shared memory, no completion to wait for (16-B aligned, multiple of 16)
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// An L2 policy under which the lines a copy brings in are the first to go. Weights and KV rows are read once per
// step and together exceed L2 many times over; streamed under this policy they leave the activations, norms, tables
// and kernel code that every step touches resident.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// one bulk copy as pieces of at most 4 KB, issued by the `n` lanes of the calling warp (lane i: pieces i, i + n, …):
// the copy engine then works on several at once rather than one long copy. Every lane calls it; the barrier's
// expected bytes (the whole copy) were raised by one lane before a __syncwarp.
__device__ __forceinline__ void bulk_g2s_lanes(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy, int lane, int n) {
    constexpr uint32_t PIECE = 4096;
    for (uint32_t o = (uint32_t)lane * PIECE; o < bytes; o += (uint32_t)n * PIECE)
        bulk_g2s_stream(static_cast<uint8_t*>(dst) + o, static_cast<const uint8_t*>(src) + o, min(PIECE, bytes - o), bar,
                        policy);
}

// a barrier among the first `threads` threads of the CTA (named barrier 1; the producer warp stays out)
__device__ __forceinline__ void bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace ocr

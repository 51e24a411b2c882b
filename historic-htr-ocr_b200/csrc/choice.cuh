// choice.cuh — the greedy token choice on the device, shared by the LM heads (CUDA-core and tensor-core) and the
// standalone choice: ocr-decode's choose (app/crates/ocr-decode/src/sampling.rs:38-62) as the reference's GPU sampler
// splits it (shaders/choose_pen.wgsl, choose_max.wgsl, choose_pick.wgsl).
#pragma once

#include "kernels.cuh"

namespace ocr {

// ---------------------------------------------------------------------------------------------------------------------
// the token choice: windowed repetition penalty (distinct tokens of the window), frequency penalty, first maximum
// ---------------------------------------------------------------------------------------------------------------------
constexpr int PEN_CAP = 64;     // window tokens listed per CTA and slot (more → the CTA scans the window per row)
constexpr int PEN_BITS = 2048;  // rows of a CTA's range covered by the membership bitmask (wider → the list)
constexpr int MAX_NB = 8;

// the window's tokens that fall in a CTA's row range [lo, hi): a bitmask over the range (one shared load per row,
// however many times a token repeats in the window) and, for ranges wider than the mask, a list
struct PenList {
    int n[MAX_NB];
    int t[MAX_NB][PEN_CAP];
    uint32_t bits[MAX_NB][PEN_BITS / 32];
};

// the window tokens of slot s that fall in [lo, hi): hist[len - min(len, window), len); `nthr` threads take part
// (barrier 1)
__device__ inline void pen_prefilter(PenList& pl, int nb, int slot0, const LmArgs& a, int lo, int hi, int nthr) {
    const int tid = threadIdx.x;
    const bool masked = hi - lo <= PEN_BITS;
    if (tid < MAX_NB) pl.n[tid] = 0;
    if (masked)
        for (int i = tid; i < nb * (PEN_BITS / 32); i += nthr) pl.bits[i / (PEN_BITS / 32)][i % (PEN_BITS / 32)] = 0u;
    bar_sync(1, nthr);
    if (a.sample && a.rp != 1.0f) {
        for (int s = 0; s < nb; s++) {
            const int b = slot0 + s;
            if (a.active && !a.active[b]) continue;
            const int len = a.len[b];
            const int start = len - min(len, a.window);
            const int32_t* h = a.hist + (long)b * a.hist_cap;
            for (int j = start + tid; j < len; j += nthr) {
                const int t = h[j];
                if (t >= lo && t < hi) {
                    if (masked) {
                        atomicOr(&pl.bits[s][(t - lo) >> 5], 1u << ((t - lo) & 31));
                    } else {
                        const int k = atomicAdd(&pl.n[s], 1);
                        if (k < PEN_CAP) pl.t[s][k] = t;
                    }
                }
            }
        }
    }
    bar_sync(1, nthr);
}

// the choice's value of logit v of token t in slot b, given whether t is in the slot's window (choose(): rp on window
// members — a product for negative logits, an IEEE quotient otherwise — then − fp * count)
__device__ __forceinline__ float pen_value(float v, bool member, int b, int t, const LmArgs& a, int n_vocab) {
    if (a.rp != 1.0f && member) v = v < 0.0f ? __fmul_rn(v, a.rp) : __fdiv_rn(v, a.rp);
    if (a.use_fp) {
        const long k = (long)b * (long)n_vocab + t;
        if (a.counts[k] != 0u) v = __fsub_rn(v, a.fpen[k]);
    }
    return v;
}

// the choice's value of logit v of token t (in the CTA's range [lo, hi)) in slot s (choose(): rp on window members,
// then − fp * count)
__device__ __forceinline__ float pen_apply(const PenList& pl, int s, int b, int t, float v, const LmArgs& a,
                                           int n_vocab, int lo, int hi) {
    if (a.rp != 1.0f) {
        const int n = pl.n[s];
        bool member = false;
        if (hi - lo <= PEN_BITS) {
            member = (pl.bits[s][(t - lo) >> 5] >> ((t - lo) & 31)) & 1u;
        } else if (n <= PEN_CAP) {
            for (int k = 0; k < n; k++) member |= (pl.t[s][k] == t);
        } else {
            const int len = a.len[b];
            const int32_t* h = a.hist + (long)b * a.hist_cap;
            for (int j = len - min(len, a.window); j < len && !member; j++) member = (h[j] == t);
        }
        return pen_value(v, member, b, t, a, n_vocab);
    }
    return pen_value(v, false, b, t, a, n_vocab);
}

// The CTA's best per slot → part; the last CTA of the grid row (threadfence + ticket, no waiting) reduces all parts
// and records the choice. Called by every thread of the CTA.
__device__ inline void choice_finish(const float* bv_sm, const uint32_t* bi_sm, int nb, int slot0, const LmArgs& a,
                                     int n_vocab) {
    const int grid = gridDim.x;
    float* part = a.part;  // [B][grid] (value, index) pairs, then [B] NaN-at-token-0 flags
    if (threadIdx.x < nb) {
        const int b = slot0 + threadIdx.x;
        part[((long)b * grid + blockIdx.x) * 2] = bv_sm[threadIdx.x];
        reinterpret_cast<uint32_t*>(part)[((long)b * grid + blockIdx.x) * 2 + 1] = bi_sm[threadIdx.x];
    }
    __threadfence();
    __shared__ uint32_t ticket;
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(&a.done[blockIdx.y], 1u);
    __syncthreads();
    if (ticket != (uint32_t)grid - 1) return;
    __threadfence();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int* nan_flags = reinterpret_cast<const int*>(part + (long)a.nb * grid * 2);
    for (int s = warp; s < nb; s += blockDim.x / 32) {
        const int b = slot0 + s;
        float v = -INFINITY;
        uint32_t idx = NO_INDEX;
        for (int c = lane; c < grid; c += 32) {
            const float w = __ldcg(part + ((long)b * grid + c) * 2);
            const uint32_t j = __ldcg(reinterpret_cast<const uint32_t*>(part) + ((long)b * grid + c) * 2 + 1);
            if (better(w, j, v, idx)) {
                v = w;
                idx = j;
            }
        }
        warp_argmax(v, idx);
        if (lane == 0 && (!a.active || a.active[b])) {
            // every logit NaN, or logit 0 NaN: token 0 (ocr-decode's argmax starts at index 0 and a NaN never loses)
            const int nan0 = __ldcg(nan_flags + b);
            const int32_t t = (idx == NO_INDEX || nan0) ? 0 : (int32_t)idx;
            const int len = a.len[b];
            a.tok[b] = t;
            if (len < a.hist_cap) a.hist[(long)b * a.hist_cap + len] = t;
            else dev_error(a.err, DEV_BAD_INDEX);
            a.len[b] = len + 1;
            if (a.advance_pos) a.pos[b] += 1;
            if (a.remaining) {
                const int32_t r = a.remaining[b] - 1;
                a.remaining[b] = r;
                if (r <= 0 && a.active_w) a.active_w[b] = 0;
            }
            if (a.use_fp) {
                const long k = (long)b * n_vocab + t;
                const uint32_t c = a.counts[k] + 1u;
                a.counts[k] = c;
                a.fpen[k] = __fmul_rn(a.fp, (float)c);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) a.done[blockIdx.y] = 0u;
}

}  // namespace ocr

// k_attn.cu — decode attention of one token per slot over the f16 KV cache, GQA, split over the keys ("flash
// decoding"): the reference's qkv_post.wgsl (q/k RMSNorm → RoPE NEOX → K/V store), attn_decode.wgsl (per-chunk softmax
// partials m, l, o[128]) and attn_merge.wgsl (M = max m, L = Σ l e^(m−M), O = Σ o e^(m−M) / L) in one kernel.
//
// Grid (splits, n_kv, slots), 128 threads. A CTA owns one kv head (its G = n_head / n_kv query heads) and a
// contiguous key range [k0, k1) (≤ KEYS_MAX keys) of the slot's pos + 1 keys; k0, k1 come from the device-side
// position, so one captured graph serves every step. KV layout [slot][kv head][n_ctx][128] f16: the range is one
// contiguous run of K and one of V, each moved into shared memory by one bulk-async copy issued before the kernel
// waits on its predecessor (no earlier kernel still writes those rows; the row at pos is computed here and written to
// both the cache and shared memory). Scores: 8 lanes per key (16 dims each), 4 keys per warp per pass; P·V: a warp per
// key stripe, lane = 4 dims; all from shared memory. The last CTA of a (slot, kv head) to finish merges the partials
// (threadfence + ticket, counter reset by that CTA; no waiting on other CTAs). The one mbarrier wait is bounded.
#include "kernels.cuh"

namespace ocr {

constexpr int AT_THREADS = 128;
constexpr int HD = 128;          // head dim (TextConfig::from_gguf requires 128, text.rs:57-60)
constexpr int KEYS_MAX = 192;    // keys per CTA: K + V tiles 96 KB of shared memory
constexpr int MAX_SPLITS = 256;  // key ranges per (slot, kv head): the merge keeps one weight per range in smem

__device__ __forceinline__ float block_sum128(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    return red[0] + red[1] + red[2] + red[3];
}

__device__ __forceinline__ float block_max128(float v, float* red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    return fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
}

template <int G>
__global__ void __launch_bounds__(AT_THREADS) k_attn_decode(AttnArgs a, int per_max) {
    extern __shared__ __align__(128) uint8_t sm[];
    __half* Ks = reinterpret_cast<__half*>(sm);             // [per_max][128]
    __half* Vs = Ks + (size_t)per_max * HD;                  // [per_max][128]
    float* sc = reinterpret_cast<float*>(Vs + (size_t)per_max * HD);  // [G][per_max]
    __shared__ __align__(8) uint64_t bar;
    __shared__ float qs[G][HD];
    __shared__ float tmp2[G + 1][HD];
    __shared__ float red[4];
    __shared__ float red2[4][G + 1];
    __shared__ float mw[G][MAX_SPLITS];
    __shared__ float lw[G][MAX_SPLITS];
    __shared__ float osum[4][G][HD];
    __shared__ uint32_t ticket;
    const int b = blockIdx.z, j = blockIdx.y, sp = blockIdx.x, t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    const int S = gridDim.x;
    const int n_head = a.n_head;

    // the slot's position was written by the previous step (its last kernel completed before this step began)
    if (a.active && !a.active[b]) return;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.n_ctx) {
        if (sp == 0 && j == 0 && t == 0) dev_error(a.err, DEV_BAD_POS);
        return;
    }
    const int n_keys = pos + 1;
    const int per = (n_keys + S - 1) / S;
    const int k0 = min(n_keys, sp * per), k1 = min(n_keys, k0 + per);
    if (k1 - k0 > per_max) {  // the launch sized per_max for this n_ctx; anything else is a bad position
        if (t == 0) dev_error(a.err, DEV_BAD_POS);
        return;
    }
    const long head_base = ((long)b * a.n_kv + j) * a.n_ctx;
    __half* kb = a.kc + head_base * HD;
    __half* vb = a.vc + head_base * HD;
    const int kend = min(k1, pos);  // rows [k0, kend) are in the cache already; the row at pos is written below
    const bool copy = kend > k0;
    if (t == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        if (copy) {
            const uint32_t bytes = (uint32_t)(kend - k0) * HD * 2;
            mbar_expect_tx(&bar, 2 * bytes);
            bulk_g2s(Ks, kb + (long)k0 * HD, bytes, &bar);
            bulk_g2s(Vs, vb + (long)k0 * HD, bytes, &bar);
        }
        pdl_trigger();
    }
    pdl_wait();

    // q heads (and, in the CTA whose range holds pos, the new k head): RMSNorm x weight, then RoPE NEOX — all heads'
    // loads issued together, one reduction round, one rotation exchange
    const float* qkv = a.qkv + (long)b * a.qkv_stride;
    const float* cs = a.rope + (long)pos * HD;  // [64][2]
    const bool own = pos >= k0 && pos < k1;
    constexpr int NH = G + 1;
    float raw[NH];
#pragma unroll
    for (int g = 0; g < G; g++) raw[g] = qkv[(j * G + g) * HD + t];
    raw[G] = own ? qkv[(a.n_head + j) * HD + t] : 0.0f;
    const float vraw = own ? qkv[(a.n_head + a.n_kv + j) * HD + t] : 0.0f;
    const float wq = a.q_norm[t], wk = a.k_norm[t];
    const float cr = cs[2 * (t & 63)], sr = cs[2 * (t & 63) + 1];
#pragma unroll
    for (int g = 0; g < NH; g++) {
        const float s2 = warp_sum(raw[g] * raw[g]);
        if (lane == 0) red2[warp][g] = s2;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < NH; g++) {
        const float tot = red2[0][g] + red2[1][g] + red2[2][g] + red2[3][g];
        tmp2[g][t] = raw[g] * (1.0f / sqrtf(tot / (float)HD + a.eps)) * (g < G ? wq : wk);
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < NH; g++) {
        const float r = t < 64 ? tmp2[g][t] * cr - tmp2[g][t + 64] * sr : tmp2[g][t - 64] * sr + tmp2[g][t] * cr;
        if (g < G) qs[g][t] = r * a.scale;
        else if (own) {
            // the new token's K / V row: to the cache and to the shared tiles
            const __half kh = __float2half_rn(r), vh = __float2half_rn(vraw);
            kb[(long)pos * HD + t] = kh;
            vb[(long)pos * HD + t] = vh;
            Ks[(pos - k0) * HD + t] = kh;
            Vs[(pos - k0) * HD + t] = vh;
        }
    }
    __syncthreads();
    // every thread waits for the tiles; the CTA leaves together if any wait gave up
    const int ok = copy ? (int)mbar_wait(&bar, 0, a.err) : 1;
    if (!__syncthreads_and(ok)) return;

    // scores: lane group (lane >> 3) takes one key, lane & 7 its 16 dims
    const int n = k1 - k0;
    const int sub = lane >> 3, part = lane & 7;
    float qr[G][16];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < 16; i++) qr[g][i] = qs[g][part * 16 + i];
    for (int base = 0; base < n; base += 16) {
        const int key = base + warp * 4 + sub;
        const bool valid = key < n;
        float d[G];
#pragma unroll
        for (int g = 0; g < G; g++) d[g] = 0.0f;
        if (valid) {
            const uint4* kp = reinterpret_cast<const uint4*>(Ks + key * HD + part * 16);
            const uint4 u0 = kp[0], u1 = kp[1];
            const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
            const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f0 = __half22float2(h0[i]), f1 = __half22float2(h1[i]);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    d[g] = fmaf(qr[g][2 * i], f0.x, d[g]);
                    d[g] = fmaf(qr[g][2 * i + 1], f0.y, d[g]);
                    d[g] = fmaf(qr[g][8 + 2 * i], f1.x, d[g]);
                    d[g] = fmaf(qr[g][8 + 2 * i + 1], f1.y, d[g]);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            d[g] += __shfl_xor_sync(FULL, d[g], 4);
            d[g] += __shfl_xor_sync(FULL, d[g], 2);
            d[g] += __shfl_xor_sync(FULL, d[g], 1);
        }
        if (valid && part == 0)
#pragma unroll
            for (int g = 0; g < G; g++) sc[g * per_max + key] = d[g];
    }
    __syncthreads();
    // softmax of every head at once: one max round, one sum round
    float m[G], l[G];
    {
        float mx[G];
#pragma unroll
        for (int g = 0; g < G; g++) mx[g] = -INFINITY;
        for (int i = t; i < n; i += AT_THREADS)
#pragma unroll
            for (int g = 0; g < G; g++) mx[g] = fmaxf(mx[g], sc[g * per_max + i]);
#pragma unroll
        for (int g = 0; g < G; g++) {
            mx[g] = warp_max(mx[g]);
            if (lane == 0) red2[warp][g] = mx[g];
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < G; g++) m[g] = fmaxf(fmaxf(red2[0][g], red2[1][g]), fmaxf(red2[2][g], red2[3][g]));
        __syncthreads();
        float sm_[G];
#pragma unroll
        for (int g = 0; g < G; g++) sm_[g] = 0.0f;
        for (int i = t; i < n; i += AT_THREADS)
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float p = expf(sc[g * per_max + i] - m[g]);
                sc[g * per_max + i] = p;
                sm_[g] += p;
            }
#pragma unroll
        for (int g = 0; g < G; g++) {
            sm_[g] = warp_sum(sm_[g]);
            if (lane == 0) red2[warp][g] = sm_[g];
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < G; g++) l[g] = (red2[0][g] + red2[1][g]) + (red2[2][g] + red2[3][g]);
    }
    __syncthreads();
    // P·V: warp w takes keys w, w + 4, …; lane owns dims 4 lane … 4 lane + 3
    float o[G][4];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < 4; i++) o[g][i] = 0.0f;
#pragma unroll 4
    for (int key = warp; key < n; key += 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(Vs + key * HD + lane * 4);
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float p = sc[g * per_max + key];
            o[g][0] = fmaf(p, v0.x, o[g][0]);
            o[g][1] = fmaf(p, v0.y, o[g][1]);
            o[g][2] = fmaf(p, v1.x, o[g][2]);
            o[g][3] = fmaf(p, v1.y, o[g][3]);
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < 4; i++) osum[warp][g][lane * 4 + i] = o[g][i];
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int h = j * G + g;
        float* pp = a.part + (((long)b * n_head + h) * S + sp) * (HD + 2);
        const float ov = osum[0][g][t] + osum[1][g][t] + osum[2][g][t] + osum[3][g][t];
        pp[2 + t] = n > 0 ? ov : 0.0f;
        if (t == 0) {
            pp[0] = n > 0 ? m[g] : -INFINITY;
            pp[1] = n > 0 ? l[g] : 0.0f;
        }
    }
    __threadfence();
    __syncthreads();
    if (t == 0) ticket = atomicAdd(&a.done[(long)b * a.n_kv + j], 1u);
    __syncthreads();
    if (ticket != (uint32_t)S - 1) return;
    __threadfence();
    // the merge: every split's (m, l) and this thread's o values loaded in one go; then each thread folds the splits
    // itself (S is small: no reductions, no further round trips unless S > OC)
    constexpr int OC = 64 / G;
    for (int q = t; q < S * G; q += AT_THREADS) {
        const int g = q / S, s2 = q - g * S;
        const float* pp = a.part + (((long)b * n_head + j * G + g) * S + s2) * (HD + 2);
        mw[g][s2] = __ldcg(pp);
        lw[g][s2] = __ldcg(pp + 1);
    }
    float ov[G][OC];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float* pb = a.part + ((long)b * n_head + j * G + g) * S * (HD + 2) + 2 + t;
#pragma unroll
        for (int u = 0; u < OC; u++) ov[g][u] = u < S ? __ldcg(pb + (long)u * (HD + 2)) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < S; s2++) M = fmaxf(M, mw[g][s2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int u = 0; u < OC; u++)
            if (u < S) {
                const float w = expf(mw[g][u] - M);
                L = fmaf(lw[g][u], w, L);
                O = fmaf(ov[g][u], w, O);
            }
        const float* pb = a.part + ((long)b * n_head + j * G + g) * S * (HD + 2) + 2 + t;
        for (int s2 = OC; s2 < S; s2++) {
            const float w = expf(mw[g][s2] - M);
            L = fmaf(lw[g][s2], w, L);
            O = fmaf(__ldcg(pb + (long)s2 * (HD + 2)), w, O);
        }
        a.out[(long)b * a.out_stride + (j * G + g) * HD + t] = O / L;
    }
    if (t == 0) a.done[(long)b * a.n_kv + j] = 0u;
}

int attention_splits(int num_sms, int nb, int n_kv, int n_ctx) {
    // one wave of CTAs at least; at most KEYS_MAX keys per CTA at the session's longest context
    const int heads = nb * n_kv;
    int s = (num_sms + heads - 1) / heads;
    const int min_s = (n_ctx + KEYS_MAX - 1) / KEYS_MAX;
    if (s < min_s) s = min_s;
    if (s > n_ctx) s = n_ctx;
    if (s > MAX_SPLITS) s = MAX_SPLITS;  // (n_ctx <= MAX_SPLITS * KEYS_MAX, checked at session creation)
    if (s < 1) s = 1;
    return s;
}

template <int G>
static void launch_t(cudaStream_t st, const AttnArgs& a, bool pdl) {
    const int per_max = (a.n_ctx + a.splits - 1) / a.splits;
    const size_t smem = (size_t)per_max * HD * 2 * 2 + (size_t)G * per_max * sizeof(float);
    auto kern = k_attn_decode<G>;
    static bool configured = false;
    if (!configured) {
        // the opt-in limit: what the SM offers a CTA minus this kernel's static shared memory
        cudaFuncAttributes fa;
        cudaFuncGetAttributes(&fa, kern);
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - (int)fa.sharedSizeBytes);
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.splits, (unsigned)a.n_kv, (unsigned)a.nb);
    cfg.blockDim = dim3(AT_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, a, per_max);
}

void launch_attention_decode(cudaStream_t st, const AttnArgs& a, bool pdl) {
    const int G = a.n_head / a.n_kv;
    if (G == 1) launch_t<1>(st, a, pdl);
    else if (G == 2) launch_t<2>(st, a, pdl);
    else if (G == 4) launch_t<4>(st, a, pdl);
    else launch_t<8>(st, a, pdl);
}

}  // namespace ocr

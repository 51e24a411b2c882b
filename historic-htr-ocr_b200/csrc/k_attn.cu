// k_attn.cu — decode attention of one token per slot over the f16 KV cache, GQA, split over the keys ("flash
// decoding"): the reference's qkv_post.wgsl (q/k RMSNorm → RoPE NEOX → K/V store), attn_decode.wgsl (per-chunk softmax
// partials m, l, o[128]) and attn_merge.wgsl (M = max m, L = Σ l e^(m−M), O = Σ o e^(m−M) / L) in one kernel.
//
// Grid (splits, n_kv, slots), 128 threads. A CTA owns one kv head (its G = n_head / n_kv query heads) and one
// contiguous key range [k0, k1) of the slot's pos + 1 keys (k0, k1 from the device-side position, so one captured
// graph serves every step). KV cache layout [slot][kv head][n_ctx][128] f16: a key range is one contiguous run,
// prefetched into L2 with a bulk prefetch before the kernel waits on its predecessor (no earlier kernel writes those
// rows: the position comes from the previous step, and the row at pos is written here). Scores: 8 lanes per key
// (16 dims each, two 16-B loads), 4 keys per warp per pass. P·V: a warp per key stripe, lane = 4 dims. The last CTA
// of a (slot, kv head) to finish merges the partials (threadfence + ticket, counter reset by that CTA).
#include "kernels.cuh"

namespace ocr {

constexpr int AT_THREADS = 128;
constexpr int HD = 128;  // head dim (TextConfig::from_gguf requires 128, text.rs:57-60)

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

// RMSNorm(head) * w, then NEOX rotation of (i, i + 64) by the table row `cs` — thread t owns dim t
__device__ __forceinline__ float norm_rope(float raw, const float* w, const float* cs, float eps, float* red,
                                           float* tmp) {
    const int t = threadIdx.x;
    const float ss = block_sum128(raw * raw, red);
    const float y = raw * (1.0f / sqrtf(ss / (float)HD + eps)) * w[t];
    tmp[t] = y;
    __syncthreads();
    const int k = t & 63;
    const float c = cs[2 * k], s = cs[2 * k + 1];
    const float r = t < 64 ? tmp[t] * c - tmp[t + 64] * s : tmp[t - 64] * s + tmp[t] * c;
    __syncthreads();
    return r;
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <int G>
__global__ void __launch_bounds__(AT_THREADS) k_attn_decode(AttnArgs a, int per_max) {
    extern __shared__ float sc[];  // [G][per_max] scores → probabilities
    __shared__ float qs[G][HD];
    __shared__ float tmp[HD];
    __shared__ float red[4];
    __shared__ float osum[4][G][HD];
    __shared__ float ml[G][2];
    __shared__ uint32_t ticket;
    const int b = blockIdx.z, j = blockIdx.y, sp = blockIdx.x, t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    const int S = gridDim.x;

    // the slot's position was written by an earlier step (complete before this grid's predecessor triggered)
    if (a.active && !a.active[b]) return;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.n_ctx) {
        if (sp == 0 && j == 0 && t == 0) dev_error(a.err, DEV_BAD_POS);
        return;
    }
    const int n_keys = pos + 1;
    const int per = (n_keys + S - 1) / S;
    const int k0 = min(n_keys, sp * per), k1 = min(n_keys, k0 + per);
    const long head_base = ((long)b * a.n_kv + j) * a.n_ctx;
    const __half* kb = a.kc + head_base * HD;
    const __half* vb = a.vc + head_base * HD;
    if (t == 0) {
        const int kend = min(k1, pos);  // the row at pos is written below
        if (kend > k0) {
            prefetch_l2(kb + (long)k0 * HD, (uint32_t)(kend - k0) * HD * 2);
            prefetch_l2(vb + (long)k0 * HD, (uint32_t)(kend - k0) * HD * 2);
        }
    }
    pdl_wait();

    const float* qkv = a.qkv + (long)b * a.qkv_stride;
    const float* cs = a.rope + (long)pos * HD;  // [64][2]
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float r = norm_rope(qkv[(j * G + g) * HD + t], a.q_norm, cs, a.eps, red, tmp);
        qs[g][t] = r * a.scale;
    }
    // the new token's K / V row (the CTA whose range holds pos)
    if (pos >= k0 && pos < k1) {
        const float kr = norm_rope(qkv[(a.n_head + j) * HD + t], a.k_norm, cs, a.eps, red, tmp);
        const_cast<__half*>(kb)[(long)pos * HD + t] = __float2half_rn(kr);
        const_cast<__half*>(vb)[(long)pos * HD + t] = __float2half_rn(qkv[(a.n_head + a.n_kv + j) * HD + t]);
    }
    __syncthreads();

    // scores: lane group (lane >> 3) takes one key, lane & 7 its 16 dims
    const int sub = lane >> 3, part = lane & 7;
    float qr[G][16];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < 16; i++) qr[g][i] = qs[g][part * 16 + i];
    for (int base = k0; base < k1; base += 16) {
        const int key = base + warp * 4 + sub;
        const bool valid = key < k1;
        float d[G];
#pragma unroll
        for (int g = 0; g < G; g++) d[g] = 0.0f;
        if (valid) {
            const uint4* kp = reinterpret_cast<const uint4*>(kb + (long)key * HD + part * 16);
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
            for (int g = 0; g < G; g++) sc[g * per_max + key - k0] = d[g];
    }
    __syncthreads();
    const int n = k1 - k0;
    float m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        float mx = -INFINITY;
        for (int i = t; i < n; i += AT_THREADS) mx = fmaxf(mx, sc[g * per_max + i]);
        m[g] = block_max128(mx, red);
        float s = 0.0f;
        for (int i = t; i < n; i += AT_THREADS) {
            const float p = expf(sc[g * per_max + i] - m[g]);
            sc[g * per_max + i] = p;
            s += p;
        }
        l[g] = block_sum128(s, red);
    }
    __syncthreads();
    // P·V: warp w takes keys k0 + w, k0 + w + 4, …; lane owns dims 4 lane … 4 lane + 3
    float o[G][4];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < 4; i++) o[g][i] = 0.0f;
    for (int key = k0 + warp; key < k1; key += 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(vb + (long)key * HD + lane * 4);
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float p = sc[g * per_max + key - k0];
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
    pdl_trigger();
    const int n_head = a.n_head;
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
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int h = j * G + g;
        const float* pb = a.part + ((long)b * n_head + h) * S * (HD + 2);
        if (t < 32) {
            float mx = -INFINITY;
            for (int s = t; s < S; s += 32) mx = fmaxf(mx, __ldcg(pb + (long)s * (HD + 2)));
            mx = warp_max(mx);
            float L = 0.0f;
            for (int s = t; s < S; s += 32) {
                const float ms = __ldcg(pb + (long)s * (HD + 2));
                L += __ldcg(pb + (long)s * (HD + 2) + 1) * expf(ms - mx);
            }
            L = warp_sum(L);
            if (t == 0) {
                ml[g][0] = mx;
                ml[g][1] = L;
            }
        }
        __syncthreads();
        const float M = ml[g][0];
        float O = 0.0f;
        for (int s = 0; s < S; s++) {
            const float ms = __ldcg(pb + (long)s * (HD + 2));
            O = fmaf(__ldcg(pb + (long)s * (HD + 2) + 2 + t), expf(ms - M), O);
        }
        a.out[(long)b * a.out_stride + h * HD + t] = O / ml[g][1];
    }
    if (t == 0) a.done[(long)b * a.n_kv + j] = 0u;
}

int attention_splits(int num_sms, int nb, int n_kv, int n_ctx) {
    const int heads = nb * n_kv;
    int s = (4 * num_sms + heads - 1) / heads;
    const int min_s = (n_ctx + 4095) / 4096;  // at most 4096 keys per CTA (shared-memory score buffer)
    if (s < min_s) s = min_s;
    if (s > n_ctx) s = n_ctx;
    if (s < 1) s = 1;
    return s;
}

size_t attention_smem(const AttnArgs& a) {
    const int per_max = (a.n_ctx + a.splits - 1) / a.splits;
    return (size_t)(a.n_head / a.n_kv) * per_max * sizeof(float);
}

template <int G>
static void launch_t(cudaStream_t st, const AttnArgs& a, bool pdl) {
    const int per_max = (a.n_ctx + a.splits - 1) / a.splits;
    const size_t smem = attention_smem(a);
    auto kern = k_attn_decode<G>;
    static int configured = 0;
    if (!configured) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        configured = 1;
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

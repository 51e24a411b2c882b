// stage.cuh — the activation row of a decode kernel, staged once per CTA in shared memory: loaded after the
// kernel's dependency wait (from the embedding table, or the residual plus the previous kernel's partial products),
// RMS-normalised, in the lane-blocked layout of the q8_0 dot (qdot.cuh). Shared by the matvec and the fused FFN.
#pragma once

#include "kernels.cuh"
#include "qdot.cuh"

namespace ocr {

// sum over the `nthr` consumer threads (barrier 1)
__device__ __forceinline__ float consumer_sum(float v, float* red, int nthr) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    bar_sync(1, nthr);
    if (lane == 0) red[warp] = v;
    bar_sync(1, nthr);
    float t = 0.0f;
    for (int k = 0; k < nthr / 32; k++) t += red[k];
    return t;
}

// x rows → smem in the lane-blocked layout (x_out written by the `writer` CTA): from the embedding table when a.tok, plus the partial products when
// a.xadd, RMS-normalised and scaled by the norm weights when a.nw. Two shapes. One float4 per thread (K <= 4 x the
// threads: every normed input here, its norm weights `wn0` loaded by the caller before its dependency wait): the
// row's loads all in flight at once, the values held in registers across the norm's reduction. Wider rows in
// passes of XU float4s per thread, every load of a pass issued before any is used.
// KT: the row length fixed at compile time (0: a.w.cols); NADD_T: the count of partial products (0: a.n_add).
constexpr int XU = 8;
template <int KT = 0, int NADD_T = 0>
__device__ __forceinline__ void stage_x(float* xsf, int nch, int nb, int slot0, const MvArgs& a, float* red, int nthr,
                                    float4 wn0, bool writer) {
    const int K = KT ? KT : a.w.cols, K4 = K >> 2;
    const int n_add = NADD_T ? NADD_T : a.n_add;
    const bool write_x = a.x_out != nullptr && writer;
    float4* xs4 = reinterpret_cast<float4*>(xsf);
    const int tid = threadIdx.x;
    for (int s = 0; s < nb; s++) {
        const int b = slot0 + s;
        const uint8_t* er = nullptr;
        if (a.tok) {
            const int t = a.tok[b];
            if (t >= 0 && t < a.emb.rows) er = a.emb.w + (long)t * a.emb.stride;
        }
        // element group i4 (4 columns) of the input row
        auto load = [&](int i4) -> float4 {
            if (a.tok) {
                if (!er) return make_float4(0.f, 0.f, 0.f, 0.f);
                const uint32_t q = *reinterpret_cast<const uint32_t*>(er + 4 * i4);
                const float d = __half2float(reinterpret_cast<const __half*>(er + K)[i4 >> 3]);
                return make_float4((float)(int8_t)(q & 0xff) * d, (float)(int8_t)((q >> 8) & 0xff) * d,
                                   (float)(int8_t)((q >> 16) & 0xff) * d, (float)(int8_t)(q >> 24) * d);
            }
            return reinterpret_cast<const float4*>(a.x + (long)b * a.x_stride)[i4];
        };
        float4* xo = write_x ? reinterpret_cast<float4*>(a.x_out + (long)b * a.x_stride) : nullptr;
        if (K4 <= nthr) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (tid < K4) {
                if (a.xadd) {
                    // x + (p_0 + … + p_{n-1}): every load in flight, the partials summed in order
                    const float4* pa = reinterpret_cast<const float4*>(a.xadd) + (long)b * n_add * K4 + tid;
                    float4 pv[MAX_ADD];
                    v = load(tid);
#pragma unroll
                    for (int k = 0; k < MAX_ADD; k++)
                        if (k < n_add) pv[k] = pa[(long)k * K4];
                    float4 o = pv[0];
#pragma unroll
                    for (int k = 1; k < MAX_ADD; k++)
                        if (k < n_add) o = make_float4(o.x + pv[k].x, o.y + pv[k].y, o.z + pv[k].z, o.w + pv[k].w);
                    v = make_float4(v.x + o.x, v.y + o.y, v.z + o.z, v.w + o.w);
                } else {
                    v = load(tid);
                }
                if (xo) xo[tid] = v;
            }
            if (a.nw) {
                const float ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, v.w * v.w)));
                const float tot = consumer_sum(ss, red, nthr);
                const float scale = 1.0f / sqrtf(tot / (float)K + a.eps);
                v = make_float4(v.x * scale * wn0.x, v.y * scale * wn0.y, v.z * scale * wn0.z, v.w * scale * wn0.w);
            }
            if (tid < K4) xs4[xs_index(s, nch, 4 * tid) >> 2] = v;
        } else {
            float ss = 0.0f;
            for (int base = 0; base < K4; base += XU * nthr) {
                float4 v[XU];
#pragma unroll
                for (int u = 0; u < XU; u++) {
                    const int i4 = base + u * nthr + tid;
                    if (i4 < K4) v[u] = load(i4);
                }
#pragma unroll
                for (int u = 0; u < XU; u++) {
                    const int i4 = base + u * nthr + tid;
                    if (i4 < K4) {
                        if (xo) xo[i4] = v[u];
                        ss = fmaf(v[u].x, v[u].x, fmaf(v[u].y, v[u].y, fmaf(v[u].z, v[u].z, fmaf(v[u].w, v[u].w, ss))));
                        xs4[xs_index(s, nch, 4 * i4) >> 2] = v[u];
                    }
                }
            }
            if (a.nw) {
                const float tot = consumer_sum(ss, red, nthr);
                const float scale = 1.0f / sqrtf(tot / (float)K + a.eps);
                for (int c = tid; c < K; c += nthr) {
                    const int k = xs_index(s, nch, c);
                    xsf[k] = xsf[k] * scale * a.nw[c];
                }
            }
        }
        // the last chunk's columns past K: lanes there see zero quants, the staged values must be finite
        for (int c = K + 4 * tid; c < nch * 512; c += 4 * nthr) xs4[xs_index(s, nch, c) >> 2] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

}  // namespace ocr

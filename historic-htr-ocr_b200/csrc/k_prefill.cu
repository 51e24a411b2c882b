// k_prefill.cu — the prompt's batch evaluation (TextModel::prefill, text.rs:437-521): embedding gather
// (embed_q8_0.wgsl), row RMSNorm (rms_norm.wgsl), the q8_0 projections as a tiled f32 GEMM with dequantization on
// load (matmul.wgsl's product), q/k norm + RoPE + K/V store (rms_norm + rope_neox + kv_store.wgsl), and causal GQA
// flash attention over the f16 cache (attention_causal.wgsl). f32 arithmetic throughout, like the reference's F32
// path; this fills the KV cache the decode reads.
#include "kernels.cuh"

namespace ocr {

// ---- embedding gather: rows with ids[r] >= 0 take token_embd[ids[r]]; others keep what was copied there -------------
__global__ void k_embed_rows(const int32_t* __restrict__ ids, int n, QMat emb, float* __restrict__ x) {
    const int dim = emb.cols;
    const long total = (long)n * dim;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / dim), c = (int)(i % dim);
        const int t = ids[r];
        if (t >= 0 && t < emb.rows) {
            const uint8_t* row = emb.w + (long)t * emb.stride;
            x[i] = (float)(int8_t)row[c] * __half2float(reinterpret_cast<const __half*>(row + dim)[c / 32]);
        }
    }
}

void launch_embed_rows(cudaStream_t st, const int32_t* ids, int n, QMat emb, float* x) {
    const long total = (long)n * emb.cols;
    int grid = (int)((total + 255) / 256);
    if (grid > 4096) grid = 4096;
    k_embed_rows<<<grid, 256, 0, st>>>(ids, n, emb, x);
}

// ---- RMSNorm rows: y = x * (1 / sqrt(mean x^2 + eps)) * w ------------------------------------------------------------
__global__ void k_rmsnorm_rows(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                               int dim, float eps) {
    __shared__ float red[8];
    const float* xr = x + (long)blockIdx.x * dim;
    float s = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.0f;
    for (int k = 0; k < (int)(blockDim.x >> 5); k++) t += red[k];
    const float scale = 1.0f / sqrtf(t / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) y[(long)blockIdx.x * dim + i] = xr[i] * scale * w[i];
}

void launch_rmsnorm_rows(cudaStream_t st, const float* x, const float* w, float* y, int rows, int dim, float eps) {
    k_rmsnorm_rows<<<rows, 256, 0, st>>>(x, w, y, dim, eps);
}

// ---- GEMM: Y[L][N] (+)= X[L][K] . W[N][K]^T, W q8_0; tile 128 x 128 x 32 (one q8_0 block per W row per k-step) ------
constexpr int GM = 128, GN = 128, GK = 32;

__global__ void __launch_bounds__(256) k_gemm_q8_0(const float* __restrict__ X, int L, QMat W, float* __restrict__ Y,
                                                   int accumulate, int swiglu) {
    __shared__ __align__(16) float As[GK][GM];
    __shared__ __align__(16) float Bs[GK][GN];
    const int K = W.cols, N = W.rows;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * GM, n0 = blockIdx.x * GN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += GK) {
        // X tile: 128 rows x 32 floats = 1024 float4, 4 per thread
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int f = tid + u * 256;
            const int r = f & (GM - 1), c4 = f >> 7;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m0 + r < L) v = *reinterpret_cast<const float4*>(X + (long)(m0 + r) * K + k0 + c4 * 4);
            As[c4 * 4 + 0][r] = v.x;
            As[c4 * 4 + 1][r] = v.y;
            As[c4 * 4 + 2][r] = v.z;
            As[c4 * 4 + 3][r] = v.w;
        }
        // W tile: 128 rows x 32 int8 (one block each): thread = (row tid / 2, 16 quants)
        {
            const int r = tid >> 1, h = tid & 1;
            float wf[16];
            if (n0 + r < N) {
                const uint8_t* row = W.w + (long)(n0 + r) * W.stride;
                const uint4 q = *reinterpret_cast<const uint4*>(row + k0 + h * 16);
                const float d = __half2float(reinterpret_cast<const __half*>(row + K)[k0 / 32]);
                i8x4_to_f32(q.x, wf + 0);
                i8x4_to_f32(q.y, wf + 4);
                i8x4_to_f32(q.z, wf + 8);
                i8x4_to_f32(q.w, wf + 12);
#pragma unroll
                for (int k = 0; k < 16; k++) wf[k] *= d;
            } else {
#pragma unroll
                for (int k = 0; k < 16; k++) wf[k] = 0.0f;
            }
#pragma unroll
            for (int k = 0; k < 16; k++) Bs[h * 16 + k][r] = wf[k];
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < GK; k++) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[k][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[k][ty * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[k][tx * 8]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[k][tx * 8 + 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m = m0 + ty * 8 + i;
        if (m >= L) continue;
        if (swiglu) {
            const int N2 = N / 2;
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const int n = n0 + tx * 8 + j;
                if (n + 1 < N) {
                    const float g = acc[i][j], u = acc[i][j + 1];
                    Y[(long)m * N2 + n / 2] = g / (1.0f + expf(-g)) * u;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int n = n0 + tx * 8 + j;
                if (n < N) {
                    float* yp = Y + (long)m * N + n;
                    *yp = accumulate ? *yp + acc[i][j] : acc[i][j];
                }
            }
        }
    }
}

void launch_gemm_q8_0(cudaStream_t st, const float* x, int L, QMat w, float* y, int accumulate, int swiglu) {
    dim3 grid((w.rows + GN - 1) / GN, (L + GM - 1) / GM, 1);
    k_gemm_q8_0<<<grid, 256, 0, st>>>(x, L, w, y, accumulate, swiglu);
}

// ---- q/k head norm + RoPE (q in place), K/V rows → the f16 cache ------------------------------------------------------
__global__ void k_qk_norm_rope_store(float* __restrict__ qkv, int n_head, int n_kv, const float* __restrict__ q_norm,
                                     const float* __restrict__ k_norm, const float* __restrict__ rope, int pos0,
                                     float eps, __half* __restrict__ kc, __half* __restrict__ vc, int n_ctx) {
    __shared__ float red[4];
    __shared__ float tmp[128];
    const int r = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
    const int width = (n_head + 2 * n_kv) * 128;
    float* row = qkv + (long)r * width;
    const int pos = pos0 + r;
    if (h >= n_head + n_kv) {
        const int j = h - n_head - n_kv;
        vc[((long)j * n_ctx + pos) * 128 + t] = __float2half_rn(row[h * 128 + t]);
        return;
    }
    const float x = row[h * 128 + t];
    float s = warp_sum(x * x);
    if ((t & 31) == 0) red[t >> 5] = s;
    __syncthreads();
    const float tot = red[0] + red[1] + red[2] + red[3];
    const float* w = h < n_head ? q_norm : k_norm;
    const float y = x * (1.0f / sqrtf(tot / 128.0f + eps)) * w[t];
    tmp[t] = y;
    __syncthreads();
    const float* cs = rope + (long)pos * 128;
    const int k = t & 63;
    const float c = cs[2 * k], sn = cs[2 * k + 1];
    const float o = t < 64 ? tmp[t] * c - tmp[t + 64] * sn : tmp[t - 64] * sn + tmp[t] * c;
    if (h < n_head) row[h * 128 + t] = o;
    else kc[((long)(h - n_head) * n_ctx + pos) * 128 + t] = __float2half_rn(o);
}

void launch_qk_norm_rope_store(cudaStream_t st, float* qkv, int L, int n_head, int n_kv, const float* q_norm,
                               const float* k_norm, const float* rope, int pos0, float eps, __half* kc, __half* vc,
                               int n_ctx) {
    k_qk_norm_rope_store<<<dim3(L, n_head + 2 * n_kv, 1), 128, 0, st>>>(qkv, n_head, n_kv, q_norm, k_norm, rope, pos0,
                                                                        eps, kc, vc, n_ctx);
}

// ---- causal flash attention (f32 tiles of 64 queries x 64 keys, online softmax) -----------------------------------------
constexpr int FQ = 64, FK = 64;

__global__ void __launch_bounds__(256) k_attn_prefill(const float* __restrict__ qkv, int L, int n_head, int n_kv,
                                                      const __half* __restrict__ kc, const __half* __restrict__ vc,
                                                      int n_ctx, int pos0, float scale, float* __restrict__ out) {
    extern __shared__ float smf[];
    float* Qs = smf;                 // [128][FQ]  (dim-major)
    float* Ks = Qs + 128 * FQ;       // [128][FK]
    float* Vs = Ks + 128 * FK;       // [FK][128]
    float* Ps = Vs + FK * 128;       // [FK][FQ]
    const int h = blockIdx.y, kh = h / (n_head / n_kv);
    const int q0 = blockIdx.x * FQ;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int width = (n_head + 2 * n_kv) * 128;
    // Q tile (pre-scaled), dim-major
    for (int f = tid; f < FQ * 128; f += 256) {
        const int i = f & (FQ - 1), d = f >> 6;
        Qs[d * FQ + i] = (q0 + i < L) ? qkv[(long)(q0 + i) * width + h * 128 + d] * scale : 0.0f;
    }
    float o[4][8];
    float mrow[4], lrow[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        mrow[i] = -INFINITY;
        lrow[i] = 0.0f;
#pragma unroll
        for (int d = 0; d < 8; d++) o[i][d] = 0.0f;
    }
    const int q_last = min(L, q0 + FQ) - 1;
    const int n_keys = pos0 + q_last + 1;
    const __half* kbase = kc + (long)kh * n_ctx * 128;
    const __half* vbase = vc + (long)kh * n_ctx * 128;
    for (int kb0 = 0; kb0 < n_keys; kb0 += FK) {
        __syncthreads();
        // K dim-major (key index fastest: conflict-free stores), V key-major (dim fastest: coalesced loads)
        for (int f = tid; f < FK * 64; f += 256) {
            const int j = f & (FK - 1), d2 = f >> 6;
            float2 kv = make_float2(0.f, 0.f);
            if (kb0 + j < n_keys) kv = __half22float2(reinterpret_cast<const __half2*>(kbase + (long)(kb0 + j) * 128)[d2]);
            Ks[(2 * d2) * FK + j] = kv.x;
            Ks[(2 * d2 + 1) * FK + j] = kv.y;
        }
        for (int f = tid; f < FK * 64; f += 256) {
            const int j = f >> 6, d2 = f & 63;
            float2 vv = make_float2(0.f, 0.f);
            if (kb0 + j < n_keys) vv = __half22float2(reinterpret_cast<const __half2*>(vbase + (long)(kb0 + j) * 128)[d2]);
            Vs[j * 128 + 2 * d2] = vv.x;
            Vs[j * 128 + 2 * d2 + 1] = vv.y;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < 128; d++) {
            const float4 qv = *reinterpret_cast<const float4*>(Qs + d * FQ + ty * 4);
            const float4 kv = *reinterpret_cast<const float4*>(Ks + d * FK + tx * 4);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = fmaf(qa[i], ka[j], s[i][j]);
        }
        // causal mask + online softmax (a row's 64 scores live in the 16 threads of one half-warp)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qpos = pos0 + q0 + ty * 4 + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (kb0 + tx * 4 + j > qpos) s[i][j] = -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, off));
            const float mnew = fmaxf(mrow[i], mx);
            const float corr = mnew == -INFINITY ? 1.0f : expf(mrow[i] - mnew);
            float ps = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float p = mnew == -INFINITY ? 0.0f : expf(s[i][j] - mnew);
                s[i][j] = p;
                ps += p;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(FULL, ps, off);
            lrow[i] = lrow[i] * corr + ps;
            mrow[i] = mnew;
#pragma unroll
            for (int d = 0; d < 8; d++) o[i][d] *= corr;
#pragma unroll
            for (int j = 0; j < 4; j++) Ps[(tx * 4 + j) * FQ + ty * 4 + i] = s[i][j];
        }
        __syncthreads();
#pragma unroll 4
        for (int j = 0; j < FK; j++) {
            const float4 pv = *reinterpret_cast<const float4*>(Ps + j * FQ + ty * 4);
            const float4 v0 = *reinterpret_cast<const float4*>(Vs + j * 128 + tx * 8);
            const float4 v1 = *reinterpret_cast<const float4*>(Vs + j * 128 + tx * 8 + 4);
            const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
            const float va[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int d = 0; d < 8; d++) o[i][d] = fmaf(pa[i], va[d], o[i][d]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = q0 + ty * 4 + i;
        if (q >= L) continue;
        float* op = out + (long)q * n_head * 128 + h * 128 + tx * 8;
#pragma unroll
        for (int d = 0; d < 8; d++) op[d] = o[i][d] / lrow[i];
    }
}

void launch_attention_prefill(cudaStream_t st, const float* qkv, int L, int n_head, int n_kv, const __half* kc,
                              const __half* vc, int n_ctx, int pos0, float scale, float* out) {
    const size_t smem = (size_t)(128 * FQ + 128 * FK + FK * 128 + FK * FQ) * sizeof(float);
    static PerDeviceOnce once;  // the attribute lives in each device's context
    once([&] { cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
    k_attn_prefill<<<dim3((L + FQ - 1) / FQ, n_head, 1), 256, smem, st>>>(qkv, L, n_head, n_kv, kc, vc, n_ctx, pos0,
                                                                          scale, out);
}

}  // namespace ocr

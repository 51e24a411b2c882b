// k_matvec.cu — q8_0 dequant-matvec for decode (the reference's dmv / dmv_norm / dmv_qkv / dmv_ffn / matvec_q8_0
// kernels, shaders/*.wgsl) and the LM head fused with the greedy token choice (choose_pen / choose_max / choose_pick).
//
// Mapping (256 threads = 8 warps): a warp owns R rows at a time; lane l reads, per 512-column chunk i, the 16 quants at
// columns 512 i + 16 l (one 16-B streaming load per row: the warp's 32 loads are one contiguous 512 B) and the f16
// scale of their block. The activations x (NB slots, RMSNorm and the norm weight folded in when asked) sit in shared
// memory "lane-blocked" — float4 index ((s * nch + i) * 4 + j4) * 32 + l holds x[s][512 i + 16 l + 4 j4 … +4] — so the
// 4 float4 reads a lane makes per chunk are bank-conflict free. int8 → f32 by byte-permute into 2^23's mantissa.
// Per row: lane partial = sum over its half-blocks of scale * dot16; warp butterfly sum; the epilogue stores, adds the
// residual, or pairs interleaved gate/up rows into silu(gate) * up.
#include "kernels.cuh"

namespace ocr {

constexpr int MV_WARPS = 8;
constexpr int MV_THREADS = MV_WARPS * 32;

// dot of 16 dequantized quants (one 16-B load) with the lane's 16 activations of chunk i (4 float4 in smem)
__device__ __forceinline__ float dot16(const float* wf, const float4* xs4, int base, int lane) {
    const float4 a = xs4[base + 0 * 32 + lane];
    const float4 b = xs4[base + 1 * 32 + lane];
    const float4 c = xs4[base + 2 * 32 + lane];
    const float4 e = xs4[base + 3 * 32 + lane];
    float s0 = wf[0] * a.x, s1 = wf[1] * a.y, s2 = wf[2] * a.z, s3 = wf[3] * a.w;
    s0 = fmaf(wf[4], b.x, s0);
    s1 = fmaf(wf[5], b.y, s1);
    s2 = fmaf(wf[6], b.z, s2);
    s3 = fmaf(wf[7], b.w, s3);
    s0 = fmaf(wf[8], c.x, s0);
    s1 = fmaf(wf[9], c.y, s1);
    s2 = fmaf(wf[10], c.z, s2);
    s3 = fmaf(wf[11], c.w, s3);
    s0 = fmaf(wf[12], e.x, s0);
    s1 = fmaf(wf[13], e.y, s1);
    s2 = fmaf(wf[14], e.z, s2);
    s3 = fmaf(wf[15], e.w, s3);
    return (s0 + s1) + (s2 + s3);
}

__device__ __forceinline__ void unpack16(const uint4 w, float* wf) {
    i8x4_to_f32(w.x, wf + 0);
    i8x4_to_f32(w.y, wf + 4);
    i8x4_to_f32(w.z, wf + 8);
    i8x4_to_f32(w.w, wf + 12);
}

// the smem float index of x[s][c] in the lane-blocked layout
__device__ __forceinline__ int xs_index(int s, int nch, int c) {
    const int i = c >> 9, w = c & 511, l = w >> 4, j = w & 15;
    return ((((s * nch + i) * 4 + (j >> 2)) * 32 + l) << 2) + (j & 3);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < MV_WARPS; k++) t += red[k];
    return t;
}

// x rows → smem (optionally from the embedding table, optionally RMS-normalised and scaled by nw)
template <int NB>
__device__ __forceinline__ void stage_x(float* xsf, int nch, int K, int nb, int slot0, const float* x, int x_stride,
                                        const float* nw, float eps, const int32_t* tok, const QMat& emb, float* x_out,
                                        bool write_x, float* red) {
    for (int s = 0; s < nb; s++) {
        const int b = slot0 + s;
        float ss = 0.0f;
        int t = -1;
        if (tok) {
            t = tok[b];
            if (t < 0 || t >= emb.rows) t = -1;
        }
        for (int c = threadIdx.x; c < K; c += MV_THREADS) {
            float v;
            if (tok) v = t < 0 ? 0.0f : (float)emb.q[(long)t * K + c] * __half2float(emb.d[(long)t * (K / 32) + c / 32]);
            else v = x[(long)b * x_stride + c];
            if (write_x) x_out[(long)b * x_stride + c] = v;  // idle slots get zeros (scratch only)
            ss = fmaf(v, v, ss);
            xsf[xs_index(s, nch, c)] = v;
        }
        if (nw) {
            const float tot = block_sum(ss, red);
            const float scale = 1.0f / sqrtf(tot / (float)K + eps);
            for (int c = threadIdx.x; c < K; c += MV_THREADS) {
                const int k = xs_index(s, nch, c);
                xsf[k] = xsf[k] * scale * nw[c];
            }
        }
    }
}

template <int NB, int R, int CH>
__global__ void __launch_bounds__(MV_THREADS) k_matvec(MvArgs a) {
    extern __shared__ float4 xs4[];
    __shared__ float red[MV_WARPS];
    float* xsf = reinterpret_cast<float*>(xs4);
    const int K = a.w.cols, N = a.w.rows;
    const int nch = (K + 511) >> 9;
    const int slot0 = blockIdx.y * NB;
    const int nb = min(NB, a.nb - slot0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    pdl_wait();
    stage_x<NB>(xsf, nch, K, nb, slot0, a.x, a.x_stride, a.nw, a.eps, a.tok, a.emb, a.x_out,
                a.x_out != nullptr && blockIdx.x == 0, red);
    __syncthreads();

    const long groups = (N + R - 1) / R;
    const int kb = K >> 5;
    for (long g = (long)blockIdx.x * MV_WARPS + warp; g < groups; g += (long)gridDim.x * MV_WARPS) {
        const int row0 = (int)(g * R);
        float acc[NB][R];
#pragma unroll
        for (int s = 0; s < NB; s++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[s][r] = 0.0f;
        for (int i0 = 0; i0 < nch; i0 += CH) {
            uint4 wq[CH][R];
            float wd[CH][R];
#pragma unroll
            for (int ci = 0; ci < CH; ci++) {
                const int col = (i0 + ci) * 512 + lane * 16;
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int row = row0 + r;
                    if (i0 + ci < nch && row < N && col < K) {
                        wq[ci][r] = ld_stream(a.w.q + (long)row * K + col);
                        wd[ci][r] = __half2float(a.w.d[(long)row * kb + (col >> 5)]);
                    } else {
                        wq[ci][r] = make_uint4(0, 0, 0, 0);
                        wd[ci][r] = 0.0f;
                    }
                }
            }
#pragma unroll
            for (int ci = 0; ci < CH; ci++) {
                if (i0 + ci >= nch) break;
#pragma unroll
                for (int r = 0; r < R; r++) {
                    float wf[16];
                    unpack16(wq[ci][r], wf);
#pragma unroll
                    for (int s = 0; s < NB; s++)
                        if (s < nb) acc[s][r] = fmaf(dot16(wf, xs4, (s * nch + i0 + ci) * 128, lane), wd[ci][r], acc[s][r]);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < NB; s++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[s][r] = warp_sum(acc[s][r]);
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < NB; s++) {
                if (s >= nb) break;
                const int b = slot0 + s;
                if (a.active && !a.active[b]) continue;
                float* y = a.y + (long)b * a.y_stride;
                if (a.mode == MV_SWIGLU) {
#pragma unroll
                    for (int r = 0; r + 1 < R; r += 2) {
                        if (row0 + r + 1 < N) {
                            const float gv = acc[s][r], uv = acc[s][r + 1];
                            y[(row0 + r) >> 1] = gv / (1.0f + expf(-gv)) * uv;
                        }
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        if (row0 + r < N) {
                            if (a.mode == MV_ADD) y[row0 + r] += acc[s][r];
                            else y[row0 + r] = acc[s][r];
                        }
                    }
                }
            }
        }
    }
    pdl_trigger();
}

template <int NB, int R, int CH>
static void launch_mv_t(cudaStream_t st, const MvArgs& a, int num_sms, bool pdl) {
    const int nch = (a.w.cols + 511) / 512;
    const size_t smem = (size_t)NB * nch * 512 * sizeof(float);
    auto kern = k_matvec<NB, R, CH>;
    static int configured = 0;
    if (!configured) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        configured = 1;
    }
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, MV_THREADS, smem);
    if (occ < 1) occ = 1;
    const long groups = (a.w.rows + R - 1) / R;
    long blocks = (groups + MV_WARPS - 1) / MV_WARPS;
    const long cap = (long)num_sms * occ;
    if (blocks > cap) blocks = cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks, (unsigned)((a.nb + NB - 1) / NB), 1);
    cfg.blockDim = dim3(MV_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, a);
}

void launch_matvec(cudaStream_t st, const MvArgs& a, int num_sms, bool pdl) {
    // slots per pass: 1, 2, 4 or 8 (more slots → more passes over the weights, one per blockIdx.y)
    const int nb = a.nb;
    if (nb <= 1) launch_mv_t<1, 2, 4>(st, a, num_sms, pdl);
    else if (nb <= 2) launch_mv_t<2, 2, 2>(st, a, num_sms, pdl);
    else if (nb <= 4) launch_mv_t<4, 2, 2>(st, a, num_sms, pdl);
    else launch_mv_t<8, 2, 1>(st, a, num_sms, pdl);
}

// =====================================================================================================================
// the token choice: windowed repetition penalty (distinct tokens of the window), frequency penalty, first maximum
// =====================================================================================================================

constexpr int PEN_CAP = 64;  // window tokens kept per CTA and slot (more → the CTA scans the window per row)

struct PenList {
    int n[8];
    int t[8][PEN_CAP];
};

// the window tokens of slot s that fall in [lo, hi): hist[len - min(len, window), len)
__device__ void pen_prefilter(PenList& pl, int nb, int slot0, const LmArgs& a, int lo, int hi) {
    if (threadIdx.x < 8) pl.n[threadIdx.x] = 0;
    __syncthreads();
    if (a.sample && a.rp != 1.0f) {
        for (int s = 0; s < nb; s++) {
            const int b = slot0 + s;
            const int len = a.len[b];
            const int start = len - min(len, a.window);
            const int32_t* h = a.hist + (long)b * a.hist_cap;
            for (int j = start + threadIdx.x; j < len; j += blockDim.x) {
                const int t = h[j];
                if (t >= lo && t < hi) {
                    const int k = atomicAdd(&pl.n[s], 1);
                    if (k < PEN_CAP) pl.t[s][k] = t;
                }
            }
        }
    }
    __syncthreads();
}

// the choice's value of logit v of token t in slot s (choose(): rp on window members, then − fp * count)
__device__ __forceinline__ float pen_apply(const PenList& pl, int s, int b, int t, float v, const LmArgs& a,
                                           int n_vocab) {
    if (a.rp != 1.0f) {
        const int n = pl.n[s];
        bool member = false;
        if (n <= PEN_CAP) {
            for (int k = 0; k < n; k++) member |= (pl.t[s][k] == t);
        } else {
            const int len = a.len[b];
            const int32_t* h = a.hist + (long)b * a.hist_cap;
            for (int j = len - min(len, a.window); j < len && !member; j++) member = (h[j] == t);
        }
        if (member) v = v < 0.0f ? __fmul_rn(v, a.rp) : __fdiv_rn(v, a.rp);
    }
    if (a.use_fp) {
        const long k = (long)b * (long)n_vocab + t;
        if (a.counts[k] != 0u) v = __fsub_rn(v, a.fpen[k]);
    }
    return v;
}

// the CTA's best per slot → part; the last CTA of the grid row reduces all parts and records the choice
__device__ void choice_finish(const float* bv_sm, const uint32_t* bi_sm, int nb, int slot0, const LmArgs& a,
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

// LM head: contiguous row ranges per CTA (so the window prefilter is per CTA), R = 2 rows per warp
template <int NB>
__global__ void __launch_bounds__(MV_THREADS) k_lm_head(LmArgs a, int rows_per_cta) {
    extern __shared__ float4 xs4[];
    __shared__ float red[MV_WARPS];
    __shared__ PenList pl;
    __shared__ float bv_w[MV_WARPS][NB];
    __shared__ uint32_t bi_w[MV_WARPS][NB];
    __shared__ float bv_sm[NB];
    __shared__ uint32_t bi_sm[NB];
    constexpr int R = 2, CH = 2;
    float* xsf = reinterpret_cast<float*>(xs4);
    const int K = a.w.cols, N = a.w.rows;
    const int nch = (K + 511) >> 9;
    const int slot0 = blockIdx.y * NB;
    const int nb = min(NB, a.nb - slot0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lo = blockIdx.x * rows_per_cta, hi = min(N, lo + rows_per_cta);

    pdl_wait();
    stage_x<NB>(xsf, nch, K, nb, slot0, a.x, a.x_stride, a.nw, a.eps, nullptr, a.w, nullptr, false, red);
    pen_prefilter(pl, nb, slot0, a, lo, hi);  // (its barriers also publish the staged x)

    float bv[NB];
    uint32_t bi[NB];
#pragma unroll
    for (int s = 0; s < NB; s++) {
        bv[s] = -INFINITY;
        bi[s] = NO_INDEX;
    }
    const int kb = K >> 5;
    for (int row0 = lo + warp * R; row0 < hi; row0 += MV_WARPS * R) {
        float acc[NB][R];
#pragma unroll
        for (int s = 0; s < NB; s++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[s][r] = 0.0f;
        for (int i0 = 0; i0 < nch; i0 += CH) {
            uint4 wq[CH][R];
            float wd[CH][R];
#pragma unroll
            for (int ci = 0; ci < CH; ci++) {
                const int col = (i0 + ci) * 512 + lane * 16;
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int row = row0 + r;
                    if (i0 + ci < nch && row < hi && col < K) {
                        wq[ci][r] = ld_stream(a.w.q + (long)row * K + col);
                        wd[ci][r] = __half2float(a.w.d[(long)row * kb + (col >> 5)]);
                    } else {
                        wq[ci][r] = make_uint4(0, 0, 0, 0);
                        wd[ci][r] = 0.0f;
                    }
                }
            }
#pragma unroll
            for (int ci = 0; ci < CH; ci++) {
                if (i0 + ci >= nch) break;
#pragma unroll
                for (int r = 0; r < R; r++) {
                    float wf[16];
                    unpack16(wq[ci][r], wf);
#pragma unroll
                    for (int s = 0; s < NB; s++)
                        if (s < nb) acc[s][r] = fmaf(dot16(wf, xs4, (s * nch + i0 + ci) * 128, lane), wd[ci][r], acc[s][r]);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < NB; s++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[s][r] = warp_sum(acc[s][r]);
        // lane (s * R + r) takes logit (s, row0 + r)
#pragma unroll
        for (int s = 0; s < NB; s++) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = row0 + r;
                if (lane == s * R + r && s < nb && row < hi) {
                    const int b = slot0 + s;
                    float v = acc[s][r];
                    if (a.logits && (!a.active || a.active[b])) a.logits[(long)b * N + row] = v;
                    if (a.sample) {
                        v = pen_apply(pl, s, b, row, v, a, N);
                        if (row == 0) reinterpret_cast<int*>(a.part + (long)a.nb * gridDim.x * 2)[b] = (v != v);
                        if (better(v, (uint32_t)row, bv[s], bi[s])) {
                            bv[s] = v;
                            bi[s] = (uint32_t)row;
                        }
                    }
                }
            }
        }
    }
    pdl_trigger();
    if (!a.sample) return;
    // CTA reduce per slot: lanes holding slot s are s*R .. s*R+R-1; a warp argmax over all lanes per slot
#pragma unroll
    for (int s = 0; s < NB; s++) {
        float v = (lane >= s * R && lane < s * R + R) ? bv[s] : -INFINITY;
        uint32_t i = (lane >= s * R && lane < s * R + R) ? bi[s] : NO_INDEX;
        warp_argmax(v, i);
        if (lane == 0) {
            bv_w[warp][s] = v;
            bi_w[warp][s] = i;
        }
    }
    __syncthreads();
    if (threadIdx.x < NB) {
        float v = -INFINITY;
        uint32_t i = NO_INDEX;
        for (int w = 0; w < MV_WARPS; w++)
            if (better(bv_w[w][threadIdx.x], bi_w[w][threadIdx.x], v, i)) {
                v = bv_w[w][threadIdx.x];
                i = bi_w[w][threadIdx.x];
            }
        bv_sm[threadIdx.x] = v;
        bi_sm[threadIdx.x] = i;
    }
    __syncthreads();
    choice_finish(bv_sm, bi_sm, nb, slot0, a, N);
}

int lm_head_grid(int num_sms) { return num_sms * 4; }

template <int NB>
static void launch_lm_t(cudaStream_t st, const LmArgs& a, int num_sms, bool pdl) {
    const int nch = (a.w.cols + 511) / 512;
    const size_t smem = (size_t)NB * nch * 512 * sizeof(float);
    auto kern = k_lm_head<NB>;
    static int configured = 0;
    if (!configured) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        configured = 1;
    }
    const int grid = lm_head_grid(num_sms);
    int rpc = (a.w.rows + grid - 1) / grid;
    rpc = (rpc + 2 * MV_WARPS - 1) / (2 * MV_WARPS) * (2 * MV_WARPS);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, (unsigned)((a.nb + NB - 1) / NB), 1);
    cfg.blockDim = dim3(MV_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, a, rpc);
}

void launch_lm_head(cudaStream_t st, const LmArgs& a, int num_sms, bool pdl) {
    if (a.nb <= 1) launch_lm_t<1>(st, a, num_sms, pdl);
    else if (a.nb <= 2) launch_lm_t<2>(st, a, num_sms, pdl);
    else if (a.nb <= 4) launch_lm_t<4>(st, a, num_sms, pdl);
    else launch_lm_t<8>(st, a, num_sms, pdl);
}

// ---- the choice alone, over logits in memory ------------------------------------------------------------------------
__global__ void __launch_bounds__(MV_THREADS) k_sample(const float* __restrict__ logits, int stride, int n_vocab,
                                                         LmArgs a, int per_cta, int slot_base) {
    __shared__ PenList pl;
    __shared__ float bv_w[MV_WARPS];
    __shared__ uint32_t bi_w[MV_WARPS];
    __shared__ float bv_sm[1];
    __shared__ uint32_t bi_sm[1];
    const int b = slot_base + blockIdx.y;  // one slot per grid row
    const int lo = blockIdx.x * per_cta, hi = min(n_vocab, lo + per_cta);
    pdl_wait();
    pen_prefilter(pl, 1, b, a, lo, hi);
    float bv = -INFINITY;
    uint32_t bi = NO_INDEX;
    const float* l = logits + (long)b * stride;
    for (int t = lo + threadIdx.x; t < hi; t += blockDim.x) {
        const float v = pen_apply(pl, 0, b, t, l[t], a, n_vocab);
        if (t == 0) reinterpret_cast<int*>(a.part + (long)a.nb * gridDim.x * 2)[b] = (v != v);
        if (better(v, (uint32_t)t, bv, bi)) {
            bv = v;
            bi = (uint32_t)t;
        }
    }
    warp_argmax(bv, bi);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        bv_w[warp] = bv;
        bi_w[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = -INFINITY;
        uint32_t i = NO_INDEX;
        for (int w = 0; w < MV_WARPS; w++)
            if (better(bv_w[w], bi_w[w], v, i)) {
                v = bv_w[w];
                i = bi_w[w];
            }
        bv_sm[0] = v;
        bi_sm[0] = i;
    }
    __syncthreads();
    choice_finish(bv_sm, bi_sm, 1, b, a, n_vocab);
}

int sample_grid(int num_sms) { return num_sms; }

// the penalty alone, in place (choose_pen.wgsl's job): the same prefilter + pen_apply the fused choice uses
__global__ void __launch_bounds__(MV_THREADS) k_penalize(float* __restrict__ logits, int n_vocab, LmArgs a, int per_cta) {
    __shared__ PenList pl;
    const int lo = blockIdx.x * per_cta, hi = min(n_vocab, lo + per_cta);
    pen_prefilter(pl, 1, 0, a, lo, hi);
    for (int t = lo + threadIdx.x; t < hi; t += blockDim.x) logits[t] = pen_apply(pl, 0, 0, t, logits[t], a, n_vocab);
}

void launch_penalize(cudaStream_t st, float* logits, int n_vocab, const LmArgs& a, int num_sms) {
    const int grid = sample_grid(num_sms);
    const int per = (n_vocab + grid - 1) / grid;
    k_penalize<<<grid, MV_THREADS, 0, st>>>(logits, n_vocab, a, per);
}

void launch_sample(cudaStream_t st, const float* logits, int logits_stride, int n_vocab, const LmArgs& a,
                   int num_sms, int slot_base, int n_slots) {
    const int grid = sample_grid(num_sms);
    const int per = (n_vocab + grid - 1) / grid;
    k_sample<<<dim3(grid, n_slots, 1), MV_THREADS, 0, st>>>(logits, logits_stride, n_vocab, a, per, slot_base);
}

}  // namespace ocr

// k_ffn.cu — the decode step's feed-forward block for one slot in one kernel: the reference's dmv_ffn.wgsl
// (ffn_norm, gate|up, SwiGLU) and dmv.wgsl (down + residual), text.rs:4-10's layer order.
//
// Grid (FFN_CL, FFN_NCLU) in clusters of FFN_CL CTAs. Cluster c owns the slice h[c·HC, (c+1)·HC) of the n_ff hidden
// values (HC = n_ff / FFN_NCLU), CTA r of it HR = HC / FFN_CL of them: 2·HR consecutive rows of the interleaved
// gate|up matrix, and rows [r·dim/FFN_CL, …) of W_down's column slice c. Both are constant, so both bulk copies are
// issued before the dependency wait. After it: the residual x plus the attention's per-head o-projection partials
// (summed in order; the grid's first CTA writes the sum back as the new residual), RMS-normalised — the shared
// staging of stage.cuh — then one warp per gate/up row pair and SwiGLU; each of the HR values is pushed straight
// from registers into every CTA of the cluster (st.async into the peers' shared memory, counted on their mbarrier),
// so each CTA holds the cluster's HC values once its barrier completes — no cluster barrier on that path — and
// multiplies them by its W_down rows into the cluster's partial product of the down projection, dpart[c]. The next
// kernel adds x + dpart[0] + … in order. mbarrier waits are bounded (error flag, work skipped, every barrier still
// met).
#include <cooperative_groups.h>

#include <algorithm>

#include "stage.cuh"

namespace cg = cooperative_groups;

namespace ocr {

constexpr int FFN_THREADS = 256;
constexpr int FFN_NW = FFN_THREADS / 32;

// shared layout (bytes): gate|up rows, W_down rows, x (lane-blocked), the cluster's h (lane-blocked)
struct FfnSmem {
    int gu, wd, xs, hall, total;
};
__host__ __device__ inline FfnSmem ffn_layout(int dim, int n_ff) {
    const int HC = n_ff / FFN_NCLU, HR = HC / FFN_CL;
    FfnSmem m;
    m.gu = 0;
    m.wd = m.gu + 2 * HR * q8_stride(dim);
    m.xs = m.wd + (dim / FFN_CL) * q8_stride(HC);
    m.hall = m.xs + ((dim + 511) / 512) * 512 * 4;
    m.total = m.hall + ((HC + 511) / 512) * 512 * 4;
    return m;
}

// DIM_T / NFF_T: the model's dim and n_ff fixed at compile time (0: read from the arguments) — with the shape known
// the loops over chunks, row pairs and W_down pieces are straight-line code
template <int DIM_T, int NFF_T, int NKV_T>
__global__ void __launch_bounds__(FFN_THREADS, 2) k_ffn(FfnArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t bar_gu, bar_wd, bar_h;
    __shared__ float red[FFN_NW];
    const int r = blockIdx.x, c = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const unsigned long long t_start = a.tl ? gtimer() : 0ull;
    const int dim = DIM_T ? DIM_T : a.in.w.cols, n_ff = NFF_T ? NFF_T : a.n_ff;
    const int HC = n_ff / FFN_NCLU, HR = HC / FFN_CL, drows = dim / FFN_CL;
    const int gstride = q8_stride(dim), dstride = q8_stride(HC);
    const FfnSmem L = ffn_layout(dim, n_ff);
    uint8_t* gsm = sm + L.gu;
    uint8_t* dsm = sm + L.wd;
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    float* hall = reinterpret_cast<float*>(sm + L.hall);
    const int nchh = (HC + 511) / 512;
    if (t == 0) {
        mbar_init(&bar_gu, 1);
        mbar_init(&bar_wd, 1);
        mbar_init(&bar_h, 1);
        mbar_fence_init();
        mbar_expect_tx(&bar_h, (uint32_t)HC * 4);  // the cluster's h values, pushed by the CTAs that own them
        const uint64_t pol = l2_evict_first();
        const uint32_t gbytes = (uint32_t)(2 * HR * gstride), dbytes = (uint32_t)(drows * dstride);
        mbar_expect_tx(&bar_gu, gbytes);
        bulk_g2s_stream(gsm, a.gu.w + (size_t)2 * (c * HC + r * HR) * gstride, gbytes, &bar_gu, pol);
        mbar_expect_tx(&bar_wd, dbytes);
        bulk_g2s_stream(dsm, a.wd + ((size_t)c * dim + r * drows) * dstride, dbytes, &bar_wd, pol);
        pdl_trigger();
        l2_next(a.next, c * FFN_CL + r, FFN_NCLU * FFN_CL);
    }
    // hall's pad columns past HC are this CTA's own zeros; every barrier initialised before any CTA pushes
    for (int q = HC + 4 * t; q < nchh * 512; q += 4 * FFN_THREADS)
        *reinterpret_cast<float4*>(&hall[xs_index(0, nchh, q)]) = make_float4(0.f, 0.f, 0.f, 0.f);
    cluster_arrive_relaxed();
    float4 wn0 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.in.nw && dim <= 4 * FFN_THREADS && t < (dim >> 2)) wn0 = reinterpret_cast<const float4*>(a.in.nw)[t];
    pdl_wait();
    const unsigned long long t_dep = a.tl ? gtimer() : 0ull;

    const int nch = (dim + 511) / 512;
    stage_x<DIM_T, NKV_T>(xs, nch, 1, 0, a.in, red, FFN_THREADS, wn0, r == 0 && c == 0);
    __syncthreads();

    // gate|up: one warp per row pair, 16 columns per lane per 512-column chunk
    const bool got_gu = __all_sync(FULL, mbar_wait(&bar_gu, 0, a.err));
    cluster_wait();  // (the peers' barriers are ready)
    const uint64_t* xsp = reinterpret_cast<const uint64_t*>(xs);
    // up to PB pairs per warp at once (each chunk's x loaded once for all of them): every dot first, then the
    // reductions interleaved
    // (a compiled shape whose HR is a multiple of the warps: exactly PB pairs per warp, no bounds to test)
    constexpr int HR_T = NFF_T / FFN_NCLU / FFN_CL;
    constexpr bool EXACT = NFF_T != 0 && HR_T % FFN_NW == 0 && HR_T / FFN_NW <= 4;
    constexpr int PB = EXACT ? HR_T / FFN_NW : 4;
    for (int p0 = warp; p0 < (EXACT ? warp + 1 : HR); p0 += FFN_NW * PB) {  // (EXACT: one pass)
        float g[PB], u[PB];
#pragma unroll
        for (int k = 0; k < PB; k++) g[k] = u[k] = 0.0f;
        if (got_gu)
            for (int i = 0; i < nch; i++) {
                const int col = i * 512 + lane * 16;
                if (col >= dim) continue;
                uint64_t xp[8];
                const int base = (i * 128 + lane) * 2;
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    xp[2 * jj] = xsp[base + jj * 64];
                    xp[2 * jj + 1] = xsp[base + jj * 64 + 1];
                }
#pragma unroll
                for (int k = 0; k < PB; k++) {
                    const int p = p0 + k * FFN_NW;
                    if (EXACT || p < HR) {
                        const uint8_t* rg = gsm + (size_t)(2 * p) * gstride;
                        const uint8_t* ru = rg + gstride;
                        const float dg = __half2float(reinterpret_cast<const __half*>(rg + dim)[col >> 5]);
                        const float du = __half2float(reinterpret_cast<const __half*>(ru + dim)[col >> 5]);
                        g[k] = fmaf(dot16x2(*reinterpret_cast<const uint4*>(rg + col), xp), dg, g[k]);
                        u[k] = fmaf(dot16x2(*reinterpret_cast<const uint4*>(ru + col), xp), du, u[k]);
                    }
                }
            }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
            for (int k = 0; k < PB; k++) {
                g[k] += __shfl_xor_sync(FULL, g[k], m);
                u[k] += __shfl_xor_sync(FULL, u[k], m);
            }
        // every lane holds the sums: lane k finishes pair k (the SwiGLUs side by side), then pushes go out 8 lanes
        // per value: value k = lane / 8 to ranks lane % 8, lane % 8 + 8 (its place in every CTA's lane-blocked h)
        float gk = g[0], uk = u[0];
#pragma unroll
        for (int k = 1; k < PB; k++)
            if (lane == k) {
                gk = g[k];
                uk = u[k];
            }
        const float h = gk / (1.0f + expf(-gk)) * uk;
        const int k = lane >> 3, p = p0 + k * FFN_NW;
        const float hv = __shfl_sync(FULL, h, k);
        if (k < PB && p < HR) {
            float* dst = &hall[xs_index(0, nchh, r * HR + p)];
            for (int rr = lane & 7; rr < FFN_CL; rr += 8) st_async(cluster_addr(dst, rr), hv, cluster_addr(&bar_h, rr));
        }
    }
    cluster_arrive();  // (the final wait keeps every CTA until its peers are done with it)
    // the cluster's h slice, pushed into every CTA (lane-blocked for the down rows' dot)
    const bool got_h = __all_sync(FULL, mbar_wait_cluster(&bar_h, 0, a.err));

    // down: this CTA's rows of the slice, 8 lanes per row, 4 rows per warp
    const bool got_wd = __all_sync(FULL, mbar_wait(&bar_wd, 0, a.err));
    const uint64_t* hp = reinterpret_cast<const uint64_t*>(hall);
    float* op = a.dpart + (size_t)c * dim + r * drows;
    const int l8 = lane & 7;
    // two row groups per warp at once (rows base + lane/8 and base + 32 + lane/8)
    // (a compiled shape with exactly 8 W_down rows per warp: every row in range)
    constexpr bool DEX = NFF_T != 0 && DIM_T / FFN_CL == FFN_NW * 8;
    for (int base = warp * 4; base < (DEX ? warp * 4 + 1 : drows); base += FFN_NW * 8) {  // (DEX: one pass)
        float acc[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int rr = base + k * FFN_NW * 4 + (lane >> 3);
            constexpr int HC_T = NFF_T / FFN_NCLU;
            if constexpr (DEX && HC_T % 128 == 0)
                acc[k] = (got_wd && got_h) ? row_dot8c<HC_T / 128>(dsm + (size_t)rr * dstride, hp, l8) : 0.0f;
            else
                acc[k] = (got_wd && got_h && rr < drows) ? row_dot8(dsm + (size_t)rr * dstride, HC, hp, l8) : 0.0f;
        }
#pragma unroll
        for (int m = 4; m >= 1; m >>= 1)
#pragma unroll
            for (int k = 0; k < 2; k++) acc[k] += __shfl_xor_sync(FULL, acc[k], m);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int rr = base + k * FFN_NW * 4 + (lane >> 3);
            if (l8 == 0 && (DEX || rr < drows)) op[rr] = acc[k];
        }
    }
    cluster_wait();
    if (t == 0) tl_record(a.tl, t_start, t_dep);
}

int ffn_smem(int dim, int n_ff) {
    if (n_ff % (FFN_NCLU * FFN_CL * 4) || dim % (FFN_CL * 4) || dim % 32 || (n_ff / FFN_NCLU) % 32) return 0;
    const int total = ffn_layout(dim, n_ff).total;
    return total <= 100 * 1024 ? total : 0;  // two CTAs per SM
}

static void ffn_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, cudaStream_t st, int smem) {
    cfg = {};
    cfg.gridDim = dim3(FFN_CL, FFN_NCLU, 1);
    cfg.blockDim = dim3(FFN_THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = FFN_CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
}

// the instance for a shape: Qwen3-0.6B's (dim 1024, n_ff 3072, 8 kv heads' o-partials) compiled for it, any other
// shape generic
using FfnKernel = void (*)(FfnArgs);
static FfnKernel ffn_kernel(int dim, int n_ff, int n_add) {
    static PerDeviceOnce once;  // the attributes live in each device's context
    once([] {
        for (FfnKernel k : {k_ffn<1024, 3072, 8>, k_ffn<0, 0, 0>}) {
            cudaFuncAttributes fa;
            cudaFuncGetAttributes(&fa, k);
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - (int)fa.sharedSizeBytes);
            cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        }
    });
    return dim == 1024 && n_ff == 3072 && n_add == 8 ? k_ffn<1024, 3072, 8> : k_ffn<0, 0, 0>;
}

bool ffn_usable(int dim, int n_ff) {
    const int smem = ffn_smem(dim, n_ff);
    if (!smem) return false;
    // asked once per (device, shared memory size), under a lock
    static std::mutex mu;
    static int dev_k[16], keys[16], vals[16], n_keys = 0;
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_keys; i++)
        if (dev_k[i] == dev && keys[i] == smem) return vals[i] != 0;
    const FfnKernel kern = ffn_kernel(dim, n_ff, 8);  // (either instance: the same resources)
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    ffn_config(cfg, attr, nullptr, smem);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    if (n_keys < 16) {
        dev_k[n_keys] = dev;
        keys[n_keys] = smem;
        vals[n_keys++] = n >= FFN_NCLU;  // every cluster resident at once
    }
    return n >= FFN_NCLU;
}

void launch_ffn(cudaStream_t st, const FfnArgs& a, bool pdl) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    ffn_config(cfg, attr, st, ffn_smem(a.in.w.cols, a.n_ff));
    cfg.numAttrs = pdl ? 2 : 1;
    cudaLaunchKernelEx(&cfg, ffn_kernel(a.in.w.cols, a.n_ff, a.in.n_add), a);
}

}  // namespace ocr

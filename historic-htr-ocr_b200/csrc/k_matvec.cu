// k_matvec.cu — q8_0 dequant-matvec for decode (the reference's dmv / dmv_norm / dmv_qkv / dmv_ffn / matvec_q8_0,
// shaders/*.wgsl) and the LM head fused with the greedy token choice (choose_pen / choose_max / choose_pick).
//
// One kernel, streamed through the copy engine. A CTA owns a contiguous range of rows — one contiguous byte range in
// the row layout (kernels.cuh) — cut into stages of SR = W x R rows. Warp W (the producer; one lane) moves stage after
// stage with cp.async.bulk into a ring of NS shared-memory slots, each slot's arrival counted by an mbarrier
// (complete_tx); the first NS stages are issued BEFORE griddepcontrol.wait, since weights never depend on the previous
// kernel: their DRAM latency overlaps the previous kernel's tail. Warps 0..W-1 (consumers) wait for the previous
// kernel, stage the activations (NB slots; RMSNorm x norm weight folded in; layer 0 gathers the token's embedding row)
// in shared memory "lane-blocked" — float4 ((s * nch + i) * 4 + j4) * 32 + l holds x[s][512 i + 16 l + 4 j4 … +4] —
// then, per stage, each warp takes R rows: lane l reads the 16 quants at columns 512 i + 16 l (one conflict-free
// 16-B shared load), their block scale, dequantizes by byte-permute into 2^23's mantissa (exact), and accumulates
// scale * dot16 per slot. A consumed slot is released with an mbarrier arrive (count W). Warp butterfly sums, then the
// epilogue: store, residual add, silu(gate) * up over interleaved gate/up rows, or the LM head's choice.
// Every wait is bounded (mbar_wait → DEV_TIMEOUT); no spin on another CTA.
#include "choice.cuh"
#include "kernels.cuh"
#include "qdot.cuh"
#include "stage.cuh"

namespace ocr {

// ---------------------------------------------------------------------------------------------------------------------
// the streamed matvec
// ---------------------------------------------------------------------------------------------------------------------
constexpr int MAX_NS = 16;
constexpr int LM_NS = 3;  // the compiled 1024-wide LM head's ring: three 64-row stages (68 KB each)
constexpr int SM_HEAD = 256;  // mbarriers full[MAX_NS], empty[MAX_NS]

// two CTAs per SM for the small matrices of one or two slots (the grid is sized for it; at most 112 registers);
// wider slot batches keep their accumulators in registers at one CTA per SM. KT: the row length fixed at compile
// time (0: a.w.cols) — the LM head of a 1024-wide model runs its chunk loop and bounds as straight-line code.
template <int NB, int W, int R, int KT = 0>
__global__ void __launch_bounds__((W + 1) * 32, (W == 8 && NB <= 2) ? 2 : 1) k_mv(MvArgs a, int rpc, int ns_arg) {
    // (the compiled LM head runs a ring of LM_NS stages: its slot and phase arithmetic by constants)
    const int ns = KT ? LM_NS : ns_arg;
    extern __shared__ __align__(128) uint8_t sm[];
    const unsigned long long t_start = a.tl ? gtimer() : 0ull;
    unsigned long long t_dep = 0ull;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + MAX_NS;
    constexpr int SR = W * R;
    constexpr int NC = W * 32;  // consumer threads
    __shared__ float red[W];
    __shared__ PenList pl;
    __shared__ float bv_w[W][NB];
    __shared__ uint32_t bi_w[W][NB];
    __shared__ float bv_sm[NB];
    __shared__ uint32_t bi_sm[NB];

    const int K = KT ? KT : a.w.cols, N = a.w.rows, stride = KT ? q8_stride(KT) : a.w.stride;
    const int nch = (K + 511) >> 9;
    float* xsf = reinterpret_cast<float*>(sm + SM_HEAD);
    uint8_t* ring = sm + SM_HEAD + (size_t)NB * nch * 512 * sizeof(float);
    const size_t stage_bytes = (size_t)SR * stride;
    const int lo = blockIdx.x * rpc, hi = min(N, lo + rpc);
    const int n_stage = (hi - lo + SR - 1) / SR;
    const int slot0 = blockIdx.y * NB, nb = min(NB, a.nb - slot0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool lmhead = a.mode == MV_LMHEAD;

    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], W);
        }
        mbar_fence_init();
    }
    __syncthreads();

    float bvl = -INFINITY;  // this lane's best (LM head: the lane's slot lane / R)
    uint32_t bil = NO_INDEX;

    if (warp == W) {
        // ---- producer: weights never depend on the previous kernel, so no griddepcontrol.wait here. The warp
        // waits for a free slot, lane 0 arms its barrier, every lane issues its 4 KB pieces of the stage. ----
        const uint64_t pol = l2_evict_first();
        for (int t = 0; t < n_stage; t++) {
            const int slot = t % ns;
            if (t >= ns && !__all_sync(FULL, mbar_wait(&empty[slot], ((t / ns) - 1) & 1, a.err))) break;
            const int r0 = lo + t * SR;
            const uint32_t bytes = (uint32_t)(min(SR, hi - r0) * stride);
            if (lane == 0) mbar_expect_tx(&full[slot], bytes);
            __syncwarp();
            bulk_g2s_lanes(ring + slot * stage_bytes, a.w.w + (size_t)r0 * stride, bytes, &full[slot], pol, lane, 32);
            if (t == min(ns, n_stage) - 1 && lane == 0) {
                pdl_trigger();
                l2_next(a.next, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
            }
        }
    } else {
        // ---- consumers ----
        // Before the dependency wait: what no kernel of this step writes — the norm weights, the per-slot
        // activity, and for the LM head the window's tokens (history and length were written by the previous
        // step's choice, complete before this step's first kernel started; every later kernel launched after it).
        bool act[NB];
#pragma unroll
        for (int s = 0; s < NB; s++) act[s] = s < nb && (!a.active || a.active[slot0 + s] != 0);
        float4 wn0 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.nw && K <= 4 * NC && (int)threadIdx.x < (K >> 2)) wn0 = reinterpret_cast<const float4*>(a.nw)[threadIdx.x];
        if (lmhead) pen_prefilter(pl, nb, slot0, a.lm, lo, hi, NC);
        pdl_wait();
        if (threadIdx.x == 0 && a.tl) t_dep = gtimer();
        // for the residual add, the first stages' old values of this warp's rows are fetched now so the epilogue's
        // read-modify-write does not wait on memory
        constexpr int PF = 2;
        float yold[PF][NB][R];
        if (a.mode == MV_ADD && lane == 0) {
#pragma unroll
            for (int t = 0; t < PF; t++)
#pragma unroll
                for (int s = 0; s < NB; s++)
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        const int row = lo + t * SR + warp * R + r;
                        // (no dependence on act: all these loads go out together)
                        yold[t][s][r] = (t < n_stage && s < nb && row < hi) ? a.y[(long)(slot0 + s) * a.y_stride + row]
                                                                          : 0.0f;
                    }
        }
        // (the compiled LM head's partials, when any, are the fused FFN's FFN_NCLU)
        stage_x<KT, KT ? FFN_NCLU : 0>(xsf, nch, nb, slot0, a, red, NC, wn0, blockIdx.x == 0);
        bar_sync(1, NC);
        const uint64_t* xsp = reinterpret_cast<const uint64_t*>(xsf);  // x as f32 pairs
        // The compiled LM head (KT, one slot) takes the staged row as three int8 digits per 32-column block: with s
        // the power of two at or above max|x| / 126 over the block, x / s = d0 + d1 / 128 + d2 / 128^2 + e with
        // |d0| <= 126, |d1|, |d2| <= 64 and |e| <= 2^-15 (every step exact: power-of-two scalings and integer
        // subtractions), so a quant row's dot is three integer dots (dp4a on the raw int8 weights: no conversion)
        // combined once per 16 columns — about half the instructions of the f32 dot per quant.
        constexpr bool DIG = KT != 0 && NB == 1;
        const uint4* xdig = reinterpret_cast<const uint4*>(xsf);  // [nch][3 digits][32 lanes] x 16 int8
        const float* xsc = xsf + 3 * 4 * 32 * nch;                   // [nch][16 blocks] the block scales s
        if constexpr (DIG) {
            const int tid = threadIdx.x, i = tid >> 5, l = tid & 31;
            float v[16];
            float m = 0.0f;
            if (warp < nch) {  // (whole warps: lane pairs l, l ^ 1 hold one 32-column block)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    const float4 f = reinterpret_cast<const float4*>(xsf)[(i * 4 + jj) * 32 + l];
                    v[4 * jj] = f.x, v[4 * jj + 1] = f.y, v[4 * jj + 2] = f.z, v[4 * jj + 3] = f.w;
                }
#pragma unroll
                for (int j = 0; j < 16; j++) m = fmaxf(m, fabsf(v[j]));
                m = fmaxf(m, __shfl_xor_sync(FULL, m, 1));
            }
            bar_sync(1, NC);  // every staged value read before the region holds the digits
            if (warp < nch) {
                int e = 0;
                if (m > 0.0f) frexpf(m * (1.0f / 126.0f), &e);
                const float sc_b = m > 0.0f ? ldexpf(1.0f, e) : 1.0f, inv = m > 0.0f ? ldexpf(1.0f, -e) : 1.0f;
                uint32_t w[3][4] = {};
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float q = v[j] * inv;
                    const float d0 = rintf(q), r1 = (q - d0) * 128.0f;
                    const float d1 = rintf(r1), r2 = (r1 - d1) * 128.0f;
                    const float d2 = rintf(r2);
                    w[0][j >> 2] |= ((uint32_t)(int)d0 & 0xffu) << (8 * (j & 3));
                    w[1][j >> 2] |= ((uint32_t)(int)d1 & 0xffu) << (8 * (j & 3));
                    w[2][j >> 2] |= ((uint32_t)(int)d2 & 0xffu) << (8 * (j & 3));
                }
                uint4* xd = reinterpret_cast<uint4*>(xsf);
#pragma unroll
                for (int k = 0; k < 3; k++) xd[(i * 3 + k) * 32 + l] = make_uint4(w[k][0], w[k][1], w[k][2], w[k][3]);
                if (!(l & 1)) xsf[3 * 4 * 32 * nch + i * 16 + (l >> 1)] = sc_b;
            }
            bar_sync(1, NC);
        }
        for (int t = 0; t < n_stage; t++) {
            const int slot = t % ns;
            if (!mbar_wait(&full[slot], (t / ns) & 1, a.err)) break;
            const uint8_t* st = ring + slot * stage_bytes;
            const int r0 = lo + t * SR, nr = min(SR, hi - r0);
            float acc[NB][R];
#pragma unroll
            for (int s = 0; s < NB; s++)
#pragma unroll
                for (int r = 0; r < R; r++) acc[s][r] = 0.0f;
            if (warp * R < nr) {
                for (int i = 0; i < nch; i++) {
                    const int col = i * 512 + lane * 16;
                    uint4 wq[R];
                    float sc[R];
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        const int rr = warp * R + r;
                        if (col < K && rr < nr) {
                            const uint8_t* row = st + (size_t)rr * stride;
                            wq[r] = *reinterpret_cast<const uint4*>(row + col);
                            sc[r] = __half2float(reinterpret_cast<const __half*>(row + K)[col >> 5]);
                        } else {
                            // q = 0 (the f32 dot reads the quants biased by 128, the integer dot as they are)
                            wq[r] = DIG ? make_uint4(0u, 0u, 0u, 0u)
                                        : make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
                            sc[r] = 0.0f;
                        }
                    }
                    if constexpr (DIG) {
                        const uint4 e0 = xdig[(i * 3) * 32 + lane], e1 = xdig[(i * 3 + 1) * 32 + lane];
                        const uint4 e2 = xdig[(i * 3 + 2) * 32 + lane];
                        const float sb = xsc[i * 16 + (lane >> 1)];
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            const uint4 w = wq[r];
                            int d0 = __dp4a((int)w.x, (int)e0.x, 0), d1 = __dp4a((int)w.x, (int)e1.x, 0),
                                d2 = __dp4a((int)w.x, (int)e2.x, 0);
                            d0 = __dp4a((int)w.y, (int)e0.y, d0), d1 = __dp4a((int)w.y, (int)e1.y, d1);
                            d2 = __dp4a((int)w.y, (int)e2.y, d2);
                            d0 = __dp4a((int)w.z, (int)e0.z, d0), d1 = __dp4a((int)w.z, (int)e1.z, d1);
                            d2 = __dp4a((int)w.z, (int)e2.z, d2);
                            d0 = __dp4a((int)w.w, (int)e0.w, d0), d1 = __dp4a((int)w.w, (int)e1.w, d1);
                            d2 = __dp4a((int)w.w, (int)e2.w, d2);
                            // (|d0| < 2^18: exact in f32; the digits' weights are powers of two)
                            const float dv = fmaf((float)d2, 1.0f / 16384.0f, fmaf((float)d1, 1.0f / 128.0f, (float)d0));
                            acc[0][r] = fmaf(dv, sc[r] * sb, acc[0][r]);
                        }
                    } else {
#pragma unroll
                    for (int s = 0; s < NB; s++) {
                        if (s < nb) {
                            uint64_t xp[8];
                            const int base = ((s * nch + i) * 128 + lane) * 2;  // in f32 pairs
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                xp[2 * j] = xsp[base + j * 64];
                                xp[2 * j + 1] = xsp[base + j * 64 + 1];
                            }
#pragma unroll
                            for (int r = 0; r < R; r++) acc[s][r] = fmaf(dot16x2(wq[r], xp), sc[r], acc[s][r]);
                        }
                    }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (warp * R >= nr) continue;
#pragma unroll
            for (int s = 0; s < NB; s++)
#pragma unroll
                for (int r = 0; r < R; r++) acc[s][r] = warp_sum(acc[s][r]);
            const int row0 = r0 + warp * R;
            if (!lmhead) {
                if (lane == 0) {
#pragma unroll
                    for (int s = 0; s < NB; s++) {
                        if (s >= nb) break;
                        const int b = slot0 + s;
                        if (!act[s]) continue;
                        float* y = a.y + (long)b * a.y_stride;
                        if (a.mode == MV_SWIGLU) {
#pragma unroll
                            for (int r = 0; r + 1 < R; r += 2)
                                if (row0 + r + 1 < hi) {
                                    const float gv = acc[s][r], uv = acc[s][r + 1];
                                    y[(row0 + r) >> 1] = gv / (1.0f + expf(-gv)) * uv;
                                }
                        } else {
#pragma unroll
                            for (int r = 0; r < R; r++)
                                if (row0 + r < hi) {
                                    if (a.mode == MV_ADD) {
                                        float old;
                                        if (t < PF) {
#pragma unroll
                                            for (int tt = 0; tt < PF; tt++)
                                                if (tt == t) old = yold[tt][s][r];
                                        } else {
                                            old = y[row0 + r];
                                        }
                                        y[row0 + r] = old + acc[s][r];
                                    } else {
                                        y[row0 + r] = acc[s][r];
                                    }
                                }
                        }
                    }
                }
            } else {
                // lane s * R + r takes logit (slot s, row row0 + r): one pass of the epilogue for all of them
                const int ls = lane / R, lr = lane % R, row = row0 + lr;
                float v = 0.0f;
                bool la = false;
#pragma unroll
                for (int s = 0; s < NB; s++)
#pragma unroll
                    for (int r = 0; r < R; r++)
                        if (lane == s * R + r) {
                            v = acc[s][r];
                            la = act[s];
                        }
                if (lane < NB * R && ls < nb && row < hi) {
                    const int b = slot0 + ls;
                    if (a.y && la) a.y[(long)b * N + row] = v;
                    if (a.lm.sample) {
                        v = pen_apply(pl, ls, b, row, v, a.lm, N, lo, hi);
                        if (row == 0) reinterpret_cast<int*>(a.lm.part + (long)a.lm.nb * gridDim.x * 2)[b] = (v != v);
                        if (better(v, (uint32_t)row, bvl, bil)) {
                            bvl = v;
                            bil = (uint32_t)row;
                        }
                    }
                }
            }
        }
    }
    if (!lmhead || !a.lm.sample) {  // (uniform over the grid)
        if (threadIdx.x == 0) tl_record(a.tl, t_start, t_dep);
        return;
    }
    // ---- the LM head's choice: CTA reduce per slot, then the last CTA picks ----
    __syncthreads();
    if (warp < W) {
#pragma unroll
        for (int s = 0; s < NB; s++) {
            const bool mine = lane >= s * R && lane < s * R + R;
            float v = mine ? bvl : -INFINITY;
            uint32_t i = mine ? bil : NO_INDEX;
            warp_argmax(v, i);
            if (lane == 0) {
                bv_w[warp][s] = v;
                bi_w[warp][s] = i;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < NB) {
        float v = -INFINITY;
        uint32_t i = NO_INDEX;
        for (int w = 0; w < W; w++)
            if (better(bv_w[w][threadIdx.x], bi_w[w][threadIdx.x], v, i)) {
                v = bv_w[w][threadIdx.x];
                i = bi_w[w][threadIdx.x];
            }
        bv_sm[threadIdx.x] = v;
        bi_sm[threadIdx.x] = i;
    }
    __syncthreads();
    choice_finish(bv_sm, bi_sm, nb, slot0, a.lm, N);
    if (threadIdx.x == 0) tl_record(a.tl, t_start, t_dep);
}

// ---- launch geometry --------------------------------------------------------------------------------------------------
struct Geo {
    int W, R, rpc, grid, ns;
    size_t smem;
};

constexpr size_t SMEM_MAX = 220 * 1024;   // the streamed LM head's ring (one CTA per SM)
constexpr size_t SMEM_SMALL = 96 * 1024;  // a small matrix's ring: two CTAs (with their static memory) per SM

// streamed (> 48 MB: the LM head): one CTA per SM, 16 consumer warps x 4 rows for one slot (the activation loads
// and the per-stage waits shared by more rows; 2 for slot batches, whose accumulators need the registers), a ring
// as deep as fits. Small matrices:
// `per_sm` CTAs per SM (two when registers and shared memory allow), 8 consumer warps (x 2 rows for SwiGLU pairs,
// else 1), one or two stages each. The grid is one wave: a CTA that cannot be resident with the others would stream
// its rows after them.
static Geo geometry(const MvArgs& a, int nb_pass, int num_sms, int per_sm = 2) {
    const int N = a.w.rows, K = a.w.cols, stride = a.w.stride;
    const int nch = (K + 511) / 512;
    const size_t xs = (size_t)nb_pass * nch * 512 * 4;
    Geo g;
    const bool big = (size_t)N * stride > (size_t)48 << 20;
    const int target = big ? num_sms : per_sm * num_sms;
    if (big) {
        g.W = 16;
        g.R = nb_pass == 1 ? 4 : 2;
    } else if (a.mode == MV_SWIGLU) {
        g.W = 8;
        g.R = 2;
    } else {
        g.W = 8;
        g.R = 1;
    }
    const int SR = g.W * g.R;
    g.rpc = (N + target - 1) / target;
    g.rpc = (g.rpc + 1) / 2 * 2;  // even: interleaved gate/up pairs never straddle CTAs
    g.grid = (N + g.rpc - 1) / g.rpc;
    const int n_stage = (g.rpc + SR - 1) / SR;
    const size_t stage = (size_t)SR * stride;
    const size_t budget = (big ? SMEM_MAX : SMEM_SMALL) - SM_HEAD - xs;
    g.ns = (int)std::min<size_t>(std::min<size_t>((size_t)n_stage, MAX_NS), std::max<size_t>(1, budget / stage));
    g.smem = SM_HEAD + xs + (size_t)g.ns * stage;
    return g;
}

int lm_head_grid(int num_sms, int n_vocab, int dim) {
    MvArgs a;
    a.mode = MV_LMHEAD;
    a.w.rows = n_vocab;
    a.w.cols = dim;
    a.w.stride = q8_stride(dim);
    return geometry(a, 1, num_sms).grid;
}

template <int NB, int W, int R, int KT = 0>
static void configure_t() {
    static PerDeviceOnce once;  // the attribute lives in each device's context
    once([] {
        auto kern = k_mv<NB, W, R, KT>;
        cudaFuncAttributes fa;
        cudaFuncGetAttributes(&fa, kern);
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - (int)fa.sharedSizeBytes);
    });
}

// CTAs of this instantiation resident per SM with a small matrix's shared memory (registers decide: the build's
// count for the template), asked once per device
template <int NB, int W, int R>
static int per_sm_t() {
    configure_t<NB, W, R>();
    static PerDeviceOnce once;
    static int n_dev[MAX_DEVICES];
    const int d = current_device();
    int n = 1;
    once([&] {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_mv<NB, W, R>, (W + 1) * 32, SMEM_SMALL) !=
            cudaSuccess) {
            cudaGetLastError();
            n = 1;
        }
        n = std::max(1, std::min(2, n));
        if (d >= 0 && d < MAX_DEVICES) n_dev[d] = n;
    });
    return d >= 0 && d < MAX_DEVICES ? n_dev[d] : n;
}

template <int NB, int W, int R, int KT = 0>
static void launch_t(cudaStream_t st, const MvArgs& a, const Geo& g, bool pdl) {
    auto kern = k_mv<NB, W, R, KT>;
    configure_t<NB, W, R, KT>();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)g.grid, (unsigned)((a.nb + NB - 1) / NB), 1);
    cfg.blockDim = dim3((W + 1) * 32, 1, 1);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, a, g.rpc, g.ns);
}

template <int NB>
static void launch_nb(cudaStream_t st, const MvArgs& a, int num_sms, bool pdl) {
    Geo g = geometry(a, NB, num_sms);
    if (g.W == 16) {
        bool done = false;
        if constexpr (NB == 1) {
            if (a.w.cols == 1024 && (!a.xadd || a.n_add == FFN_NCLU) && g.ns == LM_NS) {
                launch_t<NB, 16, 4, 1024>(st, a, g, pdl);
                done = true;
            }
        }
        if (!done) launch_t<NB, 16, NB == 1 ? 4 : 2>(st, a, g, pdl);
    } else if (g.R == 2) {
        if (per_sm_t<NB, 8, 2>() < 2) g = geometry(a, NB, num_sms, 1);
        launch_t<NB, 8, 2>(st, a, g, pdl);
    } else {
        if (per_sm_t<NB, 8, 1>() < 2) g = geometry(a, NB, num_sms, 1);
        launch_t<NB, 8, 1>(st, a, g, pdl);
    }
}

void launch_matvec(cudaStream_t st, const MvArgs& a, int num_sms, bool pdl) {
    // slots per pass: 1, 2, 4 or 8 (more slots → one pass over the weights per blockIdx.y)
    if (a.nb <= 1) launch_nb<1>(st, a, num_sms, pdl);
    else if (a.nb <= 2) launch_nb<2>(st, a, num_sms, pdl);
    else if (a.nb <= 4) launch_nb<4>(st, a, num_sms, pdl);
    else launch_nb<8>(st, a, num_sms, pdl);
}

// ---------------------------------------------------------------------------------------------------------------------
// the choice alone, over logits in memory; the penalty alone
// ---------------------------------------------------------------------------------------------------------------------
constexpr int SAMPLE_THREADS = 256;

__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample(const float* __restrict__ logits, int stride, int n_vocab,
                                                             LmArgs a, int per_cta, int slot_base) {
    __shared__ PenList pl;
    __shared__ float bv_w[SAMPLE_THREADS / 32];
    __shared__ uint32_t bi_w[SAMPLE_THREADS / 32];
    __shared__ float bv_sm[1];
    __shared__ uint32_t bi_sm[1];
    const int b = slot_base + blockIdx.y;  // one slot per grid row
    const int lo = blockIdx.x * per_cta, hi = min(n_vocab, lo + per_cta);
    pdl_wait();
    pen_prefilter(pl, 1, b, a, lo, hi, SAMPLE_THREADS);
    float bv = -INFINITY;
    uint32_t bi = NO_INDEX;
    const float* l = logits + (long)b * stride;
    for (int t = lo + threadIdx.x; t < hi; t += blockDim.x) {
        const float v = pen_apply(pl, 0, b, t, l[t], a, n_vocab, lo, hi);
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
        for (int w = 0; w < SAMPLE_THREADS / 32; w++)
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

void launch_sample(cudaStream_t st, const float* logits, int logits_stride, int n_vocab, const LmArgs& a,
                   int num_sms, int slot_base, int n_slots) {
    const int grid = sample_grid(num_sms);
    const int per = (n_vocab + grid - 1) / grid;
    k_sample<<<dim3(grid, n_slots, 1), SAMPLE_THREADS, 0, st>>>(logits, logits_stride, n_vocab, a, per, slot_base);
}

__global__ void __launch_bounds__(SAMPLE_THREADS) k_penalize(float* __restrict__ logits, int n_vocab, LmArgs a,
                                                               int per_cta) {
    __shared__ PenList pl;
    const int lo = blockIdx.x * per_cta, hi = min(n_vocab, lo + per_cta);
    pen_prefilter(pl, 1, 0, a, lo, hi, SAMPLE_THREADS);
    for (int t = lo + threadIdx.x; t < hi; t += blockDim.x)
        logits[t] = pen_apply(pl, 0, 0, t, logits[t], a, n_vocab, lo, hi);
}

void launch_penalize(cudaStream_t st, float* logits, int n_vocab, const LmArgs& a, int num_sms) {
    const int grid = sample_grid(num_sms);
    const int per = (n_vocab + grid - 1) / grid;
    k_penalize<<<grid, SAMPLE_THREADS, 0, st>>>(logits, n_vocab, a, per);
}

}  // namespace ocr

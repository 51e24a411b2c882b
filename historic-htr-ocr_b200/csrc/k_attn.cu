// k_attn.cu — decode attention of one token per slot over the f16 KV cache, GQA, split over the keys ("flash
// decoding"): the reference's qkv_post.wgsl (q/k RMSNorm → RoPE NEOX → K/V store), attn_decode.wgsl (per-range softmax
// partials m, l, o[128]) and attn_merge.wgsl (M = max m, L = Σ l e^(m−M), O = Σ o e^(m−M) / L) in one kernel.
//
// Grid (CL, n_kv, slots) in thread-block clusters of CL CTAs: one cluster per (slot, kv head), CTA rank r owning a
// contiguous key range [k0, k1) of the slot's pos + 1 keys (from the device-side position: one captured graph serves
// every step). KV layout [slot][kv head][n_ctx][128] f16: a range is one contiguous run of K and one of V, moved into
// shared memory in tiles of TILE keys by bulk-async copies on a ring of up to MAX_BUF tiles (two CTAs per SM, so
// every 16-CTA cluster of a one-token step is resident at once). The first ring's copies are issued before the kernel
// waits on its predecessor — no kernel of this step writes rows below pos; the row at pos is computed here (one warp
// per head: RMSNorm by a warp reduction, RoPE in registers), stored to the cache and to an extra shared row read in
// place of its tile row. The keys are taken in rounds of the resident tiles; each of the 8 warps owns a contiguous
// eighth of a round: scores by 8 lanes per key (16 dims each), one online-softmax update per round (running max, sum,
// output rescale) and P·V with lane = 4 dims. The block meets only when the ring wraps. The warps' states merge in
// shared memory into the CTA's (o, m, l); the cluster's CL partials merge through distributed shared memory, with no
// global round trip and no atomic.
//
// Two endings. Unfused (the op entry point): each CTA merges a 1/CL slice of the output and stores it. Fused (the
// decode step): every CTA ends with the group's whole output, which it multiplies by its dim/CL rows of W_o's slice
// for this kv head (fetched before the dependency wait) into opart[b][j] — the o-projection as n_kv per-head partial
// products, summed in a fixed order by the next kernel. For G ≤ 4 the exchange is by pushes: each CTA stores its
// merged values into the shared memory of the CTA owning their 1/CL slice (st.async, counted as complete-tx on the
// owner's mbarrier), the owner merges the slice and pushes it into every CTA; G = 8 reduce-scatters and all-gathers
// with float4 reads of the ranks' partials between cluster barriers.
//
// Fused qkv (a.wqkv set; the reference's dmv_qkv.wgsl): the cluster also computes its group's (G + 2)·128 rows of
// the [q | k | v] projection. CTA r stages the slot's residual (plus the FFN's partials, RMS-normalised by attn_norm:
// stage.cuh, as the qkv matvec would), multiplies it by its RQ = (G + 2)·128 / CL rows of W_qkv — fetched before the
// dependency wait into the V region, whose V tiles are copied once the projection is done — and pushes each value
// into every CTA of the cluster before the q/k preparation. DIM_T instances are compiled for one model dim (the
// loops over chunks and rows straight-line). mbarrier waits are bounded; a warp whose wait ran out skips its work
// (the CTA's partial is void, the error flag set) but still meets every barrier.
#include <cooperative_groups.h>

#include <algorithm>

#include "kernels.cuh"
#include "stage.cuh"

namespace cg = cooperative_groups;

namespace ocr {

constexpr int AT_THREADS = 256;
constexpr int NW = AT_THREADS / 32;  // warps per CTA
constexpr int HD = 128;              // head dim (TextConfig::from_gguf requires 128, text.rs:57-60)
constexpr int TILE = 80;             // keys per tile (K + V: 40 KB; two cover a 16-way split of 2560 keys)
constexpr int MAX_BUF = 2;           // ring depth: at most 80 KB, so two CTAs share an SM
constexpr int KPW = (MAX_BUF * TILE + NW - 1) / NW;  // keys per warp per round (one per lane)
constexpr int PW = HD + 4;  // a head's partial: o[128], m, l, two floats of pad (whole float4s)

// DIM_T: the model's dim fixed at compile time (0: read from the arguments) — the staging, the projection's chunk
// loop and the o-projection's rows become straight-line code
template <int G, int CL, int DIM_T = 0>
__global__ void __launch_bounds__(AT_THREADS, G <= 4 ? 2 : 1) k_attn_decode(AttnArgs a, int n_buf_arg, int smem) {
    // (a compiled dim's instance runs with the full ring: its slot and phase arithmetic by constants)
    const int n_buf = DIM_T ? MAX_BUF : n_buf_arg;
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t fk[MAX_BUF], fv[MAX_BUF];  // a ring slot's K rows, its V rows
    __shared__ __align__(8) uint64_t obar;  // W_o slice chunks (fused o-projection)
    __shared__ __align__(8) uint64_t qbar;  // the W_qkv rows (fused qkv projection)
    __shared__ __align__(8) uint64_t gbar;  // the group's projected values, pushed by the cluster (fused qkv)
    __shared__ __align__(8) uint64_t mbar, abar;  // fused ending by pushes: the slice's partials, the merged outputs
    __shared__ float red[NW];
    __shared__ __align__(16) float gq[G <= 4 ? (G + 2) * HD : 4];  // the group's [q heads | k | v] (fused qkv, G ≤ 4)
    __shared__ __align__(16) float qs[G][HD];
    __shared__ float scw[NW][G][KPW];  // per warp: the round's scores, then probabilities
    __shared__ float wm[NW][G], wl[NW][G];
    __shared__ __align__(16) float wo[NW][G][HD];
    // this CTA's (o[128], m, l, pad) per head, read by the cluster; in the fused ending by pushes (G ≤ 4) the same
    // storage receives the ranks' values for this CTA's slice [CL][PER], then their (m, l) [CL][2]
    constexpr int PART_F = G * PW > G * HD + 2 * CL ? G * PW : G * HD + 2 * CL;
    __shared__ __align__(16) float partbuf[PART_F];
    float(*part)[PW] = reinterpret_cast<float(*)[PW]>(partbuf);
    cg::cluster_group cluster = cg::this_cluster();
    const int b = blockIdx.z, j = blockIdx.y, sp = blockIdx.x, t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    const unsigned long long t_start = a.tl ? gtimer() : 0ull;

    // the slot's position was written by the previous step (its last kernel completed before this step began); the
    // conditions below are the same for every CTA of the cluster (same slot), so a cluster leaves together
    if (a.active && !a.active[b]) return;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.n_ctx) {
        if (sp == 0 && j == 0 && t == 0) dev_error(a.err, DEV_BAD_POS);
        return;
    }
    const int n_keys = pos + 1;
    const int per = (n_keys + CL - 1) / CL;
    const int k0 = min(n_keys, sp * per), k1 = min(n_keys, k0 + per);
    const int n_tiles = (k1 - k0 + TILE - 1) / TILE;
    const long head_base = ((long)b * a.n_kv + j) * a.n_ctx;
    __half* kb = a.kc + head_base * HD;
    __half* vb = a.vc + head_base * HD;
    // shared layout: K rows [ring + 1][HD], then the V region — V rows [ring + 1][HD], holding first the W_qkv rows
    // when the qkv projection is fused (it is at least as large as those) — then the W_o region; tile tl occupies
    // rows (tl % n_buf) * TILE …, row `ring` holds the new token's K (V), written here rather than copied
    const int ring = n_buf * TILE;
    const bool fq = G <= 4 && a.wqkv.w != nullptr;
    const int RQ = (G + 2) * HD / CL;  // the fused qkv projection: this CTA's rows of the group's [q | k | v] rows
    const int qstride = DIM_T ? q8_stride(DIM_T) : a.wqkv.stride;  // W_qkv's row stride
    const int mdim = DIM_T ? DIM_T : a.dim;                          // the o-projection's rows (the model dim)
    const int vreg = max((ring + 1) * HD * 2, fq ? RQ * qstride : 0);
    __half* Ks = reinterpret_cast<__half*>(sm);
    __half* Vs = Ks + (size_t)(ring + 1) * HD;

    // the fused o-projection's W_o rows [row0, row0 + rpc) of slice j, in chunks of `ro` rows in the region after the
    // KV ring (`smem` bytes of dynamic shared memory in all)
    const int NCOL = G * HD, ostride = q8_stride(NCOL);
    const int rpc = a.wo ? mdim / CL : 0, row0 = sp * rpc;
    const bool pushm = G <= 4 && rpc > 0;  // the fused ending's exchanges as pushes
    const int kv_bytes = (ring + 1) * HD * 2 + vreg;
    uint8_t* wsm = sm + kv_bytes;
    // (a compiled dim whose rows make exactly 8 per warp: one chunk, every row in range — its W_o region holds them)
    constexpr bool OEX = DIM_T != 0 && DIM_T / CL == NW * 8;
    const int ro = OEX ? rpc : rpc ? max(1, min(rpc, (smem - kv_bytes) / ostride)) : 1;
    auto issue_o = [&](int c0) {
        const uint32_t bytes = (uint32_t)(min(ro, rpc - c0) * ostride);
        mbar_expect_tx(&obar, bytes);
        bulk_g2s(wsm, a.wo + ((size_t)j * mdim + row0 + c0) * ostride, bytes, &obar);
    };
    // rows [ts, min(te, pos)) of tile tl (the row at pos is not in the cache yet): its K rows and/or its V rows
    auto issue = [&](int tl, bool k, bool v) {
        const int slot = tl % n_buf, ts = k0 + tl * TILE, ce = min(min(k1, ts + TILE), pos);
        const uint64_t pol = l2_evict_first();
        const uint32_t bytes = ce > ts ? (uint32_t)(ce - ts) * HD * 2 : 0;
        if (k) {
            if (bytes) {
                mbar_expect_tx(&fk[slot], bytes);
                bulk_g2s_stream(Ks + (size_t)slot * TILE * HD, kb + (long)ts * HD, bytes, &fk[slot], pol);
            } else {
                mbar_arrive(&fk[slot]);  // nothing to copy: complete the phase
            }
        }
        if (v) {
            if (bytes) {
                mbar_expect_tx(&fv[slot], bytes);
                bulk_g2s_stream(Vs + (size_t)slot * TILE * HD, vb + (long)ts * HD, bytes, &fv[slot], pol);
            } else {
                mbar_arrive(&fv[slot]);
            }
        }
    };
    if (t == 0) {
        for (int i = 0; i < n_buf; i++) {
            mbar_init(&fk[i], 1);
            mbar_init(&fv[i], 1);
        }
        mbar_init(&obar, 1);
        mbar_init(&qbar, 1);
        mbar_init(&gbar, 1);
        mbar_init(&mbar, 1);
        mbar_init(&abar, 1);
        mbar_fence_init();
        if (fq) mbar_expect_tx(&gbar, (uint32_t)(G + 2) * HD * 4);
        if (pushm) {
            mbar_expect_tx(&mbar, (uint32_t)(G * HD + 2 * CL) * 4);
            mbar_expect_tx(&abar, (uint32_t)NCOL * 4);
        }
        // constant weights and the cache's rows below pos: fetched before the wait (the V rows after the fused
        // projection, whose weights borrow their region)
        for (int tl = 0; tl < min(n_buf, n_tiles); tl++) issue(tl, true, !fq);
        if (fq) {
            const int ci0 = sp * RQ;  // this CTA's first row of the group's [q heads | k | v]
            const int grow = ci0 < G * HD ? j * G * HD + ci0
                             : ci0 < (G + 1) * HD ? a.n_head * HD + j * HD + (ci0 - G * HD)
                                                  : (a.n_head + a.n_kv) * HD + j * HD + (ci0 - (G + 1) * HD);
            const uint32_t bytes = (uint32_t)(RQ * qstride);
            mbar_expect_tx(&qbar, bytes);
            bulk_g2s_stream(Vs, a.wqkv.w + (size_t)grow * qstride, bytes, &qbar, l2_evict_first());
        }
        if (rpc > 0) issue_o(0);
        pdl_trigger();
        l2_next(a.next, (b * gridDim.y + j) * CL + sp, CL * gridDim.y * gridDim.z);
    }
    // warp h prepares q head h (h < G) or the new k / v head (h = G), warps taking heads h, h + NW; lane holds dims
    // d0, d0 + 1 and their RoPE partners 64 + d0, 64 + d0 + 1. Not written by this step, so loaded before the dependency wait: the norm
    // weights and the RoPE row of pos ([64][2] cos, sin).
    constexpr int HPW = (G + 1 + NW - 1) / NW;  // heads per warp (2 for the k / v head when G = 8)
    const int d0 = lane * 2;
    float2 w_lo[HPW], w_hi[HPW];
    float4 cs = make_float4(0.f, 0.f, 0.f, 0.f);
    if (warp <= G) cs = *reinterpret_cast<const float4*>(a.rope + (long)pos * HD + 2 * d0);
#pragma unroll
    for (int u = 0; u < HPW; u++) {
        const int h = warp + u * NW;
        if (h <= G) {
            const float* wv = h < G ? a.q_norm : a.k_norm;
            w_lo[u] = *reinterpret_cast<const float2*>(wv + d0);
            w_hi[u] = *reinterpret_cast<const float2*>(wv + 64 + d0);
        }
    }
    if (fq || pushm) cluster_arrive_relaxed();  // every barrier initialised before a peer pushes (waited below)
    const int dim = DIM_T ? DIM_T : a.in.w.cols;
    float4 wn0 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (fq && a.in.nw && t < (dim >> 2)) wn0 = reinterpret_cast<const float4*>(a.in.nw)[t];
    pdl_wait();
    const unsigned long long t_dep = a.tl ? gtimer() : 0ull;

    // the fused qkv projection: the slot's residual staged (plus the FFN's partials, RMS-normalised), this CTA's RQ
    // rows (RQ / NW per warp, their dots together), each value pushed into every CTA of the cluster (st.async into
    // gq, counted on the peers' gbar), so every CTA holds the group's (G + 2)·128 values once its gbar completes
    float* qkvs = &wo[0][0][0];  // the staged row (the warps' partials come later)
    bool got_g = true;
    if (fq) {
        const int nch = (dim + 511) / 512;
        // (the partials it adds, when any, are the fused FFN's FFN_NCLU)
        stage_x<DIM_T, DIM_T ? FFN_NCLU : 0>(qkvs, nch, 1, b, a.in, red, AT_THREADS, wn0, sp == 0 && j == 0);
        __syncthreads();
        constexpr int RPW = 8;  // at most 64 rows per CTA
        const int rpw = RQ / NW;
        const bool got = __all_sync(FULL, mbar_wait(&qbar, 0, a.err));
        const uint64_t* xsp = reinterpret_cast<const uint64_t*>(qkvs);
        const uint8_t* wq = reinterpret_cast<const uint8_t*>(Vs);
        float acc[RPW];
#pragma unroll
        for (int k = 0; k < RPW; k++) acc[k] = 0.0f;
        if (got)
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
                for (int k = 0; k < RPW; k++)
                    if (k < rpw) {
                        const uint8_t* row = wq + (size_t)(warp * rpw + k) * qstride;
                        const float d = __half2float(reinterpret_cast<const __half*>(row + dim)[col >> 5]);
                        acc[k] = fmaf(dot16x2(*reinterpret_cast<const uint4*>(row + col), xp), d, acc[k]);
                    }
            }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
            for (int k = 0; k < RPW; k++) acc[k] += __shfl_xor_sync(FULL, acc[k], m);
        // every lane holds the warp's rpw values: (value k, rank rr) pairs spread over the lanes
        cluster_wait();
        for (int idx = lane; idx < rpw * CL; idx += 32) {
            const int k = idx / CL, rr = idx % CL;
            float v = acc[0];
#pragma unroll
            for (int kk = 1; kk < RPW; kk++)
                if (k == kk) v = acc[kk];
            st_async(cluster_addr(&gq[sp * RQ + warp * rpw + k], rr), v, cluster_addr(&gbar, rr));
        }
        __syncthreads();  // every warp done with the W_qkv rows: their region takes the V tiles
        if (t == 0) {
            fence_proxy_async();  // the weights' generic reads before the copy engine's writes
            for (int tl = 0; tl < min(n_buf, n_tiles); tl++) issue(tl, false, true);
        }
        got_g = __all_sync(FULL, mbar_wait_cluster(&gbar, 0, a.err));  // (if not, the CTA's partial is void)
    }

    // RMSNorm x weight (one warp reduction), RoPE NEOX in registers
    const bool own = pos >= k0 && pos < k1;
    const float* qkv = a.qkv + (long)b * a.qkv_stride;
#pragma unroll
    for (int u = 0; u < HPW; u++) {
        const int h = warp + u * NW;
        if (h > G || (h == G && !own)) continue;
        const float* xr = qkv + (long)(h < G ? j * G + h : a.n_head + j) * HD;
        if constexpr (G <= 4)
            if (fq) xr = gq + (size_t)h * HD;
        const float2 xa = *reinterpret_cast<const float2*>(xr + d0), xb = *reinterpret_cast<const float2*>(xr + 64 + d0);
        float2 va = make_float2(0.f, 0.f), vc = va;
        if (h == G) {
            const float* vr = qkv + (long)(a.n_head + a.n_kv + j) * HD;
            if constexpr (G <= 4)
                if (fq) vr = gq + (size_t)(G + 1) * HD;
            va = *reinterpret_cast<const float2*>(vr + d0);
            vc = *reinterpret_cast<const float2*>(vr + 64 + d0);
        }
        const float ss = warp_sum(xa.x * xa.x + xa.y * xa.y + xb.x * xb.x + xb.y * xb.y);
        const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
        const float n0 = xa.x * inv * w_lo[u].x, n1 = xa.y * inv * w_lo[u].y;
        const float n2 = xb.x * inv * w_hi[u].x, n3 = xb.y * inv * w_hi[u].y;
        const float r0 = n0 * cs.x - n2 * cs.y, r1 = n1 * cs.z - n3 * cs.w;  // dims d0, d0 + 1
        const float r2 = n0 * cs.y + n2 * cs.x, r3 = n1 * cs.w + n3 * cs.z;  // dims 64 + d0, 64 + d0 + 1
        if (h < G) {
            *reinterpret_cast<float2*>(&qs[h][d0]) = make_float2(r0 * a.scale, r1 * a.scale);
            *reinterpret_cast<float2*>(&qs[h][64 + d0]) = make_float2(r2 * a.scale, r3 * a.scale);
        } else {
            // the new token's K / V row: to the cache, and to the extra shared row
            const __half2 k01 = __floats2half2_rn(r0, r1), k23 = __floats2half2_rn(r2, r3);
            const __half2 v01 = __floats2half2_rn(va.x, va.y), v23 = __floats2half2_rn(vc.x, vc.y);
            *reinterpret_cast<__half2*>(kb + (long)pos * HD + d0) = k01;
            *reinterpret_cast<__half2*>(kb + (long)pos * HD + 64 + d0) = k23;
            *reinterpret_cast<__half2*>(vb + (long)pos * HD + d0) = v01;
            *reinterpret_cast<__half2*>(vb + (long)pos * HD + 64 + d0) = v23;
            *reinterpret_cast<__half2*>(Ks + (size_t)ring * HD + d0) = k01;
            *reinterpret_cast<__half2*>(Ks + (size_t)ring * HD + 64 + d0) = k23;
            *reinterpret_cast<__half2*>(Vs + (size_t)ring * HD + d0) = v01;
            *reinterpret_cast<__half2*>(Vs + (size_t)ring * HD + 64 + d0) = v23;
        }
    }
    __syncthreads();

    // ---- the key range in rounds of up to n_buf resident tiles: each warp a contiguous eighth of the round, scores,
    // one online-softmax update and P·V per round; the block meets only when the ring wraps ----
    // scores: 8 lanes per key, lane prt takes dims prt*8 … +7 and 64 + prt*8 … +7 (a quarter-warp's 16-byte reads
    // cover 128 consecutive bytes: no bank conflict)
    const int sub = lane >> 3, prt = lane & 7;
    // q as f32 pairs: [0, 4) dims prt*8 …, [4, 8) dims 64 + prt*8 …
    uint64_t qp[G][8];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float4* q4 = reinterpret_cast<const float4*>(&qs[g][0]);
        const float4 qa = q4[prt * 2], qb = q4[prt * 2 + 1], qc = q4[16 + prt * 2], qd = q4[16 + prt * 2 + 1];
        qp[g][0] = pk2(qa.x, qa.y); qp[g][1] = pk2(qa.z, qa.w); qp[g][2] = pk2(qb.x, qb.y); qp[g][3] = pk2(qb.z, qb.w);
        qp[g][4] = pk2(qc.x, qc.y); qp[g][5] = pk2(qc.z, qc.w); qp[g][6] = pk2(qd.x, qd.y); qp[g][7] = pk2(qd.z, qd.w);
    }
    // per head the running max, sum and this lane's 4 output dims as two f32 pairs
    float mw[G], lw[G];
    uint64_t o2[G][2];
#pragma unroll
    for (int g = 0; g < G; g++) {
        mw[g] = -INFINITY;
        lw[g] = 0.0f;
        o2[g][0] = o2[g][1] = 0;
    }
    bool alive = got_g;
    for (int t0 = 0; t0 < n_tiles; t0 += n_buf) {
        const int t1 = min(n_tiles, t0 + n_buf);  // tiles t0 … t1-1 sit in slots 0 … t1-t0-1
        // (the round's slots share its phase)
        alive = alive && __all_sync(FULL, mbar_wait_n<MAX_BUF>(fk, t1 - t0, (t0 / n_buf) & 1, a.err));
        const int r0 = k0 + t0 * TILE, nk = min(k1, k0 + t1 * TILE) - r0;  // the round's keys [r0, r0 + nk)
        const int prel = pos - r0;  // the new row's index in the round (outside [0, nk) elsewhere)
        const int kw = (nk + NW - 1) / NW;
        const int w0 = min(nk, warp * kw);
        int nw = alive ? min(nk, w0 + kw) - w0 : 0;  // this warp's keys
        // every pass's dot first (independent), then the passes' 8-lane reductions interleaved
        constexpr int NP = KPW / 4;  // passes of 4 keys
        float dk[NP][G];
#pragma unroll
        for (int ps = 0; ps < NP; ps++) {
            const int kk = ps * 4 + sub;
            uint64_t d[G], e[G];
#pragma unroll
            for (int g = 0; g < G; g++) d[g] = e[g] = 0;
            {
                // every pass computes (no branch in the unrolled passes): a key past the warp's share reads a row
                // of the ring (its score is never stored)
                const int i = w0 + min(kk, max(nw - 1, 0));
                const __half* kr = Ks + (size_t)(i == prel ? ring : i) * HD;
                const uint4 u0 = *reinterpret_cast<const uint4*>(kr + prt * 8);
                const uint4 u1 = *reinterpret_cast<const uint4*>(kr + 64 + prt * 8);
                const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
                const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const float2 f0 = __half22float2(h0[c]), f1 = __half22float2(h1[c]);
                    const uint64_t k0p = pk2(f0.x, f0.y), k1p = pk2(f1.x, f1.y);
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        d[g] = fma2(qp[g][c], k0p, d[g]);
                        e[g] = fma2(qp[g][4 + c], k1p, e[g]);
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float2 s2 = upk2(add2(d[g], e[g]));
                dk[ps][g] = s2.x + s2.y;
            }
        }
#pragma unroll
        for (int m = 4; m >= 1; m >>= 1)
#pragma unroll
            for (int ps = 0; ps < NP; ps++)
#pragma unroll
                for (int g = 0; g < G; g++) dk[ps][g] += __shfl_xor_sync(FULL, dk[ps][g], m);
        if (prt == 0)
#pragma unroll
            for (int ps = 0; ps < NP; ps++)
                if (ps * 4 + sub < nw)
#pragma unroll
                    for (int g = 0; g < G; g++) scw[warp][g][ps * 4 + sub] = dk[ps][g];
        __syncwarp();
        // lane = key of this warp's share: the round's max, probabilities, sum
        if (nw > 0) {
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float sc = lane < nw ? scw[warp][g][lane] : -INFINITY;
                const float mn = fmaxf(mw[g], warp_max(sc));
                const float corr = expf(mw[g] - mn);  // exp(-inf) = 0 on the first round
                const float p = lane < nw ? expf(sc - mn) : 0.0f;
                if (lane < KPW) scw[warp][g][lane] = p;  // (0 past the warp's keys: the P·V slots there)
                lw[g] = fmaf(lw[g], corr, warp_sum(p));
                const uint64_t c2 = pk2(corr, corr);
                o2[g][0] = mul2(o2[g][0], c2);
                o2[g][1] = mul2(o2[g][1], c2);
                mw[g] = mn;
            }
        }
        __syncwarp();
        alive = alive && __all_sync(FULL, mbar_wait_n<MAX_BUF>(fv, t1 - t0, (t0 / n_buf) & 1, a.err));
        if (!alive) nw = 0;
        // P·V; lane owns dims 4 lane … 4 lane + 3, over all KPW slots (no trip count): a slot past the warp's
        // keys weighs 0 on a row of its share
        if (nw > 0) {
#pragma unroll
            for (int kk = 0; kk < KPW; kk++) {
                const int i = w0 + min(kk, nw - 1);
                const uint2 u = *reinterpret_cast<const uint2*>(Vs + (size_t)(i == prel ? ring : i) * HD + lane * 4);
                const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                const uint64_t v01 = pk2(v0.x, v0.y), v23 = pk2(v1.x, v1.y);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const float p = scw[warp][g][kk];
                    const uint64_t pp = pk2(p, p);
                    o2[g][0] = fma2(pp, v01, o2[g][0]);
                    o2[g][1] = fma2(pp, v23, o2[g][1]);
                }
            }
        }
        if (t1 < n_tiles) {
            // the ring wraps: every warp is done with the round's rows before they are refilled
            __syncthreads();
            if (t == 0) {
                fence_proxy_async();
                for (int tl = t1; tl < min(n_tiles, t1 + n_buf); tl++) issue(tl, true, true);
            }
        }
    }
    // ---- the CTA's partial: merge the warps ----
    if (lane == 0)
#pragma unroll
        for (int g = 0; g < G; g++) {
            wm[warp][g] = mw[g];
            wl[warp][g] = lw[g];
        }
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float2 o01 = upk2(o2[g][0]), o23 = upk2(o2[g][1]);
        *reinterpret_cast<float4*>(&wo[warp][g][lane * 4]) = make_float4(o01.x, o01.y, o23.x, o23.y);
    }
    const bool ok = __syncthreads_and(alive);  // a warp whose copy wait ran out voids the CTA's partial
    constexpr int PER = G * HD / CL;  // the slice of the group's outputs this CTA merges
    const int q0 = sp * PER;
    float* att = &wo[0][0][0];  // the o-projection's input: the warps' partial outputs are folded by then
    const int nch = (NCOL + 511) / 512;
    bool got_in = true;
    if (!pushm) {
        for (int q = t; q < G * HD; q += AT_THREADS) {
            const int g = q / HD, d = q % HD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w][g]);
            float L = 0.0f, O = 0.0f;
            if (M != -INFINITY && ok)
#pragma unroll
                for (int w = 0; w < NW; w++) {
                    const float e = expf(wm[w][g] - M);
                    L = fmaf(wl[w][g], e, L);
                    O = fmaf(wo[w][g][d], e, O);
                }
            part[g][d] = O;
            if (d == 0) {
                part[g][HD] = (ok && L > 0.0f) ? M : -INFINITY;
                part[g][HD + 1] = ok ? L : 0.0f;
            }
        }
        // ---- the cluster's merge through distributed shared memory ----
        cluster.sync();
        if (rpc == 0) {
            // the attention output: this CTA's slice, from the CL partials
            for (int i = t; i < PER; i += AT_THREADS) {
                const int q = q0 + i, g = q / HD, d = q % HD;
                float ms[CL], ls[CL], os[CL];
#pragma unroll
                for (int r = 0; r < CL; r++) {
                    const float* rp = cluster.map_shared_rank(&part[g][0], r);
                    os[r] = rp[d];
                    ms[r] = rp[HD];
                    ls[r] = rp[HD + 1];
                }
                float M = -INFINITY;
#pragma unroll
                for (int r = 0; r < CL; r++) M = fmaxf(M, ms[r]);
                float L = 0.0f, O = 0.0f;
#pragma unroll
                for (int r = 0; r < CL; r++) {
                    const float e = ms[r] == -INFINITY ? 0.0f : expf(ms[r] - M);
                    L = fmaf(ls[r], e, L);
                    O = fmaf(os[r], e, O);
                }
                a.out[(long)b * a.out_stride + (j * G + g) * HD + d] = O / L;
            }
            cluster.sync();  // no CTA leaves while another still reads its partial
            if (t == 0) tl_record(a.tl, t_start, t_dep);
            return;
        }
        // fused: reduce-scatter (this CTA merges its slice from the ranks' partials, copied in float4s), then all-gather
        // (every CTA reads every slice) — the group's whole output in every CTA, the o-projection's input. Scratch in the
        // idle KV ring: the ranks' slice values [CL][PER], their (m, l) for the slice's head [CL][2], the weights
        // e^(m_r − M) [CL] and their sum L, this CTA's merged slice [PER] (16-B aligned for the all-gather's float4s).
        const int gs = q0 / HD;  // the slice lies within one head
        float* rsl = reinterpret_cast<float*>(sm);
        float* rml = rsl + CL * PER;
        float* ew = rml + CL * 2;
        float* mine = ew + CL + 4;
        constexpr int NSL = CL * (PER / 4);
        for (int i = t; i < NSL + CL; i += AT_THREADS) {
            if (i < NSL) {
                const int r = i / (PER / 4), q = q0 + 4 * (i % (PER / 4));
                const float* rp = cluster.map_shared_rank(&part[0][0], r);
                reinterpret_cast<float4*>(rsl)[i] = *reinterpret_cast<const float4*>(rp + (q / HD) * PW + q % HD);
            } else {
                const float* rp = cluster.map_shared_rank(&part[0][0], i - NSL);
                reinterpret_cast<float2*>(rml)[i - NSL] = *reinterpret_cast<const float2*>(rp + gs * PW + HD);
            }
        }
        __syncthreads();
        // the slice's weights once (lane r of warp 0), L summed over the ranks in order, then one output per thread —
        // the same operations in the same order as merging each output on its own
        if (warp == 0) {
            float M = -INFINITY;
#pragma unroll
            for (int r = 0; r < CL; r++) M = fmaxf(M, rml[2 * r]);
            const float m = lane < CL ? rml[2 * lane] : -INFINITY;
            const float e = m == -INFINITY ? 0.0f : expf(m - M);
            float L = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; r++) L = fmaf(rml[2 * r + 1], __shfl_sync(FULL, e, r), L);
            if (lane < CL) ew[lane] = e;
            if (lane == 0) ew[CL] = L;
        }
        if (PER <= 32) __syncwarp();  // the outputs are warp 0's own
        else __syncthreads();
        for (int i = t; i < PER; i += AT_THREADS) {
            float O = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; r++) O = fmaf(rsl[r * PER + i], ew[r], O);
            mine[i] = O / ew[CL];
        }
        cluster.sync();  // every slice merged; no rank reads `part` any more
        for (int i = t; i < NCOL / 4; i += AT_THREADS) {
            const int q = 4 * i;
            const float* rp = cluster.map_shared_rank(mine, q / PER);
            *reinterpret_cast<float4*>(&att[xs_index(0, nch, q)]) = *reinterpret_cast<const float4*>(rp + q % PER);
        }
        // no remote reads of this CTA's shared memory follow: arrive now, wait before leaving
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
        __syncthreads();
    } else {
        // fused ending by pushes: every output's CTA-merged value goes to the owner of its slice, every head's (m, l)
        // to the owners of that head's slices (into their partbuf); values first, then one barrier — wo is read
        // until then, and it receives the merged outputs after — then the pushes
        constexpr int QPT = (G * HD + AT_THREADS - 1) / AT_THREADS;
        float ov[QPT], mv[QPT], lv[QPT];
#pragma unroll
        for (int u = 0; u < QPT; u++) {
            const int q = t + u * AT_THREADS;
            ov[u] = 0.0f;
            mv[u] = -INFINITY;
            lv[u] = 0.0f;
            if (q < G * HD) {
                const int g = q / HD, d = q % HD;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w][g]);
                float L = 0.0f, O = 0.0f;
                if (M != -INFINITY && ok)
#pragma unroll
                    for (int w = 0; w < NW; w++) {
                        const float e = expf(wm[w][g] - M);
                        L = fmaf(wl[w][g], e, L);
                        O = fmaf(wo[w][g][d], e, O);
                    }
                ov[u] = O;
                mv[u] = (ok && L > 0.0f) ? M : -INFINITY;
                lv[u] = ok ? L : 0.0f;
            }
        }
        __syncthreads();
        if (!fq) cluster_wait();  // (the prologue's arrive: the peers' barriers are ready)
        float* mrs = partbuf;            // [CL][PER]
        float* mrml = partbuf + G * HD;  // [CL][2]
#pragma unroll
        for (int u = 0; u < QPT; u++) {
            const int q = t + u * AT_THREADS;
            if (q < G * HD) {
                const int s = q / PER, d = q % HD;
                st_async(cluster_addr(&mrs[sp * PER + q % PER], s), ov[u], cluster_addr(&mbar, s));
                if (d < HD / PER) {
                    const int s2 = (q / HD) * (HD / PER) + d;
                    st_async(cluster_addr(&mrml[2 * sp], s2), make_float2(mv[u], lv[u]), cluster_addr(&mbar, s2));
                }
            }
        }
        // the merged outputs' pad columns past NCOL are this CTA's zeros
        for (int q = NCOL + 4 * t; q < nch * 512; q += 4 * AT_THREADS)
            *reinterpret_cast<float4*>(&att[xs_index(0, nch, q)]) = make_float4(0.f, 0.f, 0.f, 0.f);
        const bool got_m = __all_sync(FULL, mbar_wait_cluster(&mbar, 0, a.err));
        // this CTA's slice: the ranks' weights once (lane r of warp 0), L summed over the ranks in order, then each
        // (output, rank) pair merged by one thread — the same operations in the same order as merging each output
        // on its own — and pushed into that rank's o-projection input
        float* ew = &scw[0][0][0];  // [CL] weights, then L (the scores' scratch is idle)
        if (warp == 0) {
            float M = -INFINITY;
#pragma unroll
            for (int r = 0; r < CL; r++) M = fmaxf(M, mrml[2 * r]);
            const float m = lane < CL ? mrml[2 * lane] : -INFINITY;
            const float e = m == -INFINITY ? 0.0f : expf(m - M);
            float L = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; r++) L = fmaf(mrml[2 * r + 1], __shfl_sync(FULL, e, r), L);
            if (lane < CL) ew[lane] = e;
            if (lane == 0) ew[CL] = L;
        }
        __syncthreads();
        for (int idx = t; idx < PER * CL; idx += AT_THREADS) {
            const int i = idx % PER, s = idx / PER;
            float O = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; r++) O = fmaf(mrs[r * PER + i], ew[r], O);
            st_async(cluster_addr(&att[xs_index(0, nch, q0 + i)], s), O / ew[CL], cluster_addr(&abar, s));
        }
        cluster_arrive();  // (the final wait keeps every CTA until its peers are done with it)
        got_in = got_m && __all_sync(FULL, mbar_wait_cluster(&abar, 0, a.err));
    }
    // 8 lanes per row (16-column pieces lane&7, +8, …: a row's 128 B per quarter-warp), 4 rows per warp
    const uint64_t* ap = reinterpret_cast<const uint64_t*>(att);
    float* op = a.opart + ((long)b * a.n_kv + j) * mdim + row0;
    const int l8 = lane & 7;
    for (int c0 = 0, k = 0; c0 < rpc; c0 += ro, k++) {
        const int nr = min(ro, rpc - c0);
        const bool got = __all_sync(FULL, mbar_wait(&obar, k & 1, a.err));
        if (got && got_in) {
            // two row groups per warp at once: both dots, then both reductions
            for (int base = warp * 4; base < (OEX ? warp * 4 + 1 : nr); base += NW * 8) {  // (OEX: one pass)
                float acc[2];
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const int rr = base + k * NW * 4 + (lane >> 3);
                    if constexpr (OEX && NCOL % 128 == 0)
                        acc[k] = row_dot8c<NCOL / 128>(wsm + (size_t)rr * ostride, ap, l8);
                    else
                        acc[k] = rr < nr ? row_dot8(wsm + (size_t)rr * ostride, NCOL, ap, l8) : 0.0f;
                }
#pragma unroll
                for (int m = 4; m >= 1; m >>= 1)
#pragma unroll
                    for (int k = 0; k < 2; k++) acc[k] += __shfl_xor_sync(FULL, acc[k], m);
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const int rr = base + k * NW * 4 + (lane >> 3);
                    if (l8 == 0 && (OEX || rr < nr)) op[c0 + rr] = acc[k];
                }
            }
        }
        if (c0 + ro < rpc) {
            __syncthreads();  // every warp is done with the chunk
            if (t == 0) {
                fence_proxy_async();  // the chunk's generic reads before the copy engine's writes
                issue_o(c0 + ro);
            }
        }
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (t == 0) tl_record(a.tl, t_start, t_dep);
}

int attention_splits(int num_sms, int nb, int n_kv, int n_ctx) {
    // the cluster size: 16 CTAs per (slot, kv head) while the clusters fit one wave at two CTAs per SM (a 16-cluster
    // takes 8 SMs of one GPC; a B200 holds 14 such clusters), fewer for batches
    (void)n_ctx;
    const int heads = nb * n_kv;
    if (heads * 16 <= num_sms) return 16;
    if (heads * 9 <= 2 * num_sms) return 8;
    return 4;
}

// the ring depth: the tiles of the longest range, at most MAX_BUF, and no more than keeps a CTA within half an SM's
// shared memory (two CTAs per SM: a cluster of 16 then needs 8 SMs of a GPC)
static int ring_depth(int n_ctx, int cl, int static_bytes) {
    // static_bytes: the kernel's static shared memory plus any dynamic region besides the ring
    const int tiles = ((n_ctx + cl - 1) / cl + TILE - 1) / TILE;
    const int fit = (113 * 1024 - static_bytes - 2 * HD * 2) / (2 * TILE * HD * 2);
    return std::max(1, std::min(std::min(tiles, MAX_BUF), fit));
}

template <int G, int CL>
static int static_smem() {
    static int bytes = -1;
    if (bytes < 0) {
        cudaFuncAttributes fa;
        bytes = cudaFuncGetAttributes(&fa, k_attn_decode<G, CL>) == cudaSuccess ? (int)fa.sharedSizeBytes : 0;
    }
    return bytes;
}

template <int G, int CL>
static cudaLaunchConfig_t config_t(cudaStream_t st, const AttnArgs& a, cudaLaunchAttribute* attr, int* n_buf) {
    // the fused o-projection's W_o region after the ring: up to 64 rows of the CTA's slice rows; the fused qkv
    // projection's W_qkv rows borrow the V region, which grows to hold them when the ring is short
    const size_t wo_bytes = a.wo ? (size_t)std::min(a.dim / CL, 64) * q8_stride(G * HD) : 0;
    const int wq_bytes = a.wqkv.w ? (G + 2) * HD / CL * a.wqkv.stride : 0;
    const int st_bytes = static_smem<G, CL>() + (int)wo_bytes;
    *n_buf = ring_depth(a.n_ctx, CL, st_bytes);
    if (wq_bytes > (*n_buf * TILE + 1) * HD * 2) *n_buf = ring_depth(a.n_ctx, CL, st_bytes + wq_bytes);
    const size_t kreg = (size_t)(*n_buf * TILE + 1) * HD * 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)CL, (unsigned)a.n_kv, (unsigned)a.nb);
    cfg.blockDim = dim3(AT_THREADS, 1, 1);
    cfg.dynamicSmemBytes = kreg + std::max(kreg, (size_t)wq_bytes) + wo_bytes;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// true when a cluster of CL CTAs of this kernel can be resident (16 needs 16 SMs of one GPC with the shared memory)
// the instances' launch attributes, once (every cluster size: each launches with more than 48 KB of shared memory)
template <int G, int CL>
static void configure_t() {
    static PerDeviceOnce once;  // the attributes live in each device's context
    once([] {
        auto kern = k_attn_decode<G, CL>;
        // the opt-in limit: what the SM offers a CTA minus this kernel's static shared memory
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - static_smem<G, CL>());
        if (CL > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if constexpr (G == 2 && CL == 16) {
            auto k1024 = k_attn_decode<G, CL, 1024>;  // (the same static shared memory)
            cudaFuncSetAttribute(k1024, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - static_smem<G, CL>());
            cudaFuncSetAttribute(k1024, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        }
    });
}

template <int G, int CL>
static bool usable_t(cudaStream_t st, const AttnArgs& a) {
    auto kern = k_attn_decode<G, CL>;
    configure_t<G, CL>();
    if (CL <= 8) return true;
    // asked once per (device, dynamic shared memory size), under a lock (contexts may live on several threads)
    static std::mutex mu;
    static int dev_k[16];
    static size_t keys[16];
    static bool vals[16];
    static int n_keys = 0;
    cudaLaunchAttribute attr[2];
    int n_buf = 1, n = 0;
    cudaLaunchConfig_t cfg = config_t<G, CL>(st, a, attr, &n_buf);
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_keys; i++)
        if (dev_k[i] == dev && keys[i] == cfg.dynamicSmemBytes) return vals[i];
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    if (n_keys < 16) {
        dev_k[n_keys] = dev;
        keys[n_keys] = cfg.dynamicSmemBytes;
        vals[n_keys++] = n >= 1;
    }
    return n >= 1;
}

template <int G, int CL>
static void launch_t(cudaStream_t st, const AttnArgs& a, bool pdl) {
    configure_t<G, CL>();
    cudaLaunchAttribute attr[2];
    int n_buf = 1;
    cudaLaunchConfig_t cfg = config_t<G, CL>(st, a, attr, &n_buf);
    cfg.numAttrs = pdl ? 2 : 1;
    auto kern = k_attn_decode<G, CL>;
    // Qwen3-0.6B's decode step (fused projections, dim 1024): the instance compiled for that dim
    if constexpr (G == 2 && CL == 16)
        if (a.wqkv.w && a.in.w.cols == 1024 && a.wo && a.dim == 1024 && n_buf == MAX_BUF)
            kern = k_attn_decode<G, CL, 1024>;
    cudaLaunchKernelEx(&cfg, kern, a, n_buf, (int)cfg.dynamicSmemBytes);
}

template <int G>
static int cluster_g(const AttnArgs& a) {
    if (a.splits == 16 && usable_t<G, 16>(nullptr, a)) return 16;
    if (a.splits >= 8 && usable_t<G, 8>(nullptr, a)) return 8;
    return 4;
}

int attention_cluster(const AttnArgs& a) {
    const int G = a.n_head / a.n_kv;
    return G == 1 ? cluster_g<1>(a) : G == 2 ? cluster_g<2>(a) : G == 4 ? cluster_g<4>(a) : cluster_g<8>(a);
}

bool attention_fuses_qkv(int g, int cl, int dim) {
    const int rq = (g + 2) * HD / cl;  // rows per CTA: whole, within one of q / k / v, RQ / NW per warp (≤ 8)
    return g <= 4 && (g + 2) * HD % cl == 0 && HD % rq == 0 && rq % NW == 0 && rq / NW <= 8 && rq % 4 == 0 && dim % 32 == 0 &&
           dim <= 1024 && (dim + 511) / 512 * 512 <= NW * g * HD;
}

template <int G>
static void launch_g(cudaStream_t st, const AttnArgs& a, bool pdl) {
    const int cl = cluster_g<G>(a);
    if (cl == 16) launch_t<G, 16>(st, a, pdl);
    else if (cl == 8) launch_t<G, 8>(st, a, pdl);
    else launch_t<G, 4>(st, a, pdl);
}

void launch_attention_decode(cudaStream_t st, const AttnArgs& a, bool pdl) {
    const int G = a.n_head / a.n_kv;
    if (G == 1) launch_g<1>(st, a, pdl);
    else if (G == 2) launch_g<2>(st, a, pdl);
    else if (G == 4) launch_g<4>(st, a, pdl);
    else launch_g<8>(st, a, pdl);
}

}  // namespace ocr

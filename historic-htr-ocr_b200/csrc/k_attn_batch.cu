// k_attn_batch.cu — decode attention for a batch of slots, one token each: the reference's qkv_post.wgsl (q/k RMSNorm →
// RoPE NEOX → f16 K/V store, qkv_post.wgsl:31-83), attn_decode.wgsl (per-range softmax partials m, l, o[128],
// attn_decode.wgsl:34-100) and attn_merge.wgsl (attn_merge.wgsl:22-39), shaped for throughput rather than latency.
//
// At batch 32 the attention reads 32 slots x 8 kv heads x (3072 … 4096) keys x 512 B — ~95 % of a decode step's bytes —
// so the kernel is a plain HBM stream: one CTA per (slot, kv head) (or `split` CTAs over its keys when the batch has
// too few pairs to fill the GPU), two CTAs per SM, so a 32-slot batch's 256 pairs are one wave with no cross-CTA
// merge. Warp 8 streams the (slot, head)'s key range — one contiguous run of K rows and one of V rows in the cache
// layout [slot][kv head][n_ctx][128] f16 — in 64-key tiles (16 KB of K + 16 KB of V per bulk-copy stage, a ring of
// three) under an L2 evict-first policy; the first stages are issued before griddepcontrol.wait (rows below pos are
// from earlier steps). Warps 0-7 take 8 keys of each tile: scores with 8 lanes per key (16 dims each, packed f32x2
// FMAs on the f16 rows), an online-softmax update per tile (running max, sum, rescale), then P·V with each lane owning
// 4 output dims. The new token's q heads and K/V row are prepared first (one warp per head: RMSNorm by a warp
// reduction, RoPE from the host-computed table, q pre-scaled by 1/sqrt(128)), the K/V row stored f16 to the cache by
// the CTA that owns the last key and kept in shared memory for its own last tile.
//
// Output: the G heads' merged rows o = O / L as the o-projection's operand — f16 hi / lo in the tensor-core
// contraction's layout (x16, over qd = n_head x 128 columns) — and optionally as f32 rows. With split > 1 each CTA
// writes its (m, l, o) partial and the last CTA of the pair (threadfence + ticket, no waiting) merges them in split
// order. Every mbarrier wait is bounded (mbar_wait); a wait that runs out flags DEV_TIMEOUT and voids the CTA's result.
#include "kernels.cuh"
#include "qdot.cuh"

namespace ocr {

constexpr int AB_WARPS = 8;                 // compute warps; warp 8 copies
constexpr int AB_THREADS = (AB_WARPS + 1) * 32;
constexpr int AB_TK = 64;                   // keys per tile
constexpr int AB_NBUF = 3;                  // ring stages
constexpr int AB_HD = 128;
constexpr int AB_KPW = AB_TK / AB_WARPS;    // keys per warp per tile (8: two passes of 4)
constexpr uint32_t AB_TILE_BYTES = AB_TK * AB_HD * 2;  // 16 KB of K (and of V)
constexpr int AB_PW = AB_HD + 4;            // a head's partial: o[128], m, l, pad

template <int G>
__global__ void __launch_bounds__(AB_THREADS, 2) k_attn_batch(AttnBatchArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t full[AB_NBUF], empty[AB_NBUF];
    __shared__ __align__(16) float qs[G][AB_HD];
    __shared__ __align__(16) __half knew[AB_HD], vnew[AB_HD];  // the new token's K / V row (f16, as stored)
    __shared__ float wm[AB_WARPS][G], wl[AB_WARPS][G];
    __shared__ __align__(16) float wo[AB_WARPS][G][AB_HD];
    __shared__ int s_ok;
    __shared__ uint32_t s_ticket;
    const int sp = blockIdx.x, j = blockIdx.y, b = blockIdx.z, split = gridDim.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const unsigned long long t_start = a.tl ? gtimer() : 0ull;
    __shared__ unsigned long long t_dep;
    if (a.active && !a.active[b]) return;  // (uniform over the CTA)
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.n_ctx) {
        if (sp == 0 && j == 0 && t == 0) dev_error(a.err, DEV_BAD_POS);
        return;
    }
    const int n_keys = pos + 1;
    const int per = (n_keys + split - 1) / split;
    const int k0 = min(n_keys, sp * per), k1 = min(n_keys, k0 + per);
    const int n_tiles = (k1 - k0 + AB_TK - 1) / AB_TK;
    const bool own = pos >= k0 && pos < k1;  // this CTA's range holds the new key
    const long head_base = ((long)b * a.n_kv + j) * a.n_ctx;
    __half* kb = a.kc + head_base * AB_HD;
    __half* vb = a.vc + head_base * AB_HD;
    __half* Ks = reinterpret_cast<__half*>(sm);                 // [AB_NBUF][AB_TK][128]
    __half* Vs = Ks + (size_t)AB_NBUF * AB_TK * AB_HD;          // [AB_NBUF][AB_TK][128]

    if (t == 0) {
        for (int i = 0; i < AB_NBUF; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], AB_WARPS);
        }
        s_ok = 1;
        mbar_fence_init();
    }
    __syncthreads();

    // the copies of tile i (rows [ts, min(te, pos)): the row at pos is not in the cache yet) into stage i % AB_NBUF
    auto issue = [&](int i, uint64_t pol) {
        const int s = i % AB_NBUF, ts = k0 + i * AB_TK, ce = min(min(k1, ts + AB_TK), pos);
        const uint32_t bytes = ce > ts ? (uint32_t)(ce - ts) * AB_HD * 2 : 0;
        if (bytes) {
            mbar_expect_tx(&full[s], 2 * bytes);
            bulk_g2s_stream(Ks + (size_t)s * AB_TK * AB_HD, kb + (long)ts * AB_HD, bytes, &full[s], pol);
            bulk_g2s_stream(Vs + (size_t)s * AB_TK * AB_HD, vb + (long)ts * AB_HD, bytes, &full[s], pol);
        } else {
            mbar_arrive(&full[s]);  // nothing to copy: the phase completes
        }
    };

    if (warp == AB_WARPS) {
        // ---- the copies ----
        if (lane == 0) {
            const uint64_t pol = l2_evict_first();
            const int pre = min(AB_NBUF, n_tiles);
            for (int i = 0; i < pre; i++) issue(i, pol);  // rows below pos: written by earlier steps
            pdl_trigger();
            pdl_wait();
            bool ok = true;
            int i = pre;
            for (; i < n_tiles; i++) {
                const int s = i % AB_NBUF;
                if (!mbar_wait(&empty[s], ((i / AB_NBUF) - 1) & 1, a.err)) {
                    ok = false;
                    break;
                }
                issue(i, pol);
            }
            if (!ok) s_ok = 0;
            // every copy issued has landed before the CTA may exit (bounded)
            for (int k = max(0, i - AB_NBUF); k < i; k++) mbar_wait(&full[k % AB_NBUF], (k / AB_NBUF) & 1, a.err);
        }
        __syncwarp();
    } else {
        // ---- the new token: q head h by warp h % 8, the K / V head (h = G) only in the CTA owning the last key ----
        const float4 cs = *reinterpret_cast<const float4*>(a.rope + (long)pos * AB_HD + 4 * lane);
        const int d0 = 2 * lane;  // this lane: dims d0, d0 + 1 and their RoPE partners 64 + d0, 64 + d0 + 1
        pdl_wait();
        if (t == 0 && a.tl) t_dep = gtimer();
        for (int h = warp; h <= G; h += AB_WARPS) {
            if (h == G && !own) continue;
            const float* wv = h < G ? a.q_norm : a.k_norm;
            const float2 w_lo = *reinterpret_cast<const float2*>(wv + d0);
            const float2 w_hi = *reinterpret_cast<const float2*>(wv + 64 + d0);
            const float* qkv = a.qkv + (long)b * a.qkv_stride;
            const float* xr = qkv + (long)(h < G ? j * G + h : a.n_head + j) * AB_HD;
            const float2 xa = *reinterpret_cast<const float2*>(xr + d0), xb = *reinterpret_cast<const float2*>(xr + 64 + d0);
            const float ss = warp_sum(xa.x * xa.x + xa.y * xa.y + xb.x * xb.x + xb.y * xb.y);
            const float inv = 1.0f / sqrtf(ss / (float)AB_HD + a.eps);
            const float n0 = xa.x * inv * w_lo.x, n1 = xa.y * inv * w_lo.y;
            const float n2 = xb.x * inv * w_hi.x, n3 = xb.y * inv * w_hi.y;
            // (the table row holds (cos, sin) of dims d0, d0 + 1 at 4 lane … 4 lane + 3)
            const float r0 = n0 * cs.x - n2 * cs.y, r1 = n1 * cs.z - n3 * cs.w;
            const float r2 = n0 * cs.y + n2 * cs.x, r3 = n1 * cs.w + n3 * cs.z;
            if (h < G) {
                *reinterpret_cast<float2*>(&qs[h][d0]) = make_float2(r0 * a.scale, r1 * a.scale);
                *reinterpret_cast<float2*>(&qs[h][64 + d0]) = make_float2(r2 * a.scale, r3 * a.scale);
            } else {
                const float* vr = qkv + (long)(a.n_head + a.n_kv + j) * AB_HD;
                const float2 va = *reinterpret_cast<const float2*>(vr + d0), vc = *reinterpret_cast<const float2*>(vr + 64 + d0);
                const __half2 k01 = __floats2half2_rn(r0, r1), k23 = __floats2half2_rn(r2, r3);
                const __half2 v01 = __floats2half2_rn(va.x, va.y), v23 = __floats2half2_rn(vc.x, vc.y);
                *reinterpret_cast<__half2*>(kb + (long)pos * AB_HD + d0) = k01;
                *reinterpret_cast<__half2*>(kb + (long)pos * AB_HD + 64 + d0) = k23;
                *reinterpret_cast<__half2*>(vb + (long)pos * AB_HD + d0) = v01;
                *reinterpret_cast<__half2*>(vb + (long)pos * AB_HD + 64 + d0) = v23;
                *reinterpret_cast<__half2*>(knew + d0) = k01;
                *reinterpret_cast<__half2*>(knew + 64 + d0) = k23;
                *reinterpret_cast<__half2*>(vnew + d0) = v01;
                *reinterpret_cast<__half2*>(vnew + 64 + d0) = v23;
            }
        }
        // the compute warps only (barrier 1): the copy warp may be waiting for them to free a stage
        bar_sync(1, AB_WARPS * 32);
    }

    if (warp < AB_WARPS) {
        // ---- the key range, tile by tile ----
        const int sub = lane >> 3, prt = lane & 7;  // scores: key sub of a pass of 4, dims prt*8 … and 64 + prt*8 …
        uint64_t qp[G][8];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float4* q4 = reinterpret_cast<const float4*>(&qs[g][0]);
            const float4 qa = q4[prt * 2], qb = q4[prt * 2 + 1], qc = q4[16 + prt * 2], qd = q4[16 + prt * 2 + 1];
            qp[g][0] = pk2(qa.x, qa.y); qp[g][1] = pk2(qa.z, qa.w); qp[g][2] = pk2(qb.x, qb.y); qp[g][3] = pk2(qb.z, qb.w);
            qp[g][4] = pk2(qc.x, qc.y); qp[g][5] = pk2(qc.z, qc.w); qp[g][6] = pk2(qd.x, qd.y); qp[g][7] = pk2(qd.z, qd.w);
        }
        float mw[G], lw[G];
        uint64_t o2[G][2];
#pragma unroll
        for (int g = 0; g < G; g++) {
            mw[g] = -INFINITY;
            lw[g] = 0.0f;
            o2[g][0] = o2[g][1] = 0;
        }
        bool alive = true;
        for (int i = 0; i < n_tiles; i++) {
            const int s = i % AB_NBUF;
            alive = alive && __all_sync(FULL, mbar_wait(&full[s], (i / AB_NBUF) & 1, a.err));
            const int ts = k0 + i * AB_TK, nk = min(k1 - ts, AB_TK);
            const __half* Kt = Ks + (size_t)s * AB_TK * AB_HD;
            const __half* Vt = Vs + (size_t)s * AB_TK * AB_HD;
            const int kw0 = warp * AB_KPW;  // this warp's keys kw0 … kw0 + 7 of the tile
            if (alive) {
                // scores of the warp's 8 keys: two passes of 4 keys, 8 lanes each
                float sc[2][G];
#pragma unroll
                for (int ps = 0; ps < 2; ps++) {
                    const int kk = kw0 + ps * 4 + sub;
                    const int kc = min(kk, nk - 1);  // (a key past the tile's end reads a real row; its score is dropped)
                    const __half* kr = ts + kc == pos ? knew : Kt + (size_t)kc * AB_HD;
                    const uint4 u0 = *reinterpret_cast<const uint4*>(kr + prt * 8);
                    const uint4 u1 = *reinterpret_cast<const uint4*>(kr + 64 + prt * 8);
                    const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
                    const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
                    uint64_t d[G], e[G];
#pragma unroll
                    for (int g = 0; g < G; g++) d[g] = e[g] = 0;
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
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        const float2 s2 = upk2(add2(d[g], e[g]));
                        float v = s2.x + s2.y;
                        v += __shfl_xor_sync(FULL, v, 4);
                        v += __shfl_xor_sync(FULL, v, 2);
                        v += __shfl_xor_sync(FULL, v, 1);
                        sc[ps][g] = kk < nk ? v : -INFINITY;  // (a key past the tile's end: weight 0)
                    }
                }
                // online softmax over the tile's 8 keys of this warp (each key's score sits in its 8 lanes)
                float p[2][G];
#pragma unroll
                for (int g = 0; g < G; g++) {
                    float mx = fmaxf(sc[0][g], sc[1][g]);
                    mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 16));
                    const float mn = fmaxf(mw[g], mx);
                    // (no key of the warp yet: mn stays -inf, every p 0 and corr 1)
                    const float corr = mn == -INFINITY ? 1.0f : expf(mw[g] - mn);
                    p[0][g] = mn == -INFINITY ? 0.0f : expf(sc[0][g] - mn);
                    p[1][g] = mn == -INFINITY ? 0.0f : expf(sc[1][g] - mn);
                    float ps = p[0][g] + p[1][g];
                    ps += __shfl_xor_sync(FULL, ps, 8);
                    ps += __shfl_xor_sync(FULL, ps, 16);
                    lw[g] = fmaf(lw[g], corr, ps);
                    const uint64_t c2 = pk2(corr, corr);
                    o2[g][0] = mul2(o2[g][0], c2);
                    o2[g][1] = mul2(o2[g][1], c2);
                    mw[g] = mn;
                }
                // P·V: lane owns dims 4 lane … 4 lane + 3; key kk's weight sits in lanes 8 (kk % 4) … of pass kk / 4
#pragma unroll
                for (int kk = 0; kk < AB_KPW; kk++) {
                    const int key = min(kw0 + kk, nk - 1);  // (past the tile's end: a real row at weight 0)
                    const __half* vr = ts + key == pos ? vnew : Vt + (size_t)key * AB_HD;
                    const uint2 u = *reinterpret_cast<const uint2*>(vr + lane * 4);
                    const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                    const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                    const uint64_t v01 = pk2(v0.x, v0.y), v23 = pk2(v1.x, v1.y);
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        const float pv = __shfl_sync(FULL, p[kk >> 2][g], (kk & 3) * 8);
                        const uint64_t pp = pk2(pv, pv);
                        o2[g][0] = fma2(pp, v01, o2[g][0]);
                        o2[g][1] = fma2(pp, v23, o2[g][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage
        }
        if (!alive && lane == 0) s_ok = 0;
        // ---- the warp's state → shared memory ----
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
    }
    __syncthreads();
    const bool ok = s_ok != 0;  // (a wait that ran out voids the CTA's result; the error flag is set)

    // ---- the CTA's (m, l, o) per head, the warps merged in order; then the output (or the pair's merge) ----
    // output q of the group (head q / 128, dim q % 128), q = t, t + AB_THREADS, …
    const long pair = (long)b * a.n_kv + j;
    auto cta_part = [&](int q, float& cm, float& cl, float& co) {
        const int g = q / AB_HD, d = q % AB_HD;
        cm = -INFINITY;
        cl = co = 0.0f;
#pragma unroll
        for (int w = 0; w < AB_WARPS; w++) cm = fmaxf(cm, wm[w][g]);
        if (cm != -INFINITY && ok)
#pragma unroll
            for (int w = 0; w < AB_WARPS; w++) {
                const float e = expf(wm[w][g] - cm);
                cl = fmaf(wl[w][g], e, cl);
                co = fmaf(wo[w][g][d], e, co);
            }
        if (!ok) cm = -INFINITY;  // a void partial: weight 0 in the merge
    };
    auto emit = [&](int q, float out) {
        const int col = j * G * AB_HD + q;  // the slot's output row: heads in order, 128 dims each
        if (a.out) a.out[(long)b * a.out_stride + col] = out;
        if (a.x16) {
            const __half hh = __float2half_rn(out);
            const __half hl = __float2half_rn(out - __half2float(hh));
            uint8_t* xg = a.x16 + (size_t)(b / BG_SLOTS) * x16_group_bytes(a.n_head * AB_HD);
            *reinterpret_cast<__half*>(xg + x16_offset(b % BG_SLOTS, col)) = hh;
            *reinterpret_cast<__half*>(xg + x16_offset(BG_SLOTS + b % BG_SLOTS, col)) = hl;
        }
    };
    if (split == 1) {
        for (int q = t; q < G * AB_HD; q += AB_THREADS) {
            float cm, cl, co;
            cta_part(q, cm, cl, co);
            emit(q, cl > 0.0f ? co / cl : 0.0f);
        }
        if (t == 0) tl_record(a.tl, t_start, t_dep);
        return;
    }
    // the partials of the pair's CTAs: [pair][split][G][AB_PW]; the last CTA to finish merges them in split order
    float* part = a.part + (pair * split + sp) * G * AB_PW;
    for (int q = t; q < G * AB_HD; q += AB_THREADS) {
        float cm, cl, co;
        cta_part(q, cm, cl, co);
        const int g = q / AB_HD, d = q % AB_HD;
        part[g * AB_PW + d] = co;
        if (d == 0) {
            part[g * AB_PW + AB_HD] = cm;
            part[g * AB_PW + AB_HD + 1] = cl;
        }
    }
    __threadfence();
    __syncthreads();
    if (t == 0) s_ticket = atomicAdd(&a.done[pair], 1u);
    __syncthreads();
    if (s_ticket != (uint32_t)split - 1) {
        if (t == 0) tl_record(a.tl, t_start, t_dep);
        return;
    }
    __threadfence();
    const float* pp = a.part + pair * split * G * AB_PW;
    for (int q = t; q < G * AB_HD; q += AB_THREADS) {
        const int g = q / AB_HD, d = q % AB_HD;
        float M = -INFINITY;
        for (int r = 0; r < split; r++) M = fmaxf(M, __ldcg(pp + ((long)r * G + g) * AB_PW + AB_HD));
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY)
            for (int r = 0; r < split; r++) {
                const float* pr = pp + ((long)r * G + g) * AB_PW;
                const float e = expf(__ldcg(pr + AB_HD) - M);
                L = fmaf(__ldcg(pr + AB_HD + 1), e, L);
                O = fmaf(__ldcg(pr + d), e, O);
            }
        emit(q, L > 0.0f ? O / L : 0.0f);
    }
    if (t == 0) {
        a.done[pair] = 0u;  // (self-resetting for the next launch)
        tl_record(a.tl, t_start, t_dep);
    }
}

int attn_batch_split(int num_sms, int nb, int n_kv) {
    const int pairs = nb * n_kv;
    return std::max(1, std::min(AB_MAX_SPLIT, 2 * num_sms / std::max(1, pairs)));
}

template <int G>
static void launch_g(cudaStream_t st, const AttnBatchArgs& a, int split, bool pdl) {
    static PerDeviceOnce once;
    const int smem = (int)(2 * AB_NBUF * AB_TILE_BYTES);
    once([&] { cudaFuncSetAttribute(k_attn_batch<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)split, (unsigned)a.n_kv, (unsigned)a.nb);
    cfg.blockDim = dim3(AB_THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, k_attn_batch<G>, a);
}

void launch_attention_batch(cudaStream_t st, const AttnBatchArgs& a, int split, bool pdl) {
    const int G = a.n_head / a.n_kv;
    if (G == 1) launch_g<1>(st, a, split, pdl);
    else if (G == 2) launch_g<2>(st, a, split, pdl);
    else if (G == 4) launch_g<4>(st, a, split, pdl);
    else launch_g<8>(st, a, split, pdl);
}

}  // namespace ocr

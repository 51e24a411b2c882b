// k_attn_prefill_tc.cu — attention over f16 keys and values on the 5th-generation tensor cores (tcgen05, sm_100a),
// one CTA per (tile of 128 queries, head), in two forms of one template:
//   - causal, head dim 128: the text prefill, the reference's attention_causal.wgsl (TextModel::prefill,
//     app/crates/ocr-wgpu/src/text.rs:437-521) over the f16 KV cache;
//   - full (every query sees every key), head dim 64: the vision encoder's attention over all patches, the
//     reference's attention_coop.wgsl / attention.wgsl (Vision::run, app/crates/ocr-wgpu/src/vision.rs:290-295),
//     over K / V rounded to f16 like its f16 path (vision.rs:319-327), writing the o-projection's operand.
//
// Numerics. K and V are f16, so they are tensor-core operands as they are. Each query row (f32, scaled by
// 1/sqrt(d_head) as the f32 kernels do) splits exactly into f16 hi + lo, so S = Q_hi K^T + Q_lo K^T (f32
// accumulation) is the f32 product up to the dropped remainder (below 2^-22 of each term). Softmax in two passes: the
// first takes each row's maximum over its keys, the second forms p = exp(s - max) (0 for keys the row does not see),
// sums them in key order, splits each p exactly into f16 hi + lo and accumulates O += P_hi V + P_lo V in TMEM — no
// rescaling of O. The output row is O / sum.
//
// Roles (416 threads): warps 0-3 own the 128 query rows (TMEM lanes): read S, the maxima, P, the output; warp 4 (one
// lane) allocates TMEM and issues the MMAs; warps 5-12 stage the K tiles (both passes) and the V tiles (pass 2),
// transposed so that every operand is K-major with the 128-byte swizzle — each thread issuing all its loads of a
// tile before its stores. S is double-buffered in TMEM, so the product of the next key tile runs while the rows read
// the current one. Every wait is bounded; the staging is plain loads and stores (no asynchronous copy to drain).
#include "kernels.cuh"
#include "tc.cuh"

namespace ocr {

constexpr int PA_QT = 128;       // queries per CTA: the MMA's M, one TMEM lane each
constexpr int PA_KT = 64;        // keys per tile
constexpr int PA_LOADERS = 8;    // warps 5-12: the staging
constexpr int PA_THREADS = (5 + PA_LOADERS) * 32;
// the pre-tiled form (K and V^T already in the operand layout in global memory, each tile one bulk copy): warps 0-3
// the rows, warp 4 the tensor cores, warp 5 the copies — two CTAs per SM
constexpr int PA_THREADS_TILED = 6 * 32;
__host__ __device__ constexpr int pa_threads(bool tiled) { return tiled ? PA_THREADS_TILED : PA_THREADS; }
constexpr uint32_t PA_TMEM_COLS = 256;  // S at columns 0 and 64 (double buffer), O at 128 … 128 + D
constexpr float PA_RESCALE = 8.0f;      // the one-pass form's headroom over the running maximum (log2 units)
// the shared-memory plan of head dim D: Q hi / lo, two K tiles, two V tiles (transposed), P hi / lo
// (the tiled form's V^T tiles carry 16 more rows: a row of ones, whose product with P is the row sum of P, then zeros)
template <int D, bool TILED = false>
struct PaPlan {
    static constexpr int KPT = (PA_KT * D / 8 + PA_LOADERS * 32 - 1) / (PA_LOADERS * 32);  // K pieces per thread
    static constexpr int VROWS = TILED ? D + 16 : D;    // the P V product's N
    static constexpr uint32_t Q_BYTES = PA_QT * D * 2;  // one f16 operand of the Q tile: D/64 halves of 64 dims
    static constexpr uint32_t K_BYTES = PA_KT * D * 2;  // a K tile: D/64 halves of 64 dims, 64 key rows each
    static constexpr uint32_t V_BYTES = VROWS * PA_KT * 2;  // a V tile transposed: the dim rows of the tile's 64 keys
    static constexpr uint32_t P_BYTES = PA_QT * PA_KT * 2;  // one f16 operand of P: 128 query rows of 64 keys
    static constexpr uint32_t SMEM = 2 * Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + 2 * P_BYTES + 1024;
};

struct PaShared {
    uint64_t kfull[2], kempty[2], vfull[2], vempty[2], sfull[2], sfree[2];
    uint64_t pfull, pfree, ofull, mdone;
    uint32_t tmem;
    int abort_flag;
};

// byte offset of 16-byte piece p (8 columns) of row r in a K-major 128-byte-swizzle region (64 f16 columns per row)
__device__ __forceinline__ uint32_t sw128(int r, int p) { return (uint32_t)r * 128u + (uint32_t)((p ^ (r & 7)) << 4); }

// a bounded wait that also gives up when another role has given up
__device__ __forceinline__ bool pa_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
    for (uint32_t i = 0; i < MBAR_TRIES; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    dev_error(err, DEV_TIMEOUT);
    return false;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __halves2half2(__float2half_rn(a), __float2half_rn(b));
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <int D, bool CAUSAL, bool TILED>
__global__ void __launch_bounds__(pa_threads(TILED), TILED ? 2 : 1) k_attn_tc(TcAttnArgs a) {
    constexpr int THREADS = pa_threads(TILED);
    static_assert(!TILED || D == 64, "the pre-tiled operands are written for head dim 64");
    using P = PaPlan<D, TILED>;
    const int L = a.L, pos0 = a.pos0;
    // the tiled form works in log2 units (scores times log2 e, probabilities by exp2)
    const float qscale = TILED ? a.scale * 1.4426950408889634f : a.scale;
    int* err = a.err;
    extern __shared__ uint8_t sm_raw[];
    __shared__ __align__(8) PaShared sh;
    volatile int* abort_flag = &sh.abort_flag;
    uint8_t* smp = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
    uint8_t* Qh = smp;
    uint8_t* Ql = Qh + P::Q_BYTES;
    uint8_t* Kr = Ql + P::Q_BYTES;      // [2] K tiles
    uint8_t* Vr = Kr + 2 * P::K_BYTES;  // [2] V tiles, transposed
    uint8_t* Ph = Vr + 2 * P::V_BYTES;
    uint8_t* Pl = Ph + P::P_BYTES;
    const int h = blockIdx.y, kh = h / a.group, q0 = blockIdx.x * PA_QT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // causal: keys 0 … the position of the tile's last query; full: every key
    const int n_keys = CAUSAL ? pos0 + min(L, q0 + PA_QT) : a.n_keys;
    const int T = (n_keys + PA_KT - 1) / PA_KT;
    const __half* kbase = a.k + (size_t)kh * a.kv_head_stride;
    const __half* vbase = a.v + (size_t)kh * a.kv_head_stride;

    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&sh.kfull[i], TILED ? 1 : PA_LOADERS);
            mbar_init(&sh.kempty[i], 1);
            mbar_init(&sh.vfull[i], TILED ? 1 : PA_LOADERS);
            mbar_init(&sh.vempty[i], 1);
            mbar_init(&sh.sfull[i], 1);
            mbar_init(&sh.sfree[i], 4);
        }
        mbar_init(&sh.pfull, 4);
        mbar_init(&sh.pfree, 1);
        mbar_init(&sh.ofull, 1);
        mbar_init(&sh.mdone, 1);
        sh.abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 4) {
        tmem_alloc(&sh.tmem, PA_TMEM_COLS);
        tmem_relinquish();
    }
    // the Q tile, scaled, split f16 hi / lo: row r, 8 dims per 16-byte piece, dims in D/64 halves of 64 columns (rows
    // past L zero)
    for (int e = tid; e < PA_QT * (D / 8); e += THREADS) {
        const int r = e / (D / 8), pc = e % (D / 8), hf = pc >> 3, p = pc & 7;
        uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = make_uint4(0u, 0u, 0u, 0u);
        if (q0 + r < L) {
            const float4* src = reinterpret_cast<const float4*>(a.q + (size_t)(q0 + r) * a.q_stride + h * D + pc * 8);
            const float4 a0 = src[0], a1 = src[1];
            const float v[8] = {a0.x * qscale, a0.y * qscale, a0.z * qscale, a0.w * qscale,
                                a1.x * qscale, a1.y * qscale, a1.z * qscale, a1.w * qscale};
            float vh[8];
#pragma unroll
            for (int c = 0; c < 8; c++) vh[c] = __half2float(__float2half_rn(v[c]));
            hi = make_uint4(pack_h2(vh[0], vh[1]), pack_h2(vh[2], vh[3]), pack_h2(vh[4], vh[5]), pack_h2(vh[6], vh[7]));
            lo = make_uint4(pack_h2(v[0] - vh[0], v[1] - vh[1]), pack_h2(v[2] - vh[2], v[3] - vh[3]),
                            pack_h2(v[4] - vh[4], v[5] - vh[5]), pack_h2(v[6] - vh[6], v[7] - vh[7]));
        }
        *reinterpret_cast<uint4*>(Qh + hf * (PA_QT * 128) + sw128(r, p)) = hi;
        *reinterpret_cast<uint4*>(Ql + hf * (PA_QT * 128) + sw128(r, p)) = lo;
    }
    if constexpr (TILED) {  // rows D … D + 15 of both V^T buffers: ones, then zeros (the copies never write them)
        for (int e = tid; e < 2 * 16 * 8; e += THREADS) {
            const int b = e / 128, r = (e / 8) % 16, p = e % 8;
            const uint32_t one = r == 0 ? 0x3C003C00u : 0u;
            *reinterpret_cast<uint4*>(Vr + b * P::V_BYTES + sw128(D + r, p)) = make_uint4(one, one, one, one);
        }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem;
    const uint32_t tS = tmem, tO = tmem + 128;

    if (TILED && warp == 5) {
        // ---- the copies: each tile's K, then its V^T (one bulk copy each) ----
        if (lane == 0) {
            bool ok = true;
            uint32_t kn[2] = {0u, 0u}, vn[2] = {0u, 0u};  // copies issued per ring slot
            for (int t = 0; t < T && ok; t++) {  // each tile's K, then its V^T (one pass)
                const int ks = t & 1;
                if (t >= 2 && !(ok = pa_wait(&sh.kempty[ks], ((t >> 1) - 1) & 1, abort_flag, err))) break;
                mbar_expect_tx(&sh.kfull[ks], P::K_BYTES);
                bulk_g2s(Kr + ks * P::K_BYTES, kbase + (size_t)t * PA_KT * D, P::K_BYTES, &sh.kfull[ks]);
                kn[ks]++;
                if (t >= 2 && !(ok = pa_wait(&sh.vempty[ks], ((t >> 1) - 1) & 1, abort_flag, err))) break;
                mbar_expect_tx(&sh.vfull[ks], D * PA_KT * 2);  // (the dim rows; the ones row stays)
                bulk_g2s(Vr + ks * P::V_BYTES, vbase + (size_t)t * PA_KT * D, D * PA_KT * 2, &sh.vfull[ks]);
                vn[ks]++;
            }
            if (!ok) *abort_flag = 1;
            // every copy landed before the shared memory is given back (bounded; the last phase of each slot)
            for (int i = 0; i < 2; i++) {
                if (kn[i]) mbar_wait(&sh.kfull[i], (kn[i] - 1) & 1, err);
                if (vn[i]) mbar_wait(&sh.vfull[i], (vn[i] - 1) & 1, err);
            }
        }
        __syncwarp();
    } else if (!TILED && warp >= 5) {
        // ---- staging: pass 1 the K tiles; pass 2 each tile's K, then its V transposed ----
        const int lt = tid - 5 * 32;
        bool ok = true;
        for (int seq = 0; seq < 2 * T && ok; seq++) {
            const int t = seq < T ? seq : seq - T, kb0 = t * PA_KT, ks = seq & 1;
            if (seq >= 2 && !pa_wait(&sh.kempty[ks], ((seq >> 1) - 1) & 1, abort_flag, err)) {
                ok = false;
                break;
            }
            uint8_t* kt = Kr + ks * P::K_BYTES;
            uint4 kv[P::KPT];
#pragma unroll
            for (int i = 0; i < P::KPT; i++) {  // every load of the thread's pieces in flight, then the stores
                const int e = lt + i * PA_LOADERS * 32, r = e / (D / 8), pc = e % (D / 8);
                kv[i] = make_uint4(0u, 0u, 0u, 0u);
                if (e < PA_KT * (D / 8) && kb0 + r < n_keys)
                    kv[i] = *reinterpret_cast<const uint4*>(kbase + (size_t)(kb0 + r) * D + pc * 8);
            }
#pragma unroll
            for (int i = 0; i < P::KPT; i++) {
                const int e = lt + i * PA_LOADERS * 32, r = e / (D / 8), pc = e % (D / 8), hf = pc >> 3, p = pc & 7;
                if (e < PA_KT * (D / 8)) *reinterpret_cast<uint4*>(kt + hf * (PA_KT * 128) + sw128(r, p)) = kv[i];
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.kfull[ks]);
            if (seq < T) continue;
            // V of tile t: 8 x 8 blocks (keys 8a …, dims 8b …) transposed in registers into rows of the dims
            const int vs = t & 1;
            if (t >= 2 && !pa_wait(&sh.vempty[vs], ((t >> 1) - 1) & 1, abort_flag, err)) {
                ok = false;
                break;
            }
            uint8_t* vt = Vr + vs * P::V_BYTES;
            for (int e = lt; e < (PA_KT / 8) * (D / 8); e += PA_LOADERS * 32) {
                const int ka = e % (PA_KT / 8), b = e / (PA_KT / 8);
                uint32_t w[8][4];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int key = kb0 + 8 * ka + i;
                    uint4 x = make_uint4(0u, 0u, 0u, 0u);
                    if (key < n_keys) x = *reinterpret_cast<const uint4*>(vbase + (size_t)key * D + 8 * b);
                    w[i][0] = x.x, w[i][1] = x.y, w[i][2] = x.z, w[i][3] = x.w;
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;  // the high or the low half of each pair
                    const int wi = j >> 1;
                    const uint4 o = make_uint4(__byte_perm(w[0][wi], w[1][wi], sel), __byte_perm(w[2][wi], w[3][wi], sel),
                                               __byte_perm(w[4][wi], w[5][wi], sel), __byte_perm(w[6][wi], w[7][wi], sel));
                    *reinterpret_cast<uint4*>(vt + sw128(8 * b + j, ka)) = o;
                }
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.vfull[vs]);
        }
        if (!ok) *abort_flag = 1;
    } else if (warp == 4) {
        // ---- the tensor cores ----
        if (lane == 0) {
            const uint32_t idS = bg_idesc(PA_KT), idO = bg_idesc(P::VROWS);
            bool ok = true, any = false;
            // S[sq % 2] = Q K^T for the K tile of staging sequence `seq`
            auto qk = [&](int sq, int seq) -> bool {
                const int sb = sq & 1, ks = seq & 1;
                if (sq >= 2 && !pa_wait(&sh.sfree[sb], ((sq >> 1) - 1) & 1, abort_flag, err)) return false;
                if (!pa_wait(&sh.kfull[ks], (seq >> 1) & 1, abort_flag, err)) return false;
                tc_fence_after();
                const uint32_t qh = smem_u32(Qh), ql = smem_u32(Ql), kt = smem_u32(Kr + ks * P::K_BYTES);
#pragma unroll
                for (int k = 0; k < D / 16; k++) {  // 16 dims per step, 4 steps per 64-dim half
                    const uint32_t oq = (k >> 2) * (PA_QT * 128) + (k & 3) * 32;
                    const uint32_t ok_ = (k >> 2) * (PA_KT * 128) + (k & 3) * 32;
                    mma_f16(tS + sb * PA_KT, bg_desc(qh + oq), bg_desc(kt + ok_), idS, k > 0 ? 1u : 0u);
                    mma_f16(tS + sb * PA_KT, bg_desc(ql + oq), bg_desc(kt + ok_), idS, 1u);
                }
                mma_commit(&sh.sfull[sb]);
                mma_commit(&sh.kempty[ks]);
                any = true;
                return true;
            };
            // two passes (the row maxima, then P V): S of sequence number T + t is tile t's second product; the tiled
            // form makes one pass (sequence t = tile t)
            const int s0 = TILED ? 0 : T;
            if constexpr (!TILED)
                for (int t = 0; t < T && ok; t++) ok = qk(t, t);
            if (ok) ok = qk(s0, s0);
            for (int t = 0; t < T && ok; t++) {
                if (t + 1 < T && !(ok = qk(s0 + t + 1, s0 + t + 1))) break;  // the next tile's S while the rows read this
                const int vs = t & 1;
                if (!pa_wait(&sh.pfull, t & 1, abort_flag, err) ||
                    !pa_wait(&sh.vfull[vs], (t >> 1) & 1, abort_flag, err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ph = smem_u32(Ph), pl = smem_u32(Pl), vt = smem_u32(Vr + vs * P::V_BYTES);
#pragma unroll
                for (int k = 0; k < PA_KT / 16; k++) {
                    mma_f16(tO, bg_desc(ph + k * 32), bg_desc(vt + k * 32), idO, (t > 0 || k > 0) ? 1u : 0u);
                    if constexpr (!TILED) mma_f16(tO, bg_desc(pl + k * 32), bg_desc(vt + k * 32), idO, 1u);
                }
                mma_commit(&sh.pfree);
                mma_commit(&sh.vempty[vs]);
            }
            if (ok) mma_commit(&sh.ofull);
            if (any) {  // every MMA complete before the TMEM is freed (bounded, abort or not)
                mma_commit(&sh.mdone);
                mbar_wait(&sh.mdone, 0, err);
            }
        }
        __syncwarp();
    } else {
        // ---- the rows: thread tid owns query q0 + tid (TMEM lane tid) ----
        const int qpos = pos0 + q0 + tid;
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        float m = -INFINITY, l = 0.0f;
        uint32_t sv[PA_KT];
        bool ok = true;
        auto read_s = [&](int sq) -> bool {
            const int sb = sq & 1;
            if (!pa_wait(&sh.sfull[sb], (sq >> 1) & 1, abort_flag, err)) return false;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < PA_KT / 16; c++) tmem_ld16(tS + lane_base + sb * PA_KT + c * 16, sv + c * 16);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.sfree[sb]);
            return true;
        };
        if constexpr (TILED) {
            // one pass, online: m is the running maximum (log2 units); a tile whose maximum exceeds it by more than
            // PA_RESCALE rescales l and the row of O (after the previous P V completes) — otherwise p = 2^(s - m)
            // <= 2^PA_RESCALE stays in f16's range. P is rounded to f16 (the reference's f16 path rounds P so).
            for (int t = 0; t < T && ok; t++) {
                if (!(ok = read_s(t))) break;
                const bool edge = (t + 1) * PA_KT > n_keys;  // the last tile may hold keys past n_keys
                float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
                for (int j = 0; j < PA_KT; j++)
                    if (!edge || t * PA_KT + j < n_keys) mq[j & 3] = fmaxf(mq[j & 3], __uint_as_float(sv[j]));
                const float mt = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
                bool waited = false;
                if (t == 0) {
                    m = mt;
                } else if (__any_sync(FULL, mt > m + PA_RESCALE)) {
                    // (warp-uniform: the TMEM loads and stores are collective over the warp's 32 lanes; a row whose
                    // maximum did not move scales by 1)
                    if (!(ok = pa_wait(&sh.pfree, (t - 1) & 1, abort_flag, err))) break;  // P V of t - 1 done
                    waited = true;
                    const bool up = mt > m + PA_RESCALE;
                    const float f = up ? exp2f(m - mt) : 1.0f;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < P::VROWS / 16; c++) {  // (the row sum's column with O)
                        uint32_t o[16];
                        tmem_ld16(tO + lane_base + c * 16, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int d = 0; d < 16; d++) o[d] = __float_as_uint(__uint_as_float(o[d]) * f);
                        tmem_st16(tO + lane_base + c * 16, o);
                    }
                    tmem_wait_st();
                    if (up) m = mt;
                }
                uint32_t pk[PA_KT / 2];
#pragma unroll
                for (int j = 0; j < PA_KT; j += 2) {
                    float p0 = exp2f(__uint_as_float(sv[j]) - m), p1 = exp2f(__uint_as_float(sv[j + 1]) - m);
                    if (edge) {
                        if (t * PA_KT + j >= n_keys) p0 = 0.0f;
                        if (t * PA_KT + j + 1 >= n_keys) p1 = 0.0f;
                    }
                    pk[j >> 1] = pack_h2(p0, p1);  // (the row sum comes from the ones row of V^T)
                }
                if (t >= 1 && !waited && !(ok = pa_wait(&sh.pfree, (t - 1) & 1, abort_flag, err))) break;
#pragma unroll
                for (int p = 0; p < PA_KT / 8; p++)
                    *reinterpret_cast<uint4*>(Ph + sw128(tid, p)) =
                        make_uint4(pk[4 * p], pk[4 * p + 1], pk[4 * p + 2], pk[4 * p + 3]);
                tc_fence_before();    // (the rescaled O, before the tensor cores accumulate into it)
                fence_proxy_async();  // the generic stores, before the tensor cores read them
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.pfull);
            }
        }
        for (int t = 0; t < T && ok && !TILED; t++) {
            if (!(ok = read_s(t))) break;
#pragma unroll
            for (int j = 0; j < PA_KT; j++)
                if (CAUSAL ? t * PA_KT + j <= qpos : t * PA_KT + j < n_keys) m = fmaxf(m, __uint_as_float(sv[j]));
        }
        for (int t = 0; t < T && ok && !TILED; t++) {
            if (!(ok = read_s(T + t))) break;
            if (t >= 1 && !(ok = pa_wait(&sh.pfree, (t - 1) & 1, abort_flag, err))) break;  // P·V of t - 1 done
#pragma unroll
            for (int p = 0; p < PA_KT / 8; p++) {
                float pv[8], ph[8];
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const int j = p * 8 + c;
                    const bool seen = CAUSAL ? t * PA_KT + j <= qpos : t * PA_KT + j < n_keys;
                    pv[c] = seen ? expf(__uint_as_float(sv[j]) - m) : 0.0f;
                    l += pv[c];
                    ph[c] = __half2float(__float2half_rn(pv[c]));
                }
                const uint4 hi = make_uint4(pack_h2(ph[0], ph[1]), pack_h2(ph[2], ph[3]), pack_h2(ph[4], ph[5]),
                                            pack_h2(ph[6], ph[7]));
                const uint4 lo = make_uint4(pack_h2(pv[0] - ph[0], pv[1] - ph[1]), pack_h2(pv[2] - ph[2], pv[3] - ph[3]),
                                            pack_h2(pv[4] - ph[4], pv[5] - ph[5]), pack_h2(pv[6] - ph[6], pv[7] - ph[7]));
                *reinterpret_cast<uint4*>(Ph + sw128(tid, p)) = hi;
                *reinterpret_cast<uint4*>(Pl + sw128(tid, p)) = lo;
            }
            fence_proxy_async();  // the generic stores, before the tensor cores read them
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.pfull);
        }
        // the output row: O / sum, as f32 (out) and / or split f16 hi / lo into the next contraction's operand (out16)
        if (ok && pa_wait(&sh.ofull, 0, abort_flag, err)) {
            tc_fence_after();
            if constexpr (TILED) {  // the row sum of the rounded P, column D of the product
                uint32_t o[16];
                tmem_ld16(tO + lane_base + D, o);
                tmem_wait_ld();
                l = __uint_as_float(o[0]);
            }
            const float inv = 1.0f / l;
            const int row = q0 + tid;
            uint8_t* g16 = a.out16 ? a.out16 + (size_t)(row / BG_SLOTS) * x16_group_bytes(a.out16_K) : nullptr;
#pragma unroll
            for (int c = 0; c < D / 16; c++) {
                uint32_t o[16];
                tmem_ld16(tO + lane_base + c * 16, o);
                tmem_wait_ld();
                if (row < L) {
                    float y[16];
#pragma unroll
                    for (int d = 0; d < 16; d++) y[d] = __uint_as_float(o[d]) * inv;
                    if (a.out) {
                        float4* op = reinterpret_cast<float4*>(a.out + (size_t)row * a.out_stride + h * D + c * 16);
#pragma unroll
                        for (int d = 0; d < 4; d++) op[d] = make_float4(y[4 * d], y[4 * d + 1], y[4 * d + 2], y[4 * d + 3]);
                    }
                    if (g16) {
#pragma unroll
                        for (int hp = 0; hp < 2; hp++) {  // two 8-column pieces
                            float yh[8];
#pragma unroll
                            for (int d = 0; d < 8; d++) yh[d] = __half2float(__float2half_rn(y[8 * hp + d]));
                            const float* yy = y + 8 * hp;
                            const int col = h * D + c * 16 + 8 * hp, n = row % BG_SLOTS;
                            *reinterpret_cast<uint4*>(g16 + x16_offset(n, col)) =
                                make_uint4(pack_h2(yh[0], yh[1]), pack_h2(yh[2], yh[3]), pack_h2(yh[4], yh[5]),
                                           pack_h2(yh[6], yh[7]));
                            *reinterpret_cast<uint4*>(g16 + x16_offset(BG_SLOTS + n, col)) =
                                make_uint4(pack_h2(yy[0] - yh[0], yy[1] - yh[1]), pack_h2(yy[2] - yh[2], yy[3] - yh[3]),
                                           pack_h2(yy[4] - yh[4], yy[5] - yh[5]), pack_h2(yy[6] - yh[6], yy[7] - yh[7]));
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, PA_TMEM_COLS);
    }
}

template <int D, bool CAUSAL, bool TILED>
static void launch_tc(cudaStream_t st, const TcAttnArgs& a) {
    static PerDeviceOnce once;
    once([] {
        cudaFuncSetAttribute(k_attn_tc<D, CAUSAL, TILED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)PaPlan<D, TILED>::SMEM);
    });
    k_attn_tc<D, CAUSAL, TILED><<<dim3((a.L + PA_QT - 1) / PA_QT, a.n_head, 1), pa_threads(TILED),
                                  PaPlan<D, TILED>::SMEM, st>>>(a);
}

void launch_attention_prefill_tc(cudaStream_t st, const float* qkv, int L, int n_head, int n_kv, const __half* kc,
                                 const __half* vc, int n_ctx, int pos0, float scale, float* out, int* err) {
    TcAttnArgs a;
    a.q = qkv;
    a.q_stride = (n_head + 2 * n_kv) * 128;
    a.L = L;
    a.n_head = n_head;
    a.group = n_head / n_kv;
    a.k = kc;
    a.v = vc;
    a.kv_head_stride = (size_t)n_ctx * 128;
    a.pos0 = pos0;
    a.scale = scale;
    a.out = out;
    a.out_stride = n_head * 128;
    a.err = err;
    launch_tc<128, true, false>(st, a);
}

void launch_attention_full_tc(cudaStream_t st, const TcAttnArgs& a) { launch_tc<64, false, true>(st, a); }

}  // namespace ocr

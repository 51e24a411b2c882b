// k_bgemm.cu — the batched decode contraction on the 5th-generation tensor cores (tcgen05, sm_100a): the reference's
// q8_0 matvecs (shaders/dmv.wgsl, dmv_qkv.wgsl, dmv_ffn.wgsl, the LM head's dmv_norm) and its tiled GEMM
// (shaders/matmul128.wgsl, the `matmul` dispatch of app/crates/ocr-wgpu/src/gpu.rs:1967-2016) for a batch of decode
// slots, Y[slot][row] = sum_k W[row][k] x[slot][k], with the same epilogues as the CUDA-core matvec (store, residual
// add, SwiGLU over interleaved gate/up rows, the LM head's windowed penalty + first-maximum choice).
//
// Numerics. Each weight q * d (int8 times the block's f16 scale) is exact in f32 and splits exactly into two f16
// values, w_hi = RN_f16(q * d) (one HMUL2) and w_lo = RN_f16(q * d - w_hi) (one HFMA2 — the remainder has at most 8
// significant bits, so it is exact unless it falls below f16's normal range); each activation splits the same way,
// x_hi = RN_f16(x), x_lo = RN_f16(x - x_hi). tcgen05.mma kind::f16 multiplies f16 pairs exactly and accumulates in f32,
// so D = w_hi x_hi + w_hi x_lo + w_lo x_hi carries the f32 matvec's result to within f32 rounding; the dropped w_lo x_lo
// is below 2^-22 of each product.
//
// Work items are 128-row tiles of W — or, for a matrix of few tiles, a tile's share of its 128-column chunks (split-K:
// every split writes its f32 partial, and the tile's last split to finish, by ticket, sums the partials in split order
// and runs the epilogue: deterministic, no waiting). One CTA per SM, persistent over items (item w, w + grid, …), 576
// threads in three roles:
//  - warp 0 (one lane), the copies: per 128-column chunk of K, one bulk copy of the tile's block of the tile-major
//    weight copy (16 KB of quants, already swizzled, + their 1 KB of block scales: one contiguous run, so the DRAM reads
//    stream) and one of the slots' activation chunk (16 KB, already in the MMA operand order), both counted on the
//    stage's mbarrier. The weights of the first stages are issued before griddepcontrol.wait (they never depend on the
//    previous kernel).
//  - warps 2-17, the dequantisation: per 64-column piece (one 16-weight item per thread), int8 -> f16 hi / lo (byte permute into 1024 + q + 128's
//    mantissa, one HSUB2, one HMUL2, one HFMA2 per pair) into one of 2 to 4 A operand buffers in the 128-byte-swizzle
//    K-major layout the tensor cores read without bank conflicts; then, per work item, the epilogue: tcgen05.ld of
//    their TMEM lanes, hi + lo columns summed, the mode's output.
//  - warp 1, the tensor cores: TMEM allocation (all 512 columns: 4 accumulator sets), and per 16-column step two MMAs
//    (M = 128) into one set — A = w_hi with B = [x_hi | x_lo] (N = 64) into its columns 0-63, A = w_lo with B = x_hi
//    (N = 32) into 64-95 — consecutive steps rotating over the sets, so four chains of dependent MMAs run side by side
//    (one chain of these small-N MMAs is bound by the accumulator's latency); tcgen05.commit releases the operand
//    buffer, the copy stage, and at an item's end the accumulators to the epilogue, which sums the sets in order.
// Every mbarrier wait is bounded; a wait that runs out sets the device error flag and a shared abort flag that every
// role polls; the copies in flight and the MMAs issued are then waited for (bounded) and the TMEM is freed before the
// CTA exits.
#include "choice.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace ocr {

constexpr int BG_M = 128;       // weight rows per tile: the MMA's M, one TMEM lane each
constexpr int BG_KC = 128;      // K columns per copy stage
constexpr int BG_KS = 64;       // K columns per dequantised operand buffer (one 128-byte swizzle atom wide)
constexpr int BG_THREADS = 576;
constexpr int BG_DQ = 512;      // dequantisation / epilogue threads (warps 2-17)
constexpr int BG_DW = BG_DQ / 32;  // their warps: 4 per TMEM lane quarter, 8 slots each
constexpr uint32_t BG_WTILE = BG_TILE_BYTES;                // a tile-major block: 16 KB of int8 quants + 1 KB of scales
constexpr uint32_t BG_AHALF = BG_M * BG_KS * 2;             // 16 KB: the hi (or lo) f16 operand of a 64-column piece
constexpr uint32_t BG_ABUF = 2 * BG_AHALF;
constexpr int BG_NA = 4;        // operand buffers at most (2 to 4, as shared memory allows)
constexpr int BG_MAX_NS = 4;    // copy stages
constexpr int BG_NACC = 4;            // accumulator sets the K steps rotate over (independent MMA chains)
constexpr uint32_t BG_SET_COLS = 128;  // a set: w_hi [x_hi | x_lo] in columns 0-63, w_lo x_hi in 64-95
constexpr uint32_t BG_TMEM_COLS = BG_NACC * BG_SET_COLS;  // all 512 columns (one CTA per SM)
constexpr int BG_SMEM_OPTIN = 227 * 1024;

// a bounded wait that also gives up when another role of the CTA has given up (`abort_flag`)
__device__ __forceinline__ bool bg_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
    for (uint32_t i = 0; i < MBAR_TRIES; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    dev_error(err, DEV_TIMEOUT);
    return false;
}

// 16 int8 quants and their f16 block scale → 8 half2 of w_hi and 8 of w_lo (w_hi + w_lo = q * d exactly)
__device__ __forceinline__ void dequant16(uint4 q, __half d, uint32_t* hi, uint32_t* lo) {
    const __half2 d2 = __half2half2(d);
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152 = 1024 + 128
    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        // 0x64bb as f16 is 1024 + bb exactly: bytes (q + 128) below the 0x64 exponent byte
        uint32_t p01 = __byte_perm(w[k], 0x64646464u, 0x5140), p23 = __byte_perm(w[k], 0x64646464u, 0x5342);
        const __half2 q01 = __hsub2(*reinterpret_cast<__half2*>(&p01), bias);
        const __half2 q23 = __hsub2(*reinterpret_cast<__half2*>(&p23), bias);
        const __half2 h01 = __hmul2(q01, d2), h23 = __hmul2(q23, d2);
        const __half2 l01 = __hfma2(q01, d2, __hneg2(h01)), l23 = __hfma2(q23, d2, __hneg2(h23));
        hi[2 * k] = *reinterpret_cast<const uint32_t*>(&h01);
        hi[2 * k + 1] = *reinterpret_cast<const uint32_t*>(&h23);
        lo[2 * k] = *reinterpret_cast<const uint32_t*>(&l01);
        lo[2 * k + 1] = *reinterpret_cast<const uint32_t*>(&l23);
    }
}

struct BgShared {
    uint64_t wfull[BG_MAX_NS], xfull[BG_MAX_NS];  // a copy stage's weights / activations landed
    uint64_t tempty[BG_MAX_NS];                    // the stage free again (its MMAs done)
    uint64_t afull[BG_NA], aempty[BG_NA];          // operand buffer written / free again
    uint64_t tfin, mdone;                          // an item's accumulator complete; every MMA done (exit)
    uint32_t tmem_base;
    int abort_flag;
    uint32_t ticket;                      // split items: this CTA's place among the tile's splits
    uint32_t pbits[BG_SLOTS][BG_M / 32];  // LM head: the tile's rows in each slot's penalty window
    float bvq[BG_DW][8];                  // LM head: each epilogue warp's best per slot
    uint32_t biq[BG_DW][8];
    float bv[BG_SLOTS];
    uint32_t bi[BG_SLOTS];
    float ssq[4][BG_SLOTS];  // MV_ADD with ssq_out: the tile's sums of squares per TMEM lane quarter and slot
};

// Work items: item w is (tile w / ksplit, split w % ksplit); a split covers chunks [c0, c1) of the K/128 chunks.
// A CTA takes items blockIdx.x, blockIdx.x + gridDim.x, … (the LM head: every tile, one split).
struct BgItem {
    int t, sp, c0, c1;
};
__device__ __forceinline__ BgItem bg_item(int w, int ksplit, int nkc) {
    BgItem it;
    it.t = w / ksplit;
    it.sp = w % ksplit;
    it.c0 = (int)((long)nkc * it.sp / ksplit);
    it.c1 = (int)((long)nkc * (it.sp + 1) / ksplit);
    return it;
}

// One instance per epilogue mode (MODE = a.mode) and operand source (XN: built from the residual, a.xn; else copied
// from x16): each launch runs only its own code, which keeps the warps' instruction fetches in cache (a single kernel
// holding every epilogue stalled its warps on instruction fetch more than on anything else).
// (18 warps: 5 on two of the SM's four sub-partitions, whose 16K registers each cap a thread at 96)
// NG: groups of 32 slots (rows of the activations) per CTA. Two for long prefills: each dequantised weight piece
// then feeds the MMAs of both groups (2 accumulator sets each), halving the dequantisation per row; one item per CTA
// pass, no split-K (the host picks it only for unsplit launches over more than one group).
// Three ("merged", for thousands of rows: the vision encoder): the three groups' activation halves land side by side
// in the stage (64 columns: g0 hi, g0 lo, g1 hi, … — 192 rows of 128 bytes), so one K step is two MMAs of N = 192,
// A = w_hi then A = w_lo into the same accumulator (w x_hi and w x_lo per group: the w_lo x_lo term, below 2^-22 of
// the product, is kept rather than dropped), over two accumulator sets of 192 columns.
template <int MODE, bool XN, int NG = 1>
__global__ void __launch_bounds__(BG_THREADS, 1)
    k_bgemm(const __grid_constant__ BgArgs a, const uint8_t* __restrict__ wtiles, int ns, int na) {
    static_assert(NG == 1 || (NG <= 3 && !XN && MODE != MV_LMHEAD), "several groups: plain operands, no LM head");
    constexpr bool MERGED = NG == 3;
    constexpr uint32_t STAGE = BG_WTILE + NG * BG_CHUNK_BYTES;  // weights + each group's activation chunk
    constexpr int NSET = MERGED ? 2 : BG_NACC / NG;                // accumulator sets (per group, unless merged)
    constexpr uint32_t MSET = 64u * NG;                            // a merged set's columns
    extern __shared__ uint8_t sm_raw[];
    __shared__ __align__(16) BgShared sh;
    volatile int* abort_flag = &sh.abort_flag;
    const unsigned long long t_start = a.tl ? gtimer() : 0ull;
    unsigned long long t_dep = 0ull;

    const int K = a.w.cols, N = a.w.rows;
    const int nkc = K / BG_KC, ksplit = a.ksplit;
    // the dynamic region starts 1024-B aligned (the 128-B swizzle's pattern repeats every 1024 B)
    uint8_t* smp = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
    uint8_t* stage0 = smp;
    uint8_t* abuf0 = smp + (size_t)ns * STAGE;
    const int n_tiles = (N + BG_M - 1) / BG_M, n_items = n_tiles * ksplit;
    // this CTA's groups grp … grp + ngr - 1 (slot0 / nb: the first group's)
    const int grp = blockIdx.y * NG, ngr = min(NG, (a.nb + BG_SLOTS - 1) / BG_SLOTS - grp);
    const int slot0 = grp * BG_SLOTS, nb = min(BG_SLOTS, a.nb - slot0);
    const uint8_t* xg = a.x16 + (size_t)grp * nkc * BG_CHUNK_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool lmhead = MODE == MV_LMHEAD;
    // the in-kernel operand needs one item per CTA whose chunks fit the stages (the host checks; a launch that breaks
    // it is refused here, before any barrier or TMEM)
    if (XN && (n_items > (int)gridDim.x || (nkc + ksplit - 1) / ksplit > ns)) {
        if (threadIdx.x == 0 && blockIdx.x == 0) dev_error(a.err, DEV_BAD_INDEX);
        return;
    }

    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; i++) {
            mbar_init(&sh.wfull[i], 1);
            mbar_init(&sh.xfull[i], XN ? BG_DW : 1);  // the copy's bytes, or each operand-building warp
            mbar_init(&sh.tempty[i], 1);
        }
        for (int i = 0; i < na; i++) {
            mbar_init(&sh.afull[i], BG_DQ / 32);
            mbar_init(&sh.aempty[i], 1);
        }
        mbar_init(&sh.tfin, 1);
        mbar_init(&sh.mdone, 1);
        sh.abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(&sh.tmem_base, BG_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;

    if (warp == 0) {
        // ---- the copies: lane 0 waits and arms, the warp's lanes issue 4 KB pieces (the copy engine works on many at
        // once; one long copy per stage drains slowly) ----
        const uint64_t pol = l2_evict_first();
        uint32_t g = 0;
        int pre = 0;
        const int w0 = blockIdx.x;
        auto wblock = [&](int t, int kc) { return wtiles + ((size_t)t * nkc + kc) * BG_TILE_BYTES; };
        if (w0 < n_items) {
            // before the dependency wait: the weight blocks of the first item's first stages
            const BgItem it = bg_item(w0, ksplit, nkc);
            pre = min(ns, it.c1 - it.c0);
            for (int s = 0; s < pre; s++) {
                if (lane == 0) mbar_expect_tx(&sh.wfull[s], BG_WTILE);
                __syncwarp();
                bulk_g2s_lanes(stage0 + (size_t)s * STAGE, wblock(it.t, it.c0 + s), BG_WTILE, &sh.wfull[s], pol,
                               lane, 32);
            }
        }
        if (lane == 0) pdl_trigger();
        pdl_wait();
        if (threadIdx.x == 0 && a.tl) t_dep = gtimer();
        bool ok = true;
        for (int w = w0; w < n_items && ok; w += gridDim.x) {
            const BgItem it = bg_item(w, ksplit, nkc);
            for (int kc = it.c0; kc < it.c1; kc++, g++) {
                const int s = (int)(g % (uint32_t)ns);
                uint8_t* st = stage0 + (size_t)s * STAGE;
                if (g >= (uint32_t)pre) {  // (the prologue issued the weights of the first `pre` stages)
                    const bool got = g < (uint32_t)ns ||
                                     (lane == 0 ? bg_wait(&sh.tempty[s], ((g / ns) - 1) & 1, abort_flag, a.err) : true);
                    if (!__all_sync(FULL, got)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) mbar_expect_tx(&sh.wfull[s], BG_WTILE);
                    __syncwarp();
                    bulk_g2s_lanes(st, wblock(it.t, kc), BG_WTILE, &sh.wfull[s], pol, lane, 32);
                }
                if (XN) continue;  // (the operand is built by warps 2-17)
                if (lane == 0) mbar_expect_tx(&sh.xfull[s], (uint32_t)ngr * BG_CHUNK_BYTES);
                __syncwarp();
                for (int gi = 0; gi < ngr; gi++) {
                    const uint8_t* src = xg + ((size_t)gi * nkc + kc) * BG_CHUNK_BYTES;
                    if (MERGED) {  // half h of group gi at h x (NG x 8 KB) + gi x 8 KB
                        for (int h = 0; h < 2; h++)
                            bulk_g2s_lanes(st + BG_WTILE + h * (NG * 8192) + gi * 8192, src + h * 8192, 8192,
                                           &sh.xfull[s], 0ull, lane, 32);
                    } else {
                        bulk_g2s_lanes(st + BG_WTILE + gi * BG_CHUNK_BYTES, src, BG_CHUNK_BYTES, &sh.xfull[s], 0ull,
                                       lane, 32);
                    }
                }
            }
        }
        // every copy issued lands before the CTA can exit (in a normal run these phases are long complete): the
        // weights of stages [0, max(g, pre)), the activations of [0, g); a stage's last phase is the only one that
        // can be incomplete (each reuse waited for the one before)
        if (lane == 0) {
            const uint32_t wi = max(g, (uint32_t)pre);
            for (int s = 0; s < ns; s++) {
                if ((uint32_t)s < wi) mbar_wait(&sh.wfull[s], (((wi - s + ns - 1) / ns) - 1) & 1, a.err);
                if ((uint32_t)s < g && !XN) mbar_wait(&sh.xfull[s], (((g - s + ns - 1) / ns) - 1) & 1, a.err);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- the tensor cores ----
        if (lane == 0) {
            const uint32_t id1 = bg_idesc(64), id2 = bg_idesc(32), idm = bg_idesc((int)MSET);
            uint32_t g = 0, ai = 0;
            bool any = false, ok = true;
            for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
                const BgItem it = bg_item(w, ksplit, nkc);
                for (int kc = it.c0; kc < it.c1 && ok; kc++, g++) {
                    const int s = (int)(g % (uint32_t)ns);
                    if (!bg_wait(&sh.xfull[s], (g / ns) & 1, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t xs = smem_u32(stage0 + (size_t)s * STAGE + BG_WTILE);
                    const int kstep0 = (kc - it.c0) * (BG_KC / 16);  // the item's K steps so far
                    for (int h = 0; h < BG_KC / BG_KS; h++, ai++) {
                        const int ab = (int)(ai % na);
                        if (!bg_wait(&sh.afull[ab], (ai / na) & 1, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t ah = smem_u32(abuf0 + (size_t)ab * BG_ABUF), al = ah + BG_AHALF;
#pragma unroll
                        for (int ks = 0; ks < BG_KS / 16; ks++) {
                            // 16 columns = 32 bytes into the swizzle atoms: A's 128 rows, B's 64 rows (half h)
                            const uint64_t dh = bg_desc(ah + ks * 32);
                            const uint64_t dl = bg_desc(al + ks * 32);
                            // consecutive K steps go to independent accumulator sets (the MMAs of one set depend
                            // on each other; of different sets, not); a set's first step overwrites it. Group gi
                            // (its activation chunk gi x 16 KB into the stage) owns sets gi x NSET …
                            const int kstep = kstep0 + h * (BG_KS / 16) + ks;
                            const uint32_t acc = kstep >= NSET ? 1u : 0u;
                            if constexpr (MERGED) {
                                const uint64_t db = bg_desc(xs + h * (NG * 8192) + ks * 32);
                                const uint32_t dset = tmem + (uint32_t)(kstep % NSET) * MSET;
                                mma_f16(dset, dh, db, idm, acc);
                                mma_f16(dset, dl, db, idm, 1u);
                                continue;
                            }
#pragma unroll
                            for (int gi = 0; gi < NG; gi++) {
                                if (gi >= ngr) break;
                                const uint64_t db = bg_desc(xs + gi * BG_CHUNK_BYTES + h * 8192 + ks * 32);
                                const uint32_t dset = tmem + (uint32_t)(gi * NSET + kstep % NSET) * BG_SET_COLS;
                                mma_f16(dset, dh, db, id1, acc);
                                mma_f16(dset + 64, dl, db, id2, acc);
                            }
                        }
                        mma_commit(&sh.aempty[ab]);
                        any = true;
                    }
                    if (ok) mma_commit(&sh.tempty[s]);
                }
                if (ok) mma_commit(&sh.tfin);
            }
            if (any) {  // every MMA complete before the accumulator is freed (bounded, abort or not)
                mma_commit(&sh.mdone);
                mbar_wait(&sh.mdone, 0, a.err);
            }
        }
        __syncwarp();
    }

    // ---- dequantisation and epilogue (warps 2-17) ----
    const int et = (int)threadIdx.x - 64, dw = warp - 2;
    const int q = warp & 3, part = dw >> 2;  // the TMEM lane quarter this warp may read; its 8 slots 8 part …
    float best_v[8];
    uint32_t best_i[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        best_v[j] = -INFINITY;
        best_i[j] = NO_INDEX;
    }
    if (warp >= 2) {
        // The weights never depend on the previous kernel: the dequantisation of the first stages runs while it
        // finishes. Everything the previous kernels write (the slots' states, the outputs this epilogue reads or
        // adds to) is read after griddepcontrol.wait, at the first item's epilogue.
        bool act[8] = {};
        // this thread's item of every 64-column piece: row 8 rg + r8, 16 columns c4; a quarter-warp takes 8 rows of one
        // 16-column piece — its reads through the copy's swizzle and its writes through the operand's (pieces 2 c4 and
        // 2 c4 + 1 of a row at (piece ^ row % 8)) are both conflict-free
        const int r8 = et & 7, c4 = (et >> 3) & 3, rg = et >> 5, drow = rg * 8 + r8;
        const int o0 = drow * 128 + (((2 * c4) ^ r8) << 4), o1 = drow * 128 + (((2 * c4 + 1) ^ r8) << 4);

        // A warp whose wait gave up (ok = false) still walks every loop, skipping waits and work, so that all sixteen
        // warps meet each named barrier of the epilogue the same number of times.
        // The normalised operand built here (a.xn; one item per CTA, its chunk c in stage c - c0): after the
        // dependency wait, each thread takes slot et / 16's 8 columns (et % 16) of every chunk: the residual row
        // times 1 / sqrt(mean of squares + eps) (the sums of squares over the row's 128-column tiles added in tile
        // order) times the norm weights, split f16 hi / lo into the stage's operand region, as the operand copy would
        // have landed it.
        bool xbuilt = !XN;
        auto build_x = [&](const BgItem& it) {
            pdl_wait();
            const int n = et >> 4, pc = et & 15, b = slot0 + n;
            const bool live = n < nb && (!a.active || a.active[b] != 0);
            float scale = 0.0f;
            if (live) {
                float tot = 0.0f;
                for (int t = 0; t < K / BG_KC; t++) tot += a.ssq_in[(size_t)t * a.nb + b];
                scale = 1.0f / sqrtf(tot / (float)K + a.eps);
            }
            for (int kc = it.c0; kc < it.c1; kc++) {
                const int s = kc - it.c0, k0 = kc * BG_KC + pc * 8;
                uint8_t* xs = stage0 + (size_t)s * STAGE + BG_WTILE;
                uint32_t hi[4] = {0u, 0u, 0u, 0u}, lo[4] = {0u, 0u, 0u, 0u};
                if (live) {
                    const float2* xr = reinterpret_cast<const float2*>(a.xn + (size_t)b * K + k0);
                    const float2* wr = reinterpret_cast<const float2*>(a.nw + k0);
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const float2 xv = xr[c], wv = wr[c];
                        const float v0 = xv.x * scale * wv.x, v1 = xv.y * scale * wv.y;
                        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
                        const __half l0 = __float2half_rn(v0 - __half2float(h0));
                        const __half l1 = __float2half_rn(v1 - __half2float(h1));
                        const __half2 hh = __halves2half2(h0, h1), ll = __halves2half2(l0, l1);
                        hi[c] = *reinterpret_cast<const uint32_t*>(&hh);
                        lo[c] = *reinterpret_cast<const uint32_t*>(&ll);
                    }
                }
                *reinterpret_cast<uint4*>(xs + x16_offset(n, pc * 8)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(xs + x16_offset(BG_SLOTS + n, pc * 8)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.xfull[s]);
            }
        };
        uint32_t g = 0, ai = 0;
        int li = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_items; w += gridDim.x, li++) {
            const BgItem it = bg_item(w, ksplit, nkc);
            for (int kc = it.c0; kc < it.c1; kc++, g++) {
                const int s = (int)(g % (uint32_t)ns);
                ok = ok && bg_wait(&sh.wfull[s], (g / ns) & 1, abort_flag, a.err);
                const uint8_t* wt = stage0 + (size_t)s * STAGE + drow * 128;
                const __half* sc = reinterpret_cast<const __half*>(stage0 + (size_t)s * STAGE + 16384 + drow * 8);
                for (int h = 0; h < BG_KC / BG_KS; h++, ai++) {
                    const int ab = (int)(ai % na);
                    // (one call site: before the first piece that waits for the tensor cores, or the item's last)
                    if (!xbuilt && (ai >= (uint32_t)na || (kc == it.c1 - 1 && h == BG_KC / BG_KS - 1))) {
                        build_x(it);
                        xbuilt = true;
                    }
                    ok = ok && (ai < (uint32_t)na || bg_wait(&sh.aempty[ab], ((ai / na) - 1) & 1, abort_flag, a.err));
                    if (!ok) continue;
                    uint8_t* ah = abuf0 + (size_t)ab * BG_ABUF;
                    const uint4 qv = *reinterpret_cast<const uint4*>(wt + (((h * 4 + c4) ^ r8) << 4));
                    const __half d = sc[(h * BG_KS + c4 * 16) >> 5];
                    uint32_t hi[8], lo[8];
                    dequant16(qv, d, hi, lo);
                    *reinterpret_cast<uint4*>(ah + o0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4*>(ah + o1) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    *reinterpret_cast<uint4*>(ah + BG_AHALF + o0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4*>(ah + BG_AHALF + o1) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                    fence_proxy_async();  // the generic stores, before the tensor cores read them
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sh.afull[ab]);
                }
            }

            // ---- the item's epilogue ----
            if (li == 0) {
                pdl_wait();
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int sl = 8 * part + j;
                    act[j] = sl < nb && (!a.active || a.active[slot0 + sl] != 0);
                }
            }
            const int r0 = it.t * BG_M, row = r0 + 32 * q + lane;
            if (lmhead && a.lm.sample && a.lm.rp != 1.0f) {  // (compiled in the LM head's instance only)
                // the window's tokens that fall in this tile, per slot (the epilogue threads, barrier 2)
                uint32_t* pb = &sh.pbits[0][0];
                for (int i = et; i < BG_SLOTS * (BG_M / 32); i += BG_DQ) pb[i] = 0u;
                bar_sync(2, BG_DQ);
                const int sl = et >> 4, pt = et & 15, b = slot0 + sl;
                if (sl < nb && (!a.active || a.active[b])) {
                    const int len = a.lm.len[b];
                    const int32_t* hst = a.lm.hist + (long)b * a.lm.hist_cap;
                    for (int jj = len - min(len, a.lm.window) + pt; jj < len; jj += 16) {
                        const int tk = hst[jj];
                        if (tk >= r0 && tk < r0 + BG_M) atomicOr(&sh.pbits[sl][(tk - r0) >> 5], 1u << ((tk - r0) & 31));
                    }
                }
                bar_sync(2, BG_DQ);
            }
            if constexpr (NG > 1) {
                // each group's sets summed in order, then its store / residual add / SwiGLU (no split, no LM head)
                ok = ok && bg_wait(&sh.tfin, li & 1, abort_flag, a.err);
                if (ok) tc_fence_after();
                for (int gi = 0; gi < ngr; gi++) {
                    float y[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) y[j] = 0.0f;
                    if (ok) {
#pragma unroll
                        for (int st = 0; st < NSET; st++) {
                            if constexpr (MERGED) {  // group gi: w x_hi in columns gi x 64 …, w x_lo 32 further
                                uint32_t rh[8], rl[8];
                                const uint32_t ta =
                                    tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)st * MSET + (uint32_t)gi * 64;
                                tmem_ld8(ta + 8 * part, rh);
                                tmem_ld8(ta + 32 + 8 * part, rl);
                                tmem_wait_ld();
#pragma unroll
                                for (int j = 0; j < 8; j++) y[j] += __uint_as_float(rh[j]) + __uint_as_float(rl[j]);
                                continue;
                            }
                            uint32_t rh[8], rl[8], rw[8];
                            const uint32_t ta =
                                tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(gi * NSET + st) * BG_SET_COLS;
                            tmem_ld8(ta + 8 * part, rh);
                            tmem_ld8(ta + 32 + 8 * part, rl);
                            tmem_ld8(ta + 64 + 8 * part, rw);
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 8; j++)
                                y[j] += (__uint_as_float(rh[j]) + __uint_as_float(rw[j])) + __uint_as_float(rl[j]);
                        }
                    }
                    if (!ok) continue;
                    const int sl0 = (grp + gi) * BG_SLOTS, nbg = min(BG_SLOTS, a.nb - sl0);
                    bool ag[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int sl = 8 * part + j;
                        ag[j] = sl < nbg && (!a.active || a.active[sl0 + sl] != 0);
                    }
                    if (MODE == MV_SWIGLU) {
                        const int col = row >> 1;
                        uint8_t* y16 = a.y16 ? a.y16 + (size_t)(grp + gi) * x16_group_bytes(N / 2) : nullptr;
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const float up = __shfl_xor_sync(FULL, y[j], 1);
                            const int sl = 8 * part + j;
                            if ((lane & 1) || !ag[j] || row >= N) continue;
                            const float gv = y[j];
                            const float hv = gv / (1.0f + expf(-gv)) * up;
                            if (a.y) a.y[(long)(sl0 + sl) * a.y_stride + col] = hv;
                            if (y16) {
                                const __half hh = __float2half_rn(hv);
                                const __half hl = __float2half_rn(hv - __half2float(hh));
                                *reinterpret_cast<__half*>(y16 + x16_offset(sl, col)) = hh;
                                *reinterpret_cast<__half*>(y16 + x16_offset(BG_SLOTS + sl, col)) = hl;
                            }
                        }
                    } else if (row < N) {
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            if (!ag[j]) continue;
                            float* yp = a.y + (long)(sl0 + 8 * part + j) * a.y_stride + row;
                            *yp = MODE == MV_ADD ? *yp + y[j] : y[j];
                        }
                    }
                }
                tc_fence_before();  // these reads, before the next item's MMAs overwrite the accumulators
                continue;
            }
            ok = ok && bg_wait(&sh.tfin, li & 1, abort_flag, a.err);
            float y[8];
#pragma unroll
            for (int j = 0; j < 8; j++) y[j] = 0.0f;
            if (ok) {
                // the sets summed in order, each as w_hi x_hi + w_hi x_lo + w_lo x_hi
                tc_fence_after();
#pragma unroll
                for (int st = 0; st < BG_NACC; st++) {
                    uint32_t rh[8], rl[8], rw[8];
                    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)st * BG_SET_COLS;
                    tmem_ld8(ta + 8 * part, rh);
                    tmem_ld8(ta + 32 + 8 * part, rl);
                    tmem_ld8(ta + 64 + 8 * part, rw);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        y[j] += (__uint_as_float(rh[j]) + __uint_as_float(rw[j])) + __uint_as_float(rl[j]);
                }
            }
            tc_fence_before();  // these reads, before the next item's MMAs overwrite the accumulator
            if (ksplit > 1) {
                // this split's share → the tile's partials [group][tile][split][32 slots][128 rows]; the last split
                // of the tile to arrive (ticket; no waiting) sums them in split order and runs the epilogue
                float* pt = a.part + (((size_t)grp * n_tiles + it.t) * ksplit) * (BG_SLOTS * BG_M);
#pragma unroll
                for (int j = 0; j < 8; j++) pt[(size_t)it.sp * BG_SLOTS * BG_M + (8 * part + j) * BG_M + 32 * q + lane] = y[j];
                __threadfence();
                bar_sync(2, BG_DQ);
                if (et == 0) sh.ticket = atomicAdd(&a.tickets[grp * n_tiles + it.t], 1u);
                bar_sync(2, BG_DQ);
                if (sh.ticket != (uint32_t)ksplit - 1) continue;  // (uniform over the epilogue warps)
                __threadfence();
                // the partials summed in split order, 0 + p_0 + p_1 + …; the loads of four splits (32 values) are in
                // flight together, so the sum waits for ksplit / 4 round trips to L2 rather than one per load
                const float* pe = pt + (8 * part) * BG_M + 32 * q + lane;
#pragma unroll
                for (int j = 0; j < 8; j++) y[j] = 0.0f;
                int r = 0;
                for (; r + 4 <= ksplit; r += 4) {
                    float v[4][8];
#pragma unroll
                    for (int u = 0; u < 4; u++)
#pragma unroll
                        for (int j = 0; j < 8; j++) v[u][j] = __ldcg(pe + (size_t)(r + u) * BG_SLOTS * BG_M + j * BG_M);
#pragma unroll
                    for (int u = 0; u < 4; u++)
#pragma unroll
                        for (int j = 0; j < 8; j++) y[j] += v[u][j];
                }
                for (; r < ksplit; r++) {
                    float v[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) v[j] = __ldcg(pe + (size_t)r * BG_SLOTS * BG_M + j * BG_M);
#pragma unroll
                    for (int j = 0; j < 8; j++) y[j] += v[j];
                }
                if (et == 0) a.tickets[grp * n_tiles + it.t] = 0u;  // (self-resetting for the next launch)
            }
            if (MODE == MV_ADD && a.ssq_out) {
                // the residual add, then its rows' sums of squares per slot for the next norm: the warp's 32 rows,
                // the tile's 4 lane quarters added in order (every warp meets the barriers, ok or not)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    float sq = 0.0f;
                    if (ok && act[j] && row < N) {
                        float* yp = a.y + (long)(slot0 + 8 * part + j) * a.y_stride + row;
                        const float v = MODE == MV_ADD ? *yp + y[j] : y[j];
                        *yp = v;
                        sq = v * v;
                    }
                    sq = warp_sum(sq);
                    if (lane == 0) sh.ssq[q][8 * part + j] = sq;
                }
                bar_sync(2, BG_DQ);
                if (et < nb) a.ssq_out[(size_t)it.t * a.nb + slot0 + et] = ((sh.ssq[0][et] + sh.ssq[1][et]) + sh.ssq[2][et]) + sh.ssq[3][et];
                bar_sync(2, BG_DQ);
                continue;
            }
            if (!ok) continue;
            if (MODE == MV_SWIGLU) {
                // rows interleaved (gate, up): the even lane of each pair writes silu(gate) * up
                const int col = row >> 1;
                uint8_t* y16 = a.y16 ? a.y16 + (size_t)grp * x16_group_bytes(N / 2) : nullptr;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float up = __shfl_xor_sync(FULL, y[j], 1);
                    const int sl = 8 * part + j;
                    if ((lane & 1) || !act[j] || row >= N) continue;
                    const float gv = y[j];
                    const float hv = gv / (1.0f + expf(-gv)) * up;
                    if (a.y) a.y[(long)(slot0 + sl) * a.y_stride + col] = hv;
                    if (y16) {
                        const __half hh = __float2half_rn(hv);
                        const __half hl = __float2half_rn(hv - __half2float(hh));
                        *reinterpret_cast<__half*>(y16 + x16_offset(sl, col)) = hh;
                        *reinterpret_cast<__half*>(y16 + x16_offset(BG_SLOTS + sl, col)) = hl;
                    }
                }
            } else if (!lmhead) {
                if (row < N) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (!act[j]) continue;
                        float* yp = a.y + (long)(slot0 + 8 * part + j) * a.y_stride + row;
                        *yp = MODE == MV_ADD ? *yp + y[j] : y[j];
                    }
                }
            } else if (row < N) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (!act[j]) continue;
                    const int sl = 8 * part + j, b = slot0 + sl;
                    if (a.y) a.y[(long)b * N + row] = y[j];
                    if (a.lm.sample) {
                        const bool member = (sh.pbits[sl][q] >> lane) & 1u;
                        const float v = pen_value(y[j], member, b, row, a.lm, N);
                        if (row == 0) reinterpret_cast<int*>(a.lm.part + (long)a.lm.nb * gridDim.x * 2)[b] = (v != v);
                        if (better(v, (uint32_t)row, best_v[j], best_i[j])) {
                            best_v[j] = v;
                            best_i[j] = (uint32_t)row;
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, BG_TMEM_COLS);
    }
    if (!lmhead || !a.lm.sample) {  // (uniform over the grid)
        if (threadIdx.x == 0) tl_record(a.tl, t_start, t_dep);
        return;
    }
    // ---- the LM head's choice: each slot's best over the CTA's tiles, then the last CTA picks ----
    if (warp >= 2) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float v = best_v[j];
            uint32_t i = best_i[j];
            warp_argmax(v, i);
            if (lane == 0) {
                sh.bvq[dw][j] = v;
                sh.biq[dw][j] = i;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < BG_SLOTS) {
        // slot sl's 8-slot part is taken by the four warps of that part (one per TMEM lane quarter)
        const int sl = threadIdx.x, pp = sl >> 3, j = sl & 7;
        float v = -INFINITY;
        uint32_t i = NO_INDEX;
        for (int w = 4 * pp; w < 4 * pp + 4; w++)
            if (better(sh.bvq[w][j], sh.biq[w][j], v, i)) {
                v = sh.bvq[w][j];
                i = sh.biq[w][j];
            }
        sh.bv[sl] = v;
        sh.bi[sl] = i;
    }
    __syncthreads();
    choice_finish(sh.bv, sh.bi, nb, slot0, a.lm, N);
    if (threadIdx.x == 0) tl_record(a.tl, t_start, t_dep);
}

// ---- the activations' operand: per slot, sum, norm, hi / lo split ---------------------------------------------------
constexpr int XP_THREADS = 256;

__global__ void __launch_bounds__(XP_THREADS) k_xprep(PrepArgs a) {
    __shared__ float red[XP_THREADS / 32];
    const int b = blockIdx.x, K = a.K, n = b % BG_SLOTS;
    uint8_t* xg = a.x16 + (size_t)(b / BG_SLOTS) * x16_group_bytes(K);
    const unsigned long long t_start = a.tl ? gtimer() : 0ull;
    pdl_trigger();  // the contraction's weight copies may start; its activation copies wait for this grid
    pdl_wait();
    const unsigned long long t_dep = a.tl ? gtimer() : 0ull;
    const bool live = b < a.nb && (!a.active || a.active[b] != 0);
    constexpr int IT = 2;  // items of 8 columns per thread: K <= 8 x 2 x 256
    float v[IT][8];
    float ss = 0.0f;
    const uint8_t* er = nullptr;
    if (live && a.tok) {
        const int t = a.tok[b];
        if (t >= 0 && t < a.emb.rows) er = a.emb.w + (long)t * a.emb.stride;
        else dev_error(a.err, DEV_BAD_INDEX);
    }
#pragma unroll
    for (int it = 0; it < IT; it++) {
        const int e = threadIdx.x + XP_THREADS * it, k0 = 8 * e;
#pragma unroll
        for (int c = 0; c < 8; c++) v[it][c] = 0.0f;
        if (!live || k0 >= K) continue;
        if (a.tok) {
            if (er) {
                const uint2 qq = *reinterpret_cast<const uint2*>(er + k0);
                const float d = __half2float(reinterpret_cast<const __half*>(er + K)[k0 >> 5]);
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const uint32_t w = c < 4 ? qq.x : qq.y;
                    v[it][c] = (float)(int8_t)((w >> (8 * (c & 3))) & 0xff) * d;
                }
            }
        } else {
            const float4* xr = reinterpret_cast<const float4*>(a.x + (long)b * a.x_stride + k0);
            const float4 x0 = xr[0], x1 = xr[1];
            v[it][0] = x0.x, v[it][1] = x0.y, v[it][2] = x0.z, v[it][3] = x0.w;
            v[it][4] = x1.x, v[it][5] = x1.y, v[it][6] = x1.z, v[it][7] = x1.w;
        }
        if (a.xadd) {
            // x + (p_0 + … + p_{n-1}), the partials summed in order
            float o[8];
            const float* pa = a.xadd + (long)b * a.n_add * K + k0;
#pragma unroll
            for (int c = 0; c < 8; c++) o[c] = pa[c];
            for (int p = 1; p < a.n_add; p++)
#pragma unroll
                for (int c = 0; c < 8; c++) o[c] += pa[(long)p * K + c];
#pragma unroll
            for (int c = 0; c < 8; c++) v[it][c] += o[c];
        }
        if (a.x_out) {
            float4* xo = reinterpret_cast<float4*>(a.x_out + (long)b * a.x_stride + k0);
            xo[0] = make_float4(v[it][0], v[it][1], v[it][2], v[it][3]);
            xo[1] = make_float4(v[it][4], v[it][5], v[it][6], v[it][7]);
        }
#pragma unroll
        for (int c = 0; c < 8; c++) ss = fmaf(v[it][c], v[it][c], ss);
    }
    float scale = 1.0f;
    if (a.nw) {
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = 0; w < XP_THREADS / 32; w++) tot += red[w];
        scale = 1.0f / sqrtf(tot / (float)K + a.eps);
    }
#pragma unroll
    for (int it = 0; it < IT; it++) {
        const int e = threadIdx.x + XP_THREADS * it, k0 = 8 * e;
        if (k0 >= K) continue;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int c = 0; c < 8; c += 2) {
            float y0 = v[it][c], y1 = v[it][c + 1];
            if (a.nw && live) {
                y0 = y0 * scale * a.nw[k0 + c];
                y1 = y1 * scale * a.nw[k0 + c + 1];
            }
            const __half h0 = __float2half_rn(y0), h1 = __float2half_rn(y1);
            const __half l0 = __float2half_rn(y0 - __half2float(h0)), l1 = __float2half_rn(y1 - __half2float(h1));
            const __half2 hh = __halves2half2(h0, h1), ll = __halves2half2(l0, l1);
            hi[c >> 1] = *reinterpret_cast<const uint32_t*>(&hh);
            lo[c >> 1] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        *reinterpret_cast<uint4*>(xg + x16_offset(n, k0)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(xg + x16_offset(BG_SLOTS + n, k0)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if (a.tl) {  // (uniform)
        __syncthreads();
        if (threadIdx.x == 0) tl_record(a.tl, t_start, t_dep);
    }
}

// ---- host ----------------------------------------------------------------------------------------------------------------
bool bgemm_shape_ok(int rows, int cols) { return rows >= 1 && cols >= 256 && cols % 256 == 0 && cols <= 4096; }

int bgemm_grid(int num_sms, int rows, int ksplit) {
    return std::max(1, std::min((rows + BG_M - 1) / BG_M * ksplit, num_sms));
}

int bgemm_ksplit(int num_sms, int rows, int cols) {
    const int tiles = (rows + BG_M - 1) / BG_M, nkc = cols / BG_KC;
    return std::max(1, std::min(nkc, num_sms / tiles));
}

size_t bgemm_part_floats(int rows, int ksplit) {
    return ksplit > 1 ? (size_t)((rows + BG_M - 1) / BG_M) * ksplit * BG_SLOTS * BG_M : 0;
}

int bgemm_tickets(int rows) { return (rows + BG_M - 1) / BG_M; }

size_t bgemm_tiled_bytes(int rows, int cols) {
    return (size_t)((rows + BG_M - 1) / BG_M) * (cols / BG_KC) * BG_TILE_BYTES;
}

// the tile-major copy (see BG_TILE_BYTES): one CTA per block, 16-byte pieces of quants swizzled, then the scales
__global__ void __launch_bounds__(256) k_tile_q8_0(QMat w, uint8_t* __restrict__ out) {
    const int nkc = w.cols / BG_KC, t = blockIdx.x / nkc, c = blockIdx.x % nkc;
    uint8_t* o = out + (size_t)blockIdx.x * BG_TILE_BYTES;
    for (int i = threadIdx.x; i < BG_M * 8; i += blockDim.x) {
        const int r = i >> 3, pc = i & 7, row = t * BG_M + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < w.rows) v = *reinterpret_cast<const uint4*>(w.w + (size_t)row * w.stride + c * BG_KC + pc * 16);
        *reinterpret_cast<uint4*>(o + r * 128 + ((pc ^ (r & 7)) << 4)) = v;
    }
    for (int r = threadIdx.x; r < BG_M; r += blockDim.x) {
        const int row = t * BG_M + r;
        uint2 v = make_uint2(0u, 0u);  // the 4 f16 scales of the chunk's 4 blocks (8-byte aligned: cols % 256 == 0)
        if (row < w.rows) v = *reinterpret_cast<const uint2*>(w.w + (size_t)row * w.stride + w.cols + c * 8);
        *reinterpret_cast<uint2*>(o + BG_M * 128 + r * 8) = v;
    }
}

void launch_tile_q8_0(cudaStream_t st, const QMat& w, uint8_t* out) {
    const int blocks = (w.rows + BG_M - 1) / BG_M * (w.cols / BG_KC);
    k_tile_q8_0<<<blocks, 256, 0, st>>>(w, out);
}

// the instances launched: (mode, operand built in the kernel)
using BgKernel = void (*)(BgArgs, const uint8_t*, int, int);
static BgKernel bg_kernel(int mode, bool xn, int ng) {
    if (ng == 3) {
        if (xn) return nullptr;
        return mode == MV_ADD ? k_bgemm<MV_ADD, false, 3> : mode == MV_SWIGLU ? k_bgemm<MV_SWIGLU, false, 3>
             : mode == MV_STORE ? k_bgemm<MV_STORE, false, 3> : nullptr;
    }
    if (ng == 2) {
        if (xn) return nullptr;
        return mode == MV_ADD ? k_bgemm<MV_ADD, false, 2> : mode == MV_SWIGLU ? k_bgemm<MV_SWIGLU, false, 2>
             : mode == MV_STORE ? k_bgemm<MV_STORE, false, 2> : nullptr;
    }
    switch (mode) {
        case MV_ADD: return xn ? nullptr : k_bgemm<MV_ADD, false>;
        case MV_SWIGLU: return xn ? k_bgemm<MV_SWIGLU, true> : k_bgemm<MV_SWIGLU, false>;
        case MV_LMHEAD: return xn ? nullptr : k_bgemm<MV_LMHEAD, false>;
        default: return xn ? k_bgemm<MV_STORE, true> : k_bgemm<MV_STORE, false>;
    }
}
static const BgKernel BG_ALL[] = {k_bgemm<MV_STORE, false>,    k_bgemm<MV_STORE, true>,     k_bgemm<MV_ADD, false>,
                                  k_bgemm<MV_SWIGLU, false>,   k_bgemm<MV_SWIGLU, true>,    k_bgemm<MV_LMHEAD, false>,
                                  k_bgemm<MV_STORE, false, 2>, k_bgemm<MV_ADD, false, 2>, k_bgemm<MV_SWIGLU, false, 2>,
                                  k_bgemm<MV_STORE, false, 3>, k_bgemm<MV_ADD, false, 3>, k_bgemm<MV_SWIGLU, false, 3>};

// the largest static shared memory of the instances (the dynamic budget is sized against it)
static int bg_static_smem() {
    static int bytes = -1;
    if (bytes < 0) {
        int b = (int)sizeof(BgShared) + 64;
        for (BgKernel k : BG_ALL) {
            cudaFuncAttributes fa;
            if (cudaFuncGetAttributes(&fa, k) == cudaSuccess) b = std::max(b, (int)fa.sharedSizeBytes);
        }
        bytes = b;
    }
    return bytes;
}

// shared memory: ns copy stages (weights + ng activation chunks each) and na operand buffers (+ the 1024-B alignment
// slack): as many operand buffers as fit beside 3 stages (2 for two groups), then as many stages as fit
static void bg_ring(int& ns, int& na, int& fixed, int ng = 1) {
    const int stage = (int)BG_WTILE + ng * (int)BG_CHUNK_BYTES;
    const int room = BG_SMEM_OPTIN - bg_static_smem() - 1024;
    na = std::max(2, std::min(BG_NA, (room - (ng == 1 ? 3 : 2) * stage) / (int)BG_ABUF));
    fixed = na * (int)BG_ABUF + 1024;
    ns = std::max(1, std::min(BG_MAX_NS, (BG_SMEM_OPTIN - bg_static_smem() - fixed) / stage));
}

bool bgemm_norm_in_ok(int num_sms, int rows, int cols, int ksplit) {
    int ns, na, fixed;
    bg_ring(ns, na, fixed);
    const int items = (rows + BG_M - 1) / BG_M * ksplit, nkc = cols / BG_KC;
    return bgemm_shape_ok(rows, cols) && items <= bgemm_grid(num_sms, rows, ksplit) && (nkc + ksplit - 1) / ksplit <= ns;
}

void launch_bgemm(cudaStream_t st, const BgArgs& a, const BgMaps& m, int num_sms, bool pdl) {
    static PerDeviceOnce once;
    once([] {
        for (BgKernel k : BG_ALL)
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, BG_SMEM_OPTIN - bg_static_smem());
    });
    // two groups of 32 rows per CTA for unsplit launches over more than one group (the long prefill): each weight
    // piece dequantised once for both
    const int groups = (a.nb + BG_SLOTS - 1) / BG_SLOTS;
    const bool multi = a.ksplit == 1 && !a.xn && a.mode != MV_LMHEAD;
    const int ng = (multi && a.wide && groups >= 3) ? 3 : (multi && groups >= 2) ? 2 : 1;
    int ns, na, fixed;
    bg_ring(ns, na, fixed, ng);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)bgemm_grid(num_sms, a.w.rows, a.ksplit), (unsigned)((groups + ng - 1) / ng), 1);
    cfg.blockDim = dim3(BG_THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)fixed + (size_t)ns * ((size_t)BG_WTILE + (size_t)ng * BG_CHUNK_BYTES);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const BgKernel k = bg_kernel(a.mode, a.xn != nullptr, ng);
    if (!k) {  // (an in-kernel operand for a mode that has no such instance: a caller's error, nothing launched)
        fprintf(stderr, "launch_bgemm: mode %d has no instance with the operand built in the kernel\n", a.mode);
        return;
    }
    cudaLaunchKernelEx(&cfg, k, a, m.tiles, ns, na);
}

void launch_xprep(cudaStream_t st, const PrepArgs& a, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.nb + BG_SLOTS - 1) / BG_SLOTS * BG_SLOTS), 1, 1);
    cfg.blockDim = dim3(XP_THREADS, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, k_xprep, a);
}

}  // namespace ocr
